// formats.cuh -- GGUF block formats on the device: one 32-element "unit" at a time.
//
// A unit is 32 consecutive weights of a row: one Q8_0 / IQ4_NL block, or one eighth of a Q4_K /
// Q3_K / Q6_K / IQ4_XS / IQ3_XXS 256-element super-block.  Every kernel that multiplies
// quantised weights by a Q8_1 activation calls unit_isum<KIND>(), the exact int32 block dot (the
// value the reference's CPU check forms, gpu_prefill.rs:111-115), and unit_term<KIND>(), the
// fp32 contribution of that dot to y.  Weights are read from shared memory (staged there by
// bulk copies in the GGUF byte layout, unchanged).
#pragma once
#include "common.cuh"

namespace ugb {

// IQ3_XXS grid: 256 entries of four unsigned magnitudes (ggml's iq3xxs_grid, the table the
// reference passes to its kernels as `grid`, frontier_tables.rs).  Read through L1: lanes of a
// warp look up different entries.
__device__ const uint32_t kIq3Grid[256] = {
#include "iq3_grid.inc"
};

// Block geometry per GGML type id.
template <int KIND> struct Fmt;
template <> struct Fmt<UGB_Q8_0> {
  static constexpr int kElems = 32, kBytes = 34;       // frontier_core.rs:54
  static constexpr int kUnitsPerBlock = 1;
  static constexpr bool kNeedsSum = false;
};
template <> struct Fmt<UGB_Q4_K> {
  static constexpr int kElems = 256, kBytes = 144;     // ggml block_q4_K
  static constexpr int kUnitsPerBlock = 8;
  static constexpr bool kNeedsSum = true;              // dmin * m * sum(q8) term
};
template <> struct Fmt<UGB_Q3_K> {
  static constexpr int kElems = 256, kBytes = 110;     // ggml block_q3_K
  static constexpr int kUnitsPerBlock = 8;
  static constexpr bool kNeedsSum = false;
};
// The reference's other formats (frontier_core.rs:54-55 sizes, :80-101 bit maps).
template <> struct Fmt<UGB_Q6_K> {
  static constexpr int kElems = 256, kBytes = 210;
  static constexpr int kUnitsPerBlock = 8;
  static constexpr bool kNeedsSum = false;
};
template <> struct Fmt<UGB_IQ3_XXS> {
  static constexpr int kElems = 256, kBytes = 98;
  static constexpr int kUnitsPerBlock = 8;
  static constexpr bool kNeedsSum = false;
};
template <> struct Fmt<UGB_IQ4_NL> {
  static constexpr int kElems = 32, kBytes = 18;
  static constexpr int kUnitsPerBlock = 1;
  static constexpr bool kNeedsSum = false;
};
template <> struct Fmt<UGB_IQ4_XS> {
  static constexpr int kElems = 256, kBytes = 136;
  static constexpr int kUnitsPerBlock = 8;
  static constexpr bool kNeedsSum = false;
};

// The activation side of one unit for one vector: 32 int8 quants (8 words), the block scale
// d_x and the block sum s = sum(q) (Q8_1).
struct XUnit {
  int q[8];
  float d;
  int s;
};

__device__ __forceinline__ void load_xunit(uint32_t q_addr, uint32_t d_addr, uint32_t s_addr,
                                           bool need_sum, XUnit &x) {
  const uint4 a = lds128(q_addr), b = lds128(q_addr + 16);
  x.q[0] = a.x; x.q[1] = a.y; x.q[2] = a.z; x.q[3] = a.w;
  x.q[4] = b.x; x.q[5] = b.y; x.q[6] = b.z; x.q[7] = b.w;
  x.d = __uint_as_float(lds32(d_addr));
  x.s = need_sum ? static_cast<int>(lds32(s_addr)) : 0;
}

// Decoded weight side of one unit, independent of the activation: the unpacked quants as
// int8x4 words plus the per-unit scale constants.
struct WUnit {
  int q[8];       // Q8_0, IQ4_*, IQ3_XXS: int8 values; Q4_K: [0,15]; Q3_K: [0,7] (biased by +4);
                  // Q6_K: [0,63] (biased by +32)
  float d;        // Q8_0 / IQ4_NL: block scale; Q4_K: d*sc; Q3_K / Q6_K: super-block d;
                  // IQ4_XS: d*(sc-32); IQ3_XXS: d*(0.5+s)*0.5
  float dm;       // Q4_K: dmin*m; unused otherwise
  int sc_lo, sc_hi;  // Q3_K / Q6_K: signed scales of the two 16-element halves
};

// Q8_0 block at a 2-byte aligned shared address: fp16 d then 32 int8 (frontier_core.rs:79).
// One 40-byte window (five 64-bit loads) holds the whole 34-byte block at any even offset.
__device__ __forceinline__ void load_wunit_q8_0(uint32_t blk, WUnit &w) {
  uint32_t s[9];
  lds_window9(blk, s);
  const uint32_t sh = (blk & 3u) * 8u;  // 0 or 16: where d starts inside s[0]
#pragma unroll
  for (int i = 0; i < 8; ++i) w.q[i] = static_cast<int>(__funnelshift_rc(s[i], s[i + 1], sh + 16));
  w.d = half_bits_to_float(s[0] >> sh);
  w.dm = 0.f;
  w.sc_lo = w.sc_hi = 0;
}

// Q4_K sub-block j (0..7) of a 16-byte aligned super-block: {fp16 d, fp16 dmin, u8
// scales[12], u8 qs[128]}.  Quants of sub-block j are nibble (j&1) of qs[32*(j/2) ...].
// kBranchFree picks the select form of the scale lookup (faster where the lanes of a warp hold
// different sub-blocks, as in the batch-1 kernels: c4 batch 1 +6%) or the branch form (1%
// faster in the batched stream kernel).
template <bool kBranchFree = true>
__device__ __forceinline__ void load_wunit_q4_k(uint32_t sb, int j, WUnit &w) {
  const uint32_t dd = lds32(sb);
  const uint32_t s0 = lds32(sb + 4), s1 = lds32(sb + 8), s2 = lds32(sb + 12);
  // scales bytes: b[0..3] = s0, b[4..7] = s1, b[8..11] = s2 (get_scale_min_k4)
  int sc, mn;
  if constexpr (kBranchFree) {
    // with jl = j mod 4: b0 = scales[jl], b1 = scales[jl + 4], b2 = scales[jl + 8]
    const uint32_t jl = static_cast<uint32_t>(j & 3);
    const uint32_t b0 = (s0 >> (8 * jl)) & 0xff, b1 = (s1 >> (8 * jl)) & 0xff, b2 = (s2 >> (8 * jl)) & 0xff;
    const bool up = j >= 4;
    sc = static_cast<int>(up ? (b2 & 0x0f) | ((b0 >> 6) << 4) : (b0 & 63));
    mn = static_cast<int>(up ? (b2 >> 4) | ((b1 >> 6) << 4) : (b1 & 63));
  } else if (j < 4) {
    sc = (s0 >> (8 * j)) & 63;
    mn = (s1 >> (8 * j)) & 63;
  } else {
    const int jj = j - 4;
    const uint32_t bj4 = (s2 >> (8 * jj)) & 0xff;   // scales[j+4]
    const uint32_t bjm4 = (s0 >> (8 * jj)) & 0xff;  // scales[j-4]
    const uint32_t bj = (s1 >> (8 * jj)) & 0xff;    // scales[j]
    sc = (bj4 & 0x0f) | ((bjm4 >> 6) << 4);
    mn = (bj4 >> 4) | ((bj >> 6) << 4);
  }
  const uint32_t qa = sb + 16 + 32 * (j >> 1);
  const uint4 a = lds128(qa), b = lds128(qa + 16);
  const uint32_t sh = 4 * (j & 1);
  const uint32_t raw[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
  for (int i = 0; i < 8; ++i) w.q[i] = static_cast<int>((raw[i] >> sh) & 0x0f0f0f0fu);
  w.d = half_bits_to_float(dd) * static_cast<float>(sc);
  w.dm = half_bits_to_float(dd >> 16) * static_cast<float>(mn);
  w.sc_lo = w.sc_hi = 0;
}

// Q3_K 32-element block c (0..7) of a 2-byte aligned super-block: {u8 hmask[32], u8 qs[64],
// u8 scales[12], fp16 d}.  Element e of block c: low bits (qs[32*(c/4)+e] >> 2*(c%4)) & 3,
// high bit (hmask[e] >> c) & 1; value = low + 4*high - 4.  Stored biased (+4) in [0,7].
__device__ __forceinline__ void load_wunit_q3_k(uint32_t sb, int c, WUnit &w) {
  uint32_t hm[8], qw[8];
  lds_words8_u2(sb, hm);
  lds_words8_u2(sb + 32 + 32 * (c >> 2), qw);
  const uint32_t sh = 2 * (c & 3);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t lo = (qw[i] >> sh) & 0x03030303u;
    const uint32_t hi = ((hm[i] >> c) & 0x01010101u) << 2;
    w.q[i] = static_cast<int>(lo | hi);
  }
  const int j0 = 2 * c, j1 = 2 * c + 1;
  const uint32_t scb = sb + 96;
  const int lo0 = (lds8(scb + (j0 & 7)) >> (4 * (j0 >> 3))) & 15;
  const int hi0 = (lds8(scb + 8 + (j0 & 3)) >> (2 * (j0 >> 2))) & 3;
  const int lo1 = (lds8(scb + (j1 & 7)) >> (4 * (j1 >> 3))) & 15;
  const int hi1 = (lds8(scb + 8 + (j1 & 3)) >> (2 * (j1 >> 2))) & 3;
  w.sc_lo = (lo0 | (hi0 << 4)) - 32;
  w.sc_hi = (lo1 | (hi1 << 4)) - 32;
  w.d = half_bits_to_float(lds16_u2(sb + 108));
  w.dm = 0.f;
}

// IQ4 non-linear code book (frontier_core.rs:68) as four words of int8 bytes, entry i in byte
// i % 4 of word i / 4.
__host__ __device__ constexpr uint32_t iq4_word(int w) {
  constexpr int kV[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};
  return (static_cast<uint32_t>(kV[4 * w] & 0xff)) | (static_cast<uint32_t>(kV[4 * w + 1] & 0xff) << 8) |
         (static_cast<uint32_t>(kV[4 * w + 2] & 0xff) << 16) | (static_cast<uint32_t>(kV[4 * w + 3] & 0xff) << 24);
}

// Code-book values of four 4-bit indices, given as the low 16 bits of `sel` (index i in bits
// 4i..4i+3), as one int8x4 word: two byte permutes over the two halves of the book, and a third
// that takes each byte from the half its index's top bit names.
__device__ __forceinline__ int iq4_lookup4(uint32_t sel) {
  const uint32_t s3 = sel & 0x7777u;
  const uint32_t lo = __byte_perm(iq4_word(0), iq4_word(1), s3);
  const uint32_t hi = __byte_perm(iq4_word(2), iq4_word(3), s3);
  return static_cast<int>(__byte_perm(lo, hi, 0x3210u | ((sel >> 1) & 0x4444u)));
}

// 16 packed quant bytes (elements e in the low nibble of byte e, elements 16 + e in the high
// nibble) -> the unit's 32 code-book values, as IQ4_NL / IQ4_XS store them (frontier_core.rs:
// 80-81, 86).
__device__ __forceinline__ void iq4_unpack(const uint32_t (&qs)[4], WUnit &w) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t v = qs[i];
    const uint32_t lo = (v & 0xfu) | ((v >> 4) & 0xf0u) | ((v >> 8) & 0xf00u) | ((v >> 12) & 0xf000u);
    const uint32_t hv = v >> 4;
    const uint32_t hi = (hv & 0xfu) | ((hv >> 4) & 0xf0u) | ((hv >> 8) & 0xf00u) | ((hv >> 12) & 0xf000u);
    w.q[i] = iq4_lookup4(lo);
    w.q[4 + i] = iq4_lookup4(hi);
  }
}

// IQ4_NL block at a 2-byte aligned address: fp16 d then 16 bytes of nibbles (frontier_core.rs:
// 80-82).  Six words from the 4-byte aligned address below hold it at either offset.
__device__ __forceinline__ void load_wunit_iq4_nl(uint32_t blk, WUnit &w) {
  const uint32_t a4 = blk & ~3u;
  uint32_t s[6];
#pragma unroll
  for (int i = 0; i < 6; ++i) s[i] = lds32(a4 + 4u * i);
  const uint32_t sh = (blk & 3u) * 8u;  // 0 or 16: where d starts inside s[0]
  uint32_t qs[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) qs[i] = __funnelshift_rc(s[i], s[i + 1], sh + 16);
  iq4_unpack(qs, w);
  w.d = half_bits_to_float(s[0] >> sh);
  w.dm = 0.f;
  w.sc_lo = w.sc_hi = 0;
}

// IQ4_XS sub-block j (0..7) of an 8-byte aligned super-block: {fp16 d, u16 scales_h, u8
// scales_l[4], u8 qs[128]}; the 6-bit scale of sub-block j is nibble j%2 of scales_l[j/2] with
// bits 2j..2j+1 of scales_h on top, minus 32 (frontier_core.rs:83-87).
__device__ __forceinline__ void load_wunit_iq4_xs(uint32_t sb, int j, WUnit &w) {
  const uint32_t hd = lds32(sb), sl = lds32(sb + 4);
  const uint2 a = lds64(sb + 8 + 16 * j), b = lds64(sb + 16 + 16 * j);
  const uint32_t qs[4] = {a.x, a.y, b.x, b.y};
  iq4_unpack(qs, w);
  const int sc = static_cast<int>(((sl >> (4 * j)) & 15u) | (((hd >> (16 + 2 * j)) & 3u) << 4));
  w.d = half_bits_to_float(hd) * static_cast<float>(sc - 32);
  w.dm = 0.f;
  w.sc_lo = w.sc_hi = 0;
}

// Q6_K 32-element unit u (0..7) of a 2-byte aligned super-block {u8 ql[128], u8 qh[64], i8
// scales[16], fp16 d} (frontier_core.rs:88-93): with half h = u/4 and group g = u%4, element l
// has low bits nibble g/2 of ql[64h + 32(g%2) + l], high bits (qh[32h + l] >> 2g) & 3, value
// (low | high << 4) - 32, stored biased (+32) in [0,63]; its scale is scales[8h + 2g + l/16].
__device__ __forceinline__ void load_wunit_q6_k(uint32_t sb, int u, WUnit &w) {
  const int h = u >> 2, g = u & 3;
  uint32_t ql[8], qh[8];
  lds_words8_u2(sb + 64 * h + 32 * (g & 1), ql);
  lds_words8_u2(sb + 128 + 32 * h, qh);
  const uint32_t sl = 4 * (g >> 1), shh = 2 * g;
#pragma unroll
  for (int i = 0; i < 8; ++i)
    w.q[i] = static_cast<int>(((ql[i] >> sl) & 0x0f0f0f0fu) | (((qh[i] >> shh) & 0x03030303u) << 4));
  const uint32_t scw = lds16_u2(sb + 192 + 8 * h + 2 * g);
  w.sc_lo = static_cast<int>(static_cast<int8_t>(scw & 0xff));
  w.sc_hi = static_cast<int>(static_cast<int8_t>(scw >> 8));
  w.d = half_bits_to_float(lds16_u2(sb + 208));
  w.dm = 0.f;
}

// Four grid magnitudes with the signs of 4 bits applied (bit i negates byte i).
__device__ __forceinline__ int signed_bytes(uint32_t mag, uint32_t bits4) {
  const uint32_t m = ((bits4 * 0x00204081u) & 0x01010101u) * 0xffu;
  return static_cast<int>(__vsub4(mag ^ m, m));
}

// IQ3_XXS sub-block j (0..7) of a 2-byte aligned super-block {fp16 d, u8 grid index[64], u32
// aux[8]} (frontier_core.rs:94-101): group g (0..3) of eight elements takes grid entries
// index[8j + 2g] and index[8j + 2g + 1], and 7 sign bits (aux[j] >> 7g) & 127 completed to
// even parity by an eighth; the sub-block scale is d * (0.5 + (aux[j] >> 28)) * 0.5.
__device__ __forceinline__ void load_wunit_iq3_xxs(uint32_t sb, int j, WUnit &w) {
  const uint32_t a = sb + 66 + 4 * j;
  const uint32_t aux = lds16_u2(a) | (lds16_u2(a + 2) << 16);
  const uint32_t ix = sb + 2 + 8 * j;
  const uint32_t i01 = lds16_u2(ix) | (lds16_u2(ix + 2) << 16);
  const uint32_t i23 = lds16_u2(ix + 4) | (lds16_u2(ix + 6) << 16);
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const uint32_t s7 = (aux >> (7 * g)) & 127u;
    const uint32_t s8 = s7 | ((__popc(s7) & 1u) << 7);
    const uint32_t idx = g < 2 ? i01 : i23;
    const uint32_t e0 = (idx >> (16 * (g & 1))) & 0xffu, e1 = (idx >> (16 * (g & 1) + 8)) & 0xffu;
    w.q[2 * g] = signed_bytes(__ldg(&kIq3Grid[e0]), s8 & 15u);
    w.q[2 * g + 1] = signed_bytes(__ldg(&kIq3Grid[e1]), s8 >> 4);
  }
  w.d = half_bits_to_float(lds16_u2(sb)) * (0.5f + static_cast<float>(aux >> 28)) * 0.5f;
  w.dm = 0.f;
  w.sc_lo = w.sc_hi = 0;
}

// Integer block dot of one unit (the value the oracle's orc_block_dots returns).
template <int KIND>
__device__ __forceinline__ int unit_isum(const WUnit &w, const XUnit &x) {
  if constexpr (KIND == UGB_Q3_K || KIND == UGB_Q6_K) {
    constexpr int kBias = KIND == UGB_Q3_K ? 4 : 32;
    int lo = 0, hi = 0, xlo = 0, xhi = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      lo = dp4a(w.q[i], x.q[i], lo);
      xlo = dp4a(0x01010101, x.q[i], xlo);
    }
#pragma unroll
    for (int i = 4; i < 8; ++i) {
      hi = dp4a(w.q[i], x.q[i], hi);
      xhi = dp4a(0x01010101, x.q[i], xhi);
    }
    return w.sc_lo * (lo - kBias * xlo) + w.sc_hi * (hi - kBias * xhi);
  } else {
    int acc = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) acc = dp4a(w.q[i], x.q[i], acc);
    return acc;
  }
}

// fp32 contribution of one unit given its integer dot (orc_matvec's per-block formula).
template <int KIND>
__device__ __forceinline__ float unit_term(const WUnit &w, const XUnit &x, int isum) {
  if constexpr (KIND == UGB_Q8_0) {
    return static_cast<float>(isum) * (w.d * x.d);
  } else if constexpr (KIND == UGB_Q4_K) {
    return x.d * (w.d * static_cast<float>(isum) - w.dm * static_cast<float>(x.s));
  } else {
    return static_cast<float>(isum) * (w.d * x.d);
  }
}

// Load the weight side of unit u of a row segment starting at shared address `seg`.
template <int KIND, bool kBranchFree = true>
__device__ __forceinline__ void load_wunit(uint32_t seg, int u, WUnit &w) {
  if constexpr (KIND == UGB_Q8_0) {
    load_wunit_q8_0(seg + 34u * u, w);
  } else if constexpr (KIND == UGB_Q4_K) {
    load_wunit_q4_k<kBranchFree>(seg + 144u * (u >> 3), u & 7, w);
  } else if constexpr (KIND == UGB_Q3_K) {
    load_wunit_q3_k(seg + 110u * (u >> 3), u & 7, w);
  } else if constexpr (KIND == UGB_Q6_K) {
    load_wunit_q6_k(seg + 210u * (u >> 3), u & 7, w);
  } else if constexpr (KIND == UGB_IQ3_XXS) {
    load_wunit_iq3_xxs(seg + 98u * (u >> 3), u & 7, w);
  } else if constexpr (KIND == UGB_IQ4_NL) {
    load_wunit_iq4_nl(seg + 18u * u, w);
  } else {
    static_assert(KIND == UGB_IQ4_XS, "unknown kind");
    load_wunit_iq4_xs(seg + 136u * (u >> 3), u & 7, w);
  }
}

}  // namespace ugb
