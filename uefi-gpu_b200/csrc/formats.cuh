// formats.cuh -- GGUF block formats on the device: one 32-element "unit" at a time.
//
// A unit is 32 consecutive weights of a row: one Q8_0 block, or one eighth of a Q4_K / Q3_K
// 256-element super-block.  Every kernel that multiplies quantised weights by a Q8_1
// activation calls unit_dot<KIND>(), which returns the exact int32 block dot (the value the
// reference's CPU check forms, gpu_prefill.rs:111-115) and the fp32 multiplier that turns it
// into the block's contribution to y.  Weights are read from shared memory (staged there by
// bulk copies in the GGUF byte layout, unchanged).
#pragma once
#include "common.cuh"

namespace ugb {

// Block geometry per GGML type id.
template <int KIND> struct Fmt;
template <> struct Fmt<UGB_Q8_0> {
  static constexpr int kElems = 32, kBytes = 34;       // frontier_core.rs:147
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
  int q[8];       // Q8_0: int8; Q4_K: [0,15]; Q3_K: [0,7] (biased by +4)
  float d;        // Q8_0: block scale; Q4_K: d*sc; Q3_K: super-block d
  float dm;       // Q4_K: dmin*m; unused otherwise
  int sc_lo, sc_hi;  // Q3_K: signed 6-bit scales of the two 16-element halves
};

// Q8_0 block at a 2-byte aligned shared address: fp16 d then 32 int8 (frontier_core.rs:172).
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

// Integer block dot of one unit (the value the oracle's orc_block_dots returns).
template <int KIND>
__device__ __forceinline__ int unit_isum(const WUnit &w, const XUnit &x) {
  if constexpr (KIND == UGB_Q3_K) {
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
    return w.sc_lo * (lo - 4 * xlo) + w.sc_hi * (hi - 4 * xhi);
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
  } else {
    load_wunit_q3_k(seg + 110u * (u >> 3), u & 7, w);
  }
}

}  // namespace ugb
