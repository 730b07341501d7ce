// mv_tc.cu -- batched Q4_K / Q8_0 decode matvec on the tensor cores (tcgen05.mma.kind::i8).
//
// Replaces the batch form of linear_dp4a / gateup_dp4a (gpu_dp4a.cu:32-64) for Q4_K and Q8_0
// weights and 5..8 activation vectors.  The arithmetic is the one every matvec of the library
// forms: per 32-element unit b of a row, the exact int32 dot I_b[t] = sum q_w * q_x (Q4_K
// nibbles 0..15 or Q8_0 int8 values, against the Q8_1 activation's int8 values), then in fp32
//
//     Q4_K: y[t][r] += xd[t][b] * (d*sc_b * I_b[t] - dmin*m_b * xs[t][b])
//     Q8_0: y[t][r] += I_b[t] * (d_b * xd[t][b])
//
// (unit_term in formats.cuh).  What changes is where the integer dots come from.  With a batch,
// the dp4a kernels spend most of their instructions unpacking quants and scales once per weight
// and vector; here the quants of 128 rows x 32 elements are unpacked once into the A operand
// (M = 128) of one tcgen05.mma against the vectors (N = 16), and the tensor core forms all
// eight dots of the unit.
//
// One CTA per SM, persistent over units (128-row tile, K chunk of 256-element super-blocks;
// a Q8_0 "super-block" is 8 consecutive blocks, 272 bytes):
//   * warp 8 streams the raw GGUF bytes of the tile's 128 rows, one super-block per row and
//     stage, into a 4-deep (Q4_K) or 3-deep (Q8_0) ring: one 2-D tensor copy (super-block x 128
//     rows) per stage.  Separate 1-D copies of each row's bytes took ~4.3 us to issue per 36 KB
//     stage, three times the workers' time for it;
//   * warps 0-3 and 4-7 form two groups that take alternate super-blocks of the unit.  Thread i
//     of a group owns row i (its TMEM lane): it decodes the row's scales, writes its unpacked
//     quants into the group's A buffer (half a super-block = 4 units per MMA step; 3 buffers for
//     Q4_K, 2 for Q8_0, whose stages are larger), and rescales the int32 dots of an earlier step
//     from tensor memory into 8 fp32 sums;
//   * warp 9 issues the MMAs.  A unit's eight 8-vector dots go to 16 columns as block pairs:
//     block 2p against B rows 0-7 (rows 8-15 read a zero region), then block 2p+1 accumulated
//     against B rows 8-15 (rows 0-7 zero), so no column is padding;
//   * the two groups' sums meet in shared memory in a fixed order.  Tiles with too few rows
//     for the SMs are also split along K: chunk partials go to the context's workspace and the
//     last CTA of a tile (a ticket per tile) adds them in chunk order.  Results are therefore
//     deterministic run to run.
// The activation vectors of the CTA's K chunk are staged once per CTA in the canonical K-major
// layout (B operand), with their scales and sums as fp32.
#include <algorithm>
#include <mutex>

#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "internal.hpp"
#include "tcgen05.cuh"

namespace ugb {
namespace {

constexpr int kTcThreads = 320;         // 8 worker warps, producer, MMA
constexpr int kTcMaxCs = 16;            // super-blocks per K chunk
// shared-memory map (the A buffers and the ring depend on the kind, TcFmt)
constexpr int kOffZlo = 256;                            // 256 zero bytes (B rows 0-7 of odd blocks)
constexpr int kOffXb = kOffZlo + 256;                   // [cs*8 units][256 B]: 8 vectors x 32 int8
constexpr int kOffZhi = kOffXb + kTcMaxCs * 8 * 256;    // 256 zero bytes (B rows 8-15 of even blocks)
constexpr int kOffXd = kOffZhi + 256;                   // [cs*8][8] f32 activation scales
constexpr int kOffXs = kOffXd + kTcMaxCs * 8 * 8 * 4;   // [cs*8][8] f32 activation sums
constexpr int kOffRed = kOffXs + kTcMaxCs * 8 * 8 * 4;  // [8][128] f32 group-1 sums
constexpr int kOffA = kOffRed + 8 * 128 * 4;            // [group][buf][4 units][4096 B]
static_assert(kOffA % 128 == 0, "operand alignment");
// D s32, A s8, B s8, both K-major, N = 16, M = 128.
constexpr uint32_t kTcIdesc = (2u << 4) | (1u << 7) | (1u << 10) | (2u << 17) | (8u << 24);
constexpr uint32_t kTcTmemCols = 256;   // [group][buf] x 32 columns (at most 192 used)

// Per kind: bytes of a 256-element super-block (a stage row), ring stages, A / TMEM buffers per
// group (the rescale trails the unpack by kBufs - 1 steps).
template <int KIND>
struct TcFmt;
template <>
struct TcFmt<UGB_Q4_K> {
  static constexpr int kSbBytes = 144, kStages = 4, kBufs = 3;
};
template <>
struct TcFmt<UGB_Q8_0> {
  static constexpr int kSbBytes = 272, kStages = 3, kBufs = 2;
};
template <int KIND>
struct TcGeo {
  using F = TcFmt<KIND>;
  static constexpr int kStageBytes = 128 * F::kSbBytes;
  static constexpr int kOffRing = kOffA + 2 * F::kBufs * 4 * 4096;
  static constexpr int kSmem = kOffRing + F::kStages * kStageBytes;
  static_assert(kOffRing % 128 == 0 && kStageBytes % 128 == 0, "tensor-copy alignment");
  static_assert(kSmem <= 227 * 1024, "one CTA per SM");
};

struct TcParams {
  CUtensorMap tmap[kMaxMatvecSegs];  // matrix i as [rows][row_bytes / 4] words, box (super-block) x 128
  int seg_row0[kMaxMatvecSegs + 1];  // rows of matrix i: [seg_row0[i], seg_row0[i + 1])
  int nseg;
  uint64_t row_bytes;
  int m, k, ns;           // rows, columns, super-blocks per row
  int cs, nch, tiles;     // super-blocks per chunk, chunks, 128-row tiles
  int nb;                 // activation vectors (<= 8; the rest of B is zero)
  const uint8_t *xq;      // vector t: quants xq + t * k, scales xd + t * nbp, sums xs + t * nbp
  const float *xd;
  const int *xs;
  int nbp;
  float *y;               // y[t * ldy + r]
  int64_t ldy;
  float *part;            // [tiles][nch][8][128] chunk partials (nch > 1)
  uint32_t *tickets;      // [tiles], zero between launches
  uint32_t *status;
};

__device__ __forceinline__ void sts128(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ void named_sync(uint32_t id, uint32_t n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}
// 2-D tensor copy of box (x, y) of the map into shared memory, completing on an mbarrier.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, int x, int y, uint32_t bar,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// K-major no-swizzle shared-memory descriptor with explicit strides (bytes): LBO between the two
// 16-byte K halves of a core-matrix pair, SBO between 8-row groups.
__device__ __forceinline__ uint64_t tc_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16) |
         (static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}

// Super-blocks of the unit's chunk and how many group g takes (alternate ones, group 0 first).
__device__ __forceinline__ int unit_sbs(const TcParams &p, int chunk) { return min(p.cs, p.ns - chunk * p.cs); }
__device__ __forceinline__ int group_sbs(int S, int g) { return (S - g + 1) / 2; }

template <int KIND>
__global__ void __launch_bounds__(kTcThreads, 1) mv_tc_kernel(const __grid_constant__ TcParams p) {
  using F = TcFmt<KIND>;
  constexpr int kTcStages = F::kStages, kTcBufs = F::kBufs, kSbBytes = F::kSbBytes, kRowStride = kSbBytes;
  constexpr int kStageBytes = TcGeo<KIND>::kStageBytes, kOffRing = TcGeo<KIND>::kOffRing;
  extern __shared__ __align__(1024) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t base = smem_u32(smem);
  // control block: full[<=4], empty[<=4], afull[2][<=3], tfull[2][<=3], drain, tmem slot, abort, last
  const uint32_t full = base, empty = base + 32, afull = base + 64, tfull = base + 112, drain = base + 160;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + 168);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
  volatile int *last_flag = reinterpret_cast<volatile int *>(tmem_slot + 2);
  const int units = p.tiles * p.nch;
  const int chunk = blockIdx.x % p.nch;  // gridDim.x is a multiple of nch: one chunk per CTA
  const int S = unit_sbs(p, chunk);

  if (threadIdx.x == 0) {
    for (int i = 0; i < kTcStages; ++i) {
      mbar_init(full + 8 * i, 1);
      mbar_init(empty + 8 * i, 4);  // one arrival per warp of the group the super-block is for
    }
    for (int i = 0; i < 2 * kTcBufs; ++i) {
      mbar_init(afull + 8 * i, 4);  // one arrival per warp of the group
      mbar_init(tfull + 8 * i, 1);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 9) {
    tmem_alloc(smem_u32(tmem_slot), kTcTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  grid_dep_launch();

  if (warp == 8) {
    // ---- producer: the raw super-blocks of the unit's rows, two per row and stage ----
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      uint32_t q = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
        const int r0 = (u / p.nch) * 128;  // a tile lies in one matrix (checked on the host)
        int s = 0;
        while (s + 1 < p.nseg && r0 >= p.seg_row0[s + 1]) ++s;
        const int y = r0 - p.seg_row0[s];
        for (int sbl = 0; sbl < S; ++sbl, ++q) {
          const uint32_t slot = q % kTcStages;
          if (q >= kTcStages && !wait_or_abort(empty + 8 * slot, ((q / kTcStages) - 1) & 1, abort_flag)) {
            ok = false;
            break;
          }
          // the whole box lands (rows past the matrix are zero-filled)
          mbar_arrive_expect_tx(full + 8 * slot, kStageBytes);
          tma_load_2d(base + kOffRing + slot * kStageBytes, &p.tmap[s], (chunk * p.cs + sbl) * (kSbBytes / 4), y,
                      full + 8 * slot, pol);
        }
      }
      // never leave with copies in flight into this CTA's shared memory
      for (uint32_t s = q > kTcStages ? q - kTcStages : 0; s < q; ++s)
        mbar_wait_bounded(full + 8 * (s % kTcStages), (s / kTcStages) & 1);
    }
  } else if (warp == 9) {
    // ---- MMA issuer: per step of a group, two block pairs into its TMEM buffer ----
    if (lane == 0) {
      uint32_t h[2] = {0, 0};
      const uint32_t zlo = base + kOffZlo, zhi = base + kOffZhi, xb = base + kOffXb;
      bool ok = true;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
        const int steps0 = 2 * group_sbs(S, 0), steps1 = 2 * group_sbs(S, 1);
        for (int j = 0; j < steps0 && ok; ++j) {
#pragma unroll
          for (int g = 0; g < 2; ++g) {
            if (!ok || j >= (g ? steps1 : steps0)) continue;
            const uint32_t buf = h[g] % kTcBufs;
            if (!wait_or_abort(afull + 8 * (kTcBufs * g + buf), (h[g] / kTcBufs) & 1, abort_flag)) {
              ok = false;
              continue;
            }
            tc_fence_after();
            const int lb0 = (2 * (j >> 1) + g) * 8 + (j & 1) * 4;  // first unit of the step in the chunk
            const uint32_t a = base + kOffA + (kTcBufs * g + buf) * 4 * 4096;
            const uint32_t d = tmem_base + static_cast<uint32_t>((kTcBufs * g + buf) * 32);
#pragma unroll
            for (int pr = 0; pr < 2; ++pr) {
              const uint32_t x0 = xb + (lb0 + 2 * pr) * 256, x1 = x0 + 256;
              mma_i8(d + 16 * pr, tc_desc(a + 2 * pr * 4096, 128, 256), tc_desc(x0, 128, zhi - x0), kTcIdesc, 0u);
              mma_i8(d + 16 * pr, tc_desc(a + (2 * pr + 1) * 4096, 128, 256), tc_desc(zlo, 128, x1 - zlo), kTcIdesc,
                     1u);
            }
            mma_commit(tfull + 8 * (kTcBufs * g + buf));
            ++h[g];
          }
        }
      }
    }
  } else {
    // ---- workers ----
    const int g = warp >> 2;                // group
    const int i = (warp & 3) * 32 + lane;   // row of the tile = TMEM lane
    const int tid = threadIdx.x;            // 0..255
    grid_dep_wait();                        // the activation comes from the previous kernel
    {
      // B operand of the chunk: unit lb, vector t, 16-byte half h at xb + lb*256 + h*128 + t*16
      const int kb0 = chunk * p.cs * 8;     // first 32-element unit of the chunk
      for (int c = tid; c < 128 * S; c += 256) {
        const int lb = c >> 4, t = (c >> 1) & 7, hf = c & 1;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (t < p.nb)
          v = __ldg(reinterpret_cast<const uint4 *>(p.xq + static_cast<int64_t>(t) * p.k + (kb0 + lb) * 32 + hf * 16));
        sts128(base + kOffXb + lb * 256 + hf * 128 + t * 16, v);
      }
      for (int c = tid; c < 64 * S; c += 256) {
        const int lb = c >> 3, t = c & 7;
        float xd = 0.f, xs = 0.f;
        if (t < p.nb) {
          xd = p.xd[static_cast<int64_t>(t) * p.nbp + kb0 + lb];
          xs = static_cast<float>(p.xs[static_cast<int64_t>(t) * p.nbp + kb0 + lb]);
        }
        reinterpret_cast<float *>(smem + kOffXd)[c] = xd;
        reinterpret_cast<float *>(smem + kOffXs)[c] = xs;
      }
      if (tid < 32) sts128(base + (tid < 16 ? kOffZlo + 16 * tid : kOffZhi + 16 * (tid - 16)), make_uint4(0, 0, 0, 0));
      fence_async_smem();
      named_sync(1, 256);
    }
    const uint32_t a_grp = base + kOffA + kTcBufs * g * 4 * 4096 + (i >> 3) * 256 + (i & 7) * 16;
    const uint32_t tq = tmem_base + (static_cast<uint32_t>((warp & 3) * 32) << 16) + static_cast<uint32_t>(kTcBufs * g * 32);
    const float *xdv = reinterpret_cast<const float *>(smem + kOffXd);
    const float *xsv = reinterpret_cast<const float *>(smem + kOffXs);
    float *red = reinterpret_cast<float *>(smem + kOffRed);
    uint32_t h = 0, q0 = 0;
    bool ok = true;
    // Waits keep `ok` uniform across the warp, so every warp-collective below (shuffles,
    // tcgen05.ld, __syncwarp) runs with all lanes or none.
    auto wait_all = [&](uint32_t bar, uint32_t parity) {
      const bool w = ok && wait_or_abort(bar, parity, abort_flag);
      ok = __all_sync(0xffffffffu, w);
      return ok;
    };

    // Q4_K: unpack half hf (units 4hf..4hf+3) of the row's super-block at `sb` into A buffer
    // `buf`: unit 2p+e of the half is nibble e of qs[64hf + 32p .. +32).
    auto unpack_q4k = [&](uint32_t sb, int hf, uint32_t buf) {
      const uint32_t a = a_grp + buf * 4 * 4096;
#pragma unroll
      for (int pr = 0; pr < 2; ++pr) {
        const uint4 x = lds128(sb + 16 + 64 * hf + 32 * pr), y = lds128(sb + 16 + 64 * hf + 32 * pr + 16);
        constexpr uint32_t kM = 0x0f0f0f0fu;
        sts128(a + 2 * pr * 4096, make_uint4(x.x & kM, x.y & kM, x.z & kM, x.w & kM));
        sts128(a + 2 * pr * 4096 + 128, make_uint4(y.x & kM, y.y & kM, y.z & kM, y.w & kM));
        sts128(a + (2 * pr + 1) * 4096, make_uint4((x.x >> 4) & kM, (x.y >> 4) & kM, (x.z >> 4) & kM, (x.w >> 4) & kM));
        sts128(a + (2 * pr + 1) * 4096 + 128,
               make_uint4((y.x >> 4) & kM, (y.y >> 4) & kM, (y.z >> 4) & kM, (y.w >> 4) & kM));
      }
    };
    // Q8_0: blocks 4hf..4hf+3 of the row's 8-block super-block at `sb` ({fp16 d, 32 x i8} at
    // 34j) into A buffer `buf`, and their scales {d, d} into cw.  The 136 bytes lie in the
    // 16-byte aligned 144-byte window from 128hf; each block's quants start at an even offset,
    // so every output word is one word of the window or a 16-bit funnel shift of two.
    auto unpack_q80 = [&](uint32_t sb, int hf, uint32_t buf, bool valid_row, uint64_t (&cw)[4]) {
      uint32_t wv[36];
#pragma unroll
      for (int k = 0; k < 9; ++k) {
        const uint4 v = valid_row ? lds128(sb + 128 * hf + 16 * k) : make_uint4(0, 0, 0, 0);
        wv[4 * k] = v.x;
        wv[4 * k + 1] = v.y;
        wv[4 * k + 2] = v.z;
        wv[4 * k + 3] = v.w;
      }
      const uint32_t a = a_grp + buf * 4 * 4096;
#pragma unroll
      for (int bb = 0; bb < 4; ++bb) {
        const int rel = 34 * (4 * hf + bb) - 128 * hf;  // block start in the window (even)
        const uint32_t dbits = (rel & 2) ? wv[rel >> 2] >> 16 : wv[rel >> 2] & 0xffffu;
        const float dj = half_bits_to_float(dbits);
        cw[bb] = pk2(dj, dj);
        const int o = rel + 2;                          // the quants
        uint32_t q[8];
#pragma unroll
        for (int k = 0; k < 8; ++k)
          q[k] = (o & 2) ? __funnelshift_r(wv[(o >> 2) + k], wv[(o >> 2) + k + 1], 16) : wv[(o >> 2) + k];
        if (valid_row) {
          sts128(a + bb * 4096, make_uint4(q[0], q[1], q[2], q[3]));
          sts128(a + bb * 4096 + 128, make_uint4(q[4], q[5], q[6], q[7]));
        }
      }
    };
    // The dots of step hh (units lb0..lb0+3 of the chunk) into the sums.  Q4_K: cw / cn hold
    // {d*sc, d*sc} and {-dmin*m, -dmin*m} of the four units; Q8_0: cw holds {d, d}.
    auto epilogue = [&](uint32_t hh, const uint64_t (&cw)[4], const uint64_t (&cn)[4], int lb0,
                        uint64_t (&acc)[4]) {
      if (!wait_all(tfull + 8 * (kTcBufs * g + hh % kTcBufs), (hh / kTcBufs) & 1)) return;
      tc_fence_after();
      uint32_t r[32];
      tmem_ld32(tq + (hh % kTcBufs) * 32, r);
      tmem_ld_wait();
#pragma unroll
      for (int bb = 0; bb < 4; ++bb) {
        const float4 d0 = *reinterpret_cast<const float4 *>(xdv + (lb0 + bb) * 8);
        const float4 d1 = *reinterpret_cast<const float4 *>(xdv + (lb0 + bb) * 8 + 4);
        const uint64_t xd2[4] = {pk2(d0.x, d0.y), pk2(d0.z, d0.w), pk2(d1.x, d1.y), pk2(d1.z, d1.w)};
        const int c0 = (bb >> 1) * 16 + (bb & 1) * 8;
        if constexpr (KIND == UGB_Q4_K) {
          const float4 s0 = *reinterpret_cast<const float4 *>(xsv + (lb0 + bb) * 8);
          const float4 s1 = *reinterpret_cast<const float4 *>(xsv + (lb0 + bb) * 8 + 4);
          const uint64_t xs2[4] = {pk2(s0.x, s0.y), pk2(s0.z, s0.w), pk2(s1.x, s1.y), pk2(s1.z, s1.w)};
#pragma unroll
          for (int tp = 0; tp < 4; ++tp) {
            // xd * (d*sc * I - dmin*m * xs), as unit_term<Q4_K>
            const uint64_t f = cvt2_i2f(r[c0 + 2 * tp], r[c0 + 2 * tp + 1]);
            const uint64_t inner = fma2(cw[bb], f, mul2(cn[bb], xs2[tp]));
            acc[tp] = fma2(xd2[tp], inner, acc[tp]);
          }
        } else {
#pragma unroll
          for (int tp = 0; tp < 4; ++tp) {
            // I * (d * xd), as unit_term<Q8_0>
            const uint64_t f = cvt2_i2f(r[c0 + 2 * tp], r[c0 + 2 * tp + 1]);
            acc[tp] = fma2(f, mul2(cw[bb], xd2[tp]), acc[tp]);
          }
        }
      }
      tc_fence_before();
    };
    auto arrive_afull = [&](uint32_t buf) {
      fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(afull + 8 * (kTcBufs * g + buf));
    };

    for (int u = blockIdx.x; u < units; u += gridDim.x) {
      const int tile = u / p.nch;
      const int row = tile * 128 + i;
      const bool valid = row < p.m;
      uint64_t acc[4] = {0, 0, 0, 0};
      // Step h unpacks half a super-block; its dots are rescaled kD steps later, so the MMA
      // round trip overlaps the steps between.  pw/pn/plb[d]: step h-1-d.
      constexpr int kD = kTcBufs - 1;
      uint64_t pw[kD][4], pn[kD][4];
      int plb[kD];
      int pending = 0;
      for (int sbl = g; sbl < S; sbl += 2) {
        const uint32_t q = q0 + sbl, slot = q % kTcStages;
        wait_all(full + 8 * slot, (q / kTcStages) & 1);
        if (!ok) continue;
        const uint32_t sb = base + kOffRing + slot * kStageBytes + i * kRowStride;
        uint4 hd = make_uint4(0, 0, 0, 0);
        if constexpr (KIND == UGB_Q4_K) {
          if (valid) hd = lds128(sb);  // {fp16 d, fp16 dmin}, scales[12] (get_scale_min_k4)
        }
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          uint64_t cw[4], cn[4] = {0, 0, 0, 0};
          if constexpr (KIND == UGB_Q4_K) {
            // units 4hf..4hf+3: sc / m of the low units from bytes 0-3 / 4-7, of the high units
            // from the low / high nibbles of bytes 8-11 and the top bits of bytes 0-7
            const float d = half_bits_to_float(hd.x), dmin = half_bits_to_float(hd.x >> 16);
            const uint32_t sc = hf == 0 ? hd.y & 0x3f3f3f3fu : (hd.w & 0x0f0f0f0fu) | ((hd.y >> 2) & 0x30303030u);
            const uint32_t mn = hf == 0 ? hd.z & 0x3f3f3f3fu : ((hd.w >> 4) & 0x0f0f0f0fu) | ((hd.z >> 2) & 0x30303030u);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float a0 = d * static_cast<float>((sc >> (8 * j)) & 0xff);
              const float b0 = -(dmin * static_cast<float>((mn >> (8 * j)) & 0xff));
              cw[j] = pk2(a0, a0);
              cn[j] = pk2(b0, b0);
            }
            if (valid) unpack_q4k(sb, hf, h % kTcBufs);
          } else {
            unpack_q80(sb, hf, h % kTcBufs, valid, cw);
          }
          if (hf == 1) {  // the stage is read: free it
            __syncwarp();
            if (lane == 0) mbar_arrive(empty + 8 * slot);
          }
          arrive_afull(h % kTcBufs);
          if (pending == kD) epilogue(h - kD, pw[kD - 1], pn[kD - 1], plb[kD - 1], acc);
#pragma unroll
          for (int d = kD - 1; d > 0; --d) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              pw[d][j] = pw[d - 1][j];
              pn[d][j] = pn[d - 1][j];
            }
            plb[d] = plb[d - 1];
          }
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            pw[0][j] = cw[j];
            pn[0][j] = cn[j];
          }
          plb[0] = sbl * 8 + hf * 4;
          pending = min(pending + 1, kD);
          ++h;
        }
      }
#pragma unroll
      for (int d = kD - 1; d >= 0; --d)  // the oldest first
        if (d < pending) epilogue(h - 1 - d, pw[d], pn[d], plb[d], acc);
      q0 += S;

      // ---- the unit's sums: group 1 hands over, group 0 adds and stores ----
      if (g == 1) {
#pragma unroll
        for (int tp = 0; tp < 4; ++tp) {
          const float2 v = upk2(acc[tp]);
          red[(2 * tp) * 128 + i] = v.x;
          red[(2 * tp + 1) * 128 + i] = v.y;
        }
      }
      named_sync(1, 256);
      float v[8];
      if (g == 0) {
#pragma unroll
        for (int tp = 0; tp < 4; ++tp) {
          const float2 a = upk2(acc[tp]);
          v[2 * tp] = a.x + red[(2 * tp) * 128 + i];
          v[2 * tp + 1] = a.y + red[(2 * tp + 1) * 128 + i];
        }
      }
      named_sync(2, 256);
      if (g == 0) {
        bool store = ok;
        if (p.nch > 1) {
          float *pp = p.part + (static_cast<int64_t>(tile) * p.nch + chunk) * 8 * 128;
#pragma unroll
          for (int t = 0; t < 8; ++t) __stcg(pp + t * 128 + i, v[t]);
          __threadfence();
          named_sync(3, 128);
          if (i == 0) {
            const uint32_t old = atomicAdd(p.tickets + tile, 1u);
            const bool last = old == static_cast<uint32_t>(p.nch - 1);
            if (last) atomicExch(p.tickets + tile, 0u);
            *last_flag = last ? 1 : 0;
          }
          named_sync(3, 128);
          store = store && *last_flag;
          if (store) {
            __threadfence();
            const float *pt = p.part + static_cast<int64_t>(tile) * p.nch * 8 * 128 + i;
#pragma unroll
            for (int t = 0; t < 8; ++t) v[t] = 0.f;
            // chunk order, four chunks' loads in flight at a time
            for (int c0 = 0; c0 < p.nch; c0 += 4) {
              float ld[4][8];
#pragma unroll
              for (int c = 0; c < 4; ++c)
#pragma unroll
                for (int t = 0; t < 8; ++t) ld[c][t] = c0 + c < p.nch ? __ldcg(pt + ((c0 + c) * 8 + t) * 128) : 0.f;
#pragma unroll
              for (int c = 0; c < 4; ++c)
#pragma unroll
                for (int t = 0; t < 8; ++t)
                  if (c0 + c < p.nch) v[t] += ld[c][t];
            }
          }
        }
        if (store && valid) {
#pragma unroll
          for (int t = 0; t < 8; ++t) {
            if (t < p.nb) {
              p.y[static_cast<int64_t>(t) * p.ldy + row] = v[t];
              if (!isfinite(v[t])) status_or(p.status, ST_NONFINITE_OUT);
            }
          }
        }
      }
    }
  }
  // Every role has finished (or given up).  Normally every MMA was consumed by the workers;
  // after an abort the MMA thread drains the tensor pipe before TMEM is freed.
  __syncthreads();
  if (warp == 9) {
    if (*abort_flag && lane == 0) {
      mma_commit(drain);
      mbar_wait_bounded(drain, 0);
    }
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, kTcTmemCols);
  }
  if (threadIdx.x == 0 && *abort_flag) status_or(p.status, ST_TIMEOUT);
}

}  // namespace

ugb_status init_matvec_tc_kernels(ugb_ctx *ctx) {
  // where a form does not fit, launch_matvec_tc declines and the dp4a kernels serve instead
  if (ctx->smem_optin >= static_cast<size_t>(TcGeo<UGB_Q4_K>::kSmem) &&
      cudaFuncSetAttribute(reinterpret_cast<const void *>(mv_tc_kernel<UGB_Q4_K>),
                           cudaFuncAttributeMaxDynamicSharedMemorySize, TcGeo<UGB_Q4_K>::kSmem) != cudaSuccess)
    return UGB_EBACKEND;
  if (ctx->smem_optin >= static_cast<size_t>(TcGeo<UGB_Q8_0>::kSmem) &&
      cudaFuncSetAttribute(reinterpret_cast<const void *>(mv_tc_kernel<UGB_Q8_0>),
                           cudaFuncAttributeMaxDynamicSharedMemorySize, TcGeo<UGB_Q8_0>::kSmem) != cudaSuccess)
    return UGB_EBACKEND;
  return UGB_OK;
}

// The K split of a plan: chunks of cs super-blocks, as many as keep every SM busy for the
// fewest super-blocks per CTA, counting about one super-block of pipeline fill and drain per
// unit (a split also pays the partial round trip).
struct TcPlan {
  int cs = 0, nch = 0, grid = 0;
};

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link against libcuda).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *f = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  });
  return fn;
}

TcPlan tc_plan(int64_t m, int64_t k, int sm_count) {
  TcPlan best;
  const int ns = static_cast<int>(k / 256);
  const int tiles = static_cast<int>((m + 127) / 128);
  int64_t best_cost = INT64_MAX;
  for (int n = 1; n <= ns; ++n) {
    const int cs = (ns + n - 1) / n;
    if (cs > kTcMaxCs) continue;
    const int nch = (ns + cs - 1) / cs;
    const int64_t u = static_cast<int64_t>(tiles) * nch;
    const int64_t grid = std::min<int64_t>(u, (sm_count / nch) * nch);
    if (grid < 1) continue;
    const int64_t cost = ((u + grid - 1) / grid) * (cs + 1) + (nch > 1 ? 1 : 0);
    if (cost < best_cost) {
      best_cost = cost;
      best.cs = cs;
      best.nch = nch;
      best.grid = static_cast<int>(grid);
    }
  }
  return best;
}

// Launch the tensor-core form for vectors [done, done + nb) of a Q4_K or Q8_0 segments launch, if
// it applies (sets *used).  Conditions: 5..8 vectors, K a multiple of 256, 16-byte aligned
// matrices and activation, every matrix but the last a whole number of 128-row tiles, and a K
// split that fits the context's workspace.
ugb_status launch_matvec_tc(ugb_ctx *ctx, cudaStream_t stream, const MatvecArgs &a, int64_t done, int nb,
                            bool *used) {
  *used = false;
  const bool q4k = a.kind == UGB_Q4_K;
  const int sb_bytes = q4k ? TcFmt<UGB_Q4_K>::kSbBytes : TcFmt<UGB_Q8_0>::kSbBytes;
  const size_t smem = q4k ? TcGeo<UGB_Q4_K>::kSmem : TcGeo<UGB_Q8_0>::kSmem;
  if ((!q4k && a.kind != UGB_Q8_0) || nb < 5 || nb > 8 || a.dots || a.k % 256 != 0 || a.nseg < 1 ||
      a.nseg > kMaxMatvecSegs || ctx->smem_optin < smem || !ctx->mv_part || a.row_bytes % 16 != 0 ||
      a.k > INT32_MAX || a.m > INT32_MAX)
    return UGB_OK;
  for (int i = 0; i < a.nseg; ++i)
    if (reinterpret_cast<uintptr_t>(a.ws[i]) % 16 != 0 || (i + 1 < a.nseg && a.seg_rows[i] % 128 != 0)) return UGB_OK;
  const PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
  if (!encode) return UGB_OK;
  const uint8_t *xq = a.xq + done * a.xl.k;
  if (reinterpret_cast<uintptr_t>(xq) % 16 != 0) return UGB_OK;
  const TcPlan pl = tc_plan(a.m, a.k, ctx->sm_count);
  const int tiles = static_cast<int>((a.m + 127) / 128);
  if (pl.nch < 1) return UGB_OK;
  if (pl.nch > 1 && (static_cast<size_t>(tiles) * pl.nch * 8 * 128 > ctx->mv_part_floats ||
                     static_cast<size_t>(tiles) > ctx->mv_ntickets))
    return UGB_OK;
  TcParams p{};
  int64_t row0 = 0;
  for (int i = 0; i < a.nseg; ++i) {
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(a.row_bytes / 4), static_cast<cuuint64_t>(a.seg_rows[i])};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(a.row_bytes)};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(sb_bytes / 4), 128};
    const cuuint32_t estr[2] = {1, 1};
    if (encode(&p.tmap[i], CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<uint8_t *>(a.ws[i]), dims, strides, box,
               estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return UGB_OK;
    p.seg_row0[i] = static_cast<int>(row0);
    row0 += a.seg_rows[i];
  }
  p.seg_row0[a.nseg] = static_cast<int>(row0);
  p.nseg = a.nseg;
  p.row_bytes = static_cast<uint64_t>(a.row_bytes);
  p.m = static_cast<int>(a.m);
  p.k = static_cast<int>(a.k);
  p.ns = static_cast<int>(a.k / 256);
  p.cs = pl.cs;
  p.nch = pl.nch;
  p.tiles = tiles;
  p.nb = nb;
  p.xq = xq;
  p.xd = reinterpret_cast<const float *>(a.xq + a.xl.d_off) + done * a.xl.nbp;
  p.xs = reinterpret_cast<const int *>(a.xq + a.xl.s_off) + done * a.xl.nbp;
  p.nbp = static_cast<int>(a.xl.nbp);
  p.y = a.y + done * a.ldy;
  p.ldy = a.ldy;
  p.part = ctx->mv_part;
  p.tickets = ctx->mv_tickets;
  p.status = ctx->status;

  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(pl.grid);
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = a.pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  void *args[] = {&p};
  const void *f = q4k ? reinterpret_cast<const void *>(mv_tc_kernel<UGB_Q4_K>)
                      : reinterpret_cast<const void *>(mv_tc_kernel<UGB_Q8_0>);
  if (cudaLaunchKernelExC(&cfg, f, args) != cudaSuccess)
    return UGB_EBACKEND;
  *used = true;
  return UGB_OK;
}

}  // namespace ugb
