// prefill.cu -- Q8 prefill: the weight repack, the token-batched activation quantiser and the
// INT8 tensor-core GEMM on tcgen05 (sm_100a).
//
// Reference: prefill_repack / prefill_quant / prefill_gemm (kernels/gpu_prefill.cu:10-59) and
// their host emitters p_quant / p_gemm (gpu_prefill.rs:22-30).  The reference multiplies a
// 16-row x 8-token x K32 mma.sync fragment per Q8_0 block and scales each block's int32 result
// by dw * dx in fp32 (fmaf((float)dot, dw*dx, acc)).  The same arithmetic is kept here:
//
//   Y[t][n] = sum over blocks b of  fmaf((float)I_b[t][n], dw[n][b] * dx[t][b], acc)
//   I_b[t][n] = sum_{i<32} qx[t][32b+i] * qw[n][32b+i]          (int32, exact)
//
// B200 form.  One CTA computes a 128-token x 128-row output tile:
//   * warp 0 streams stages of 4 K-blocks (A: 128 x 128 B of activation quants, B: 128 x 128 B
//     of weight quants, and both scale vectors) into a 4-deep shared-memory ring with 1-D bulk
//     copies -- both operands were written by the repack / quant kernels directly in the UMMA
//     canonical K-major layout, so no tensor map is needed;
//   * warp 1 issues one tcgen05.mma.kind::i8 (M=128, N=128, K=32) per K-block into one of four
//     TMEM accumulators (128 columns each, overwrite mode): every block's int32 dot lands alone,
//     and the accumulators change hands with the epilogue two blocks at a time;
//   * warps 2..17 (four per TMEM lane quarter, 32 columns each) read each block's int32 tile with
//     tcgen05.ld, scale it by dw*dx and accumulate in fp32 registers, then store the tile.
// Per-block scales are why the accumulator cannot stay in TMEM across K: the fp32 rescale of
// every 32-deep block is the bound of this kernel, not the tensor pipe.
//
// Operand layout in global memory (written by ugb_prefill_repack_q8_0 / ugb_prefill_quant):
//   quants [tile][kblock][4096 B]: one 128-row x 32-byte K-block in the canonical no-swizzle
//     K-major layout -- 16-byte core-matrix rows, offset(r, j) = (r/8)*256 + (j/16)*128 +
//     (r%8)*16 + (j%16)  (LBO = 128 B between the two 16-byte K halves, SBO = 256 B between
//     8-row groups);
//   scales [tile][kblock][128] f32 (dw converted exactly from fp16; dx = amax/127).
// Rows / tokens past the matrix are zero (quant 0, scale 0).
#include <cstring>
#include <type_traits>

#include "common.cuh"
#include "internal.hpp"
#include "prefill.hpp"
#include "prefill_quant.cuh"
#include "tcgen05.cuh"

namespace ugb {
namespace {

constexpr int kBM = kPrefillTile;         // tokens per tile (UMMA M, TMEM lanes)
constexpr int kKB = 4;                    // K-blocks (of 32) per stage
constexpr int kStages = 4;
constexpr int kAcc = 4;                   // TMEM accumulators
constexpr int kPairs = kAcc / 2;          // accumulator pairs: the unit of MMA / epilogue hand-off
static_assert(kAcc % 2 == 0 && kKB % 2 == 0, "pairs of blocks never straddle a stage or an accumulator set");
constexpr int kTileBytes = kPrefillTileBytes;         // 4096: one 128 x 32 B operand block
constexpr int kScaleBytes = kPrefillTile * 4;          // 512
constexpr int kEpiWarps = 16;
constexpr int kGemmThreads = 32 * (2 + kEpiWarps);    // 576

// Per output-tile width BN (weight rows per CTA, UMMA N): 128, or 64 for GEMMs whose 128-wide
// tiling leaves SMs idle (a 64-row CTA reads one half of each packed 128-row weight block).
template <int BN>
struct Geo {
  static constexpr int kBBytes = BN * 32;                                   // B operand per block
  static constexpr int kStageBytes = kKB * (kTileBytes + kBBytes + kScaleBytes + BN * 4);
  static constexpr int kSmem = kStages * kStageBytes + 256;                 // + barriers
  static constexpr int kTmemCols = kAcc * BN;                               // 512 or 256
  static constexpr int kCols = BN / 4;                                      // per epilogue warp
  // Instruction descriptor: D s32, A s8, B s8, both K-major, N = BN, M = 128.
  static constexpr uint32_t kIdesc = (2u << 4) | (1u << 7) | (1u << 10) |
                                     (static_cast<uint32_t>(BN >> 3) << 17) |
                                     (static_cast<uint32_t>(kBM >> 4) << 24);
};

// ---- repack: GGUF Q8_0 rows -> canonical K-major tiles -------------------------------------

// One thread per (row, K-block, 16-byte half): 16 quant bytes to their canonical place, and
// the block's fp16 scale converted exactly to f32 (prefill_repack, gpu_prefill.cu:39-46, is
// the same lossless re-layout into its mma.sync fragment order).  Rows past n are zero.
__global__ void __launch_bounds__(256) repack_q8_0_kernel(const uint8_t *__restrict__ w, int64_t n, int nb,
                                                          int64_t n_tiles, uint8_t *__restrict__ q_out,
                                                          float *__restrict__ s_out) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t total = n_tiles * kPrefillTile * nb * 2;
  if (i >= total) return;
  const int half = static_cast<int>(i & 1);
  const int b = static_cast<int>((i >> 1) % nb);
  const int64_t row = (i >> 1) / nb;
  const int64_t tile = row / kPrefillTile;
  const int r = static_cast<int>(row % kPrefillTile);
  uint32_t v[4] = {0, 0, 0, 0};
  float scale = 0.f;
  if (row < n) {
    const uint8_t *blk = w + (row * nb + b) * 34;
    const uint8_t *p = blk + 2 + half * 16;  // 2-byte aligned: assemble words from bytes
#pragma unroll
    for (int k = 0; k < 4; ++k)
      v[k] = p[4 * k] | (static_cast<uint32_t>(p[4 * k + 1]) << 8) | (static_cast<uint32_t>(p[4 * k + 2]) << 16) |
             (static_cast<uint32_t>(p[4 * k + 3]) << 24);
    scale = half_bits_to_float(blk[0] | (static_cast<uint32_t>(blk[1]) << 8));
  }
  uint8_t *dst = q_out + (tile * nb + b) * kPrefillTileBytes + canon_off(r, half * 16);
  *reinterpret_cast<uint4 *>(dst) = make_uint4(v[0], v[1], v[2], v[3]);
  if (half == 0) s_out[(tile * nb + b) * kPrefillTile + r] = scale;
}

// ---- activation quant: fp32 tokens -> canonical K-major tiles ------------------------------

// One warp per (token, K-block): the block-32 quantisation of quant_act (a = max|x|,
// d = a/127, q = clamp(rint(x * 127/a), +-127)), written in the canonical tile layout with one
// 32-bit store per four quants (prefill_quant, gpu_prefill.cu:47-59, writes the same values
// into its 8-token records).  Tokens past m are zero.
__global__ void __launch_bounds__(256) prefill_quant_kernel(const float *__restrict__ x, int64_t m, int64_t k,
                                                            int64_t ldx, int64_t m_tiles,
                                                            uint8_t *__restrict__ q_out, float *__restrict__ s_out,
                                                            uint32_t *status) {
  grid_dep_launch();
  grid_dep_wait();
  const int lane = threadIdx.x & 31;
  const int nb = static_cast<int>(k / 32);
  const int64_t gw = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (gw >= m_tiles * kPrefillTile * nb) return;
  const int b = static_cast<int>(gw % nb);
  const int64_t t = gw / nb;
  const float val = t < m ? x[t * ldx + b * 32 + lane] : 0.f;
  if (pf_quant_block(val, lane, t, b, nb, q_out, s_out) && lane == 0) status_or(status, ST_NONFINITE_IN);
}

// ---- the GEMM ------------------------------------------------------------------------------

struct GemmParams {
  const uint8_t *aq;  // activation tiles  [m_tiles][nb][4096]
  const float *as;    //                   [m_tiles][nb][128]
  const uint8_t *bq;  // weight tiles      [n_tiles][nb][4096]
  const float *bs;    //                   [n_tiles][nb][128]
  float *y;           // [m][ldy]; split s of a split-K launch writes y + s * y_split
  int64_t ldy, m, n;
  int nb;             // K-blocks of the operands' rows
  int nb_split;       // K-blocks one split sums (blockIdx.z takes blocks [z * nb_split, ...))
  int64_t y_split;
  int32_t *dots;      // optional [nb][m][n] int32 block dots (test path)
  uint32_t *status;
};

template <int BN, bool DOTS>
__global__ void __launch_bounds__(kGemmThreads, 1) prefill_gemm_kernel(GemmParams p) {
  using G = Geo<BN>;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t *ctl = smem + kStages * G::kStageBytes;
  uint64_t *full = reinterpret_cast<uint64_t *>(ctl);  // [kStages] bulk data landed
  uint64_t *empty = full + kStages;                    // [kStages] MMAs done + scales read
  uint64_t *tfull = empty + kStages;                   // [kPairs] a pair's int32 tiles ready
  uint64_t *tempty = tfull + kPairs;                   // [kPairs] a pair's tiles read by the epilogue
  uint64_t *drain = tempty + kPairs;                   // [1] final commit on abort
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
  // stage layout: [A: kKB x 4096][B: kKB x BN*32][dx: kKB x 128 f32][dw: kKB x BN f32]
  constexpr int kOffB = kKB * kTileBytes;
  constexpr int kOffSA = kOffB + kKB * G::kBBytes;
  constexpr int kOffSB = kOffSA + kKB * kScaleBytes;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t m_tile = blockIdx.x;
  const int64_t n_col0 = static_cast<int64_t>(blockIdx.y) * BN;  // first output column
  const int64_t w_tile = n_col0 / kPrefillTile;                  // packed 128-row weight tile
  const int w_half = static_cast<int>((n_col0 % kPrefillTile) / BN);  // which BN rows of it
  // this CTA's K-blocks: [kb0, kb0 + nb) of the rows' p.nb (all of them unless split)
  const int kb0 = static_cast<int>(blockIdx.z) * p.nb_split;
  const int nb = min(p.nb_split, p.nb - kb0);
  float *const y_out = p.y + static_cast<int64_t>(blockIdx.z) * p.y_split;
  const int n_stages = (nb + kKB - 1) / kKB;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(smem_u32(&full[i]), 1);
      mbar_init(smem_u32(&empty[i]), kEpiWarps + 1);
    }
    for (int i = 0; i < kPairs; ++i) {
      mbar_init(smem_u32(&tfull[i]), 1);
      mbar_init(smem_u32(&tempty[i]), kEpiWarps);
    }
    mbar_init(smem_u32(drain), 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), G::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  grid_dep_launch();

  if (warp == 0) {
    // ---- producer: one elected lane streams stages of kKB K-blocks ----
    if (lane == 0) {
      grid_dep_wait();  // the activation tiles come from the preceding quant kernel
      const uint64_t pol = policy_evict_last();
      const uint8_t *a_base = p.aq + (m_tile * p.nb + kb0) * kTileBytes;
      const uint8_t *b_base = p.bq + (w_tile * p.nb + kb0) * kTileBytes + w_half * G::kBBytes;
      const float *sa_base = p.as + (m_tile * p.nb + kb0) * kPrefillTile;
      const float *sb_base = p.bs + (w_tile * p.nb + kb0) * kPrefillTile + w_half * BN;
      int issued = 0;
      for (int s = 0; s < n_stages; ++s) {
        const int slot = s % kStages;
        if (s >= kStages && !wait_or_abort(smem_u32(&empty[slot]), ((s / kStages) - 1) & 1, abort_flag)) break;
        const int b0 = s * kKB, nblk = min(kKB, nb - b0);
        uint8_t *st = smem + slot * G::kStageBytes;
        const uint32_t bar = smem_u32(&full[slot]);
        mbar_arrive_expect_tx(bar, nblk * (kTileBytes + G::kBBytes + kScaleBytes + BN * 4));
        bulk_g2s(smem_u32(st), a_base + static_cast<int64_t>(b0) * kTileBytes, nblk * kTileBytes, bar, pol);
        bulk_g2s(smem_u32(st + kOffSA), sa_base + static_cast<int64_t>(b0) * kPrefillTile, nblk * kScaleBytes, bar,
                 pol);
        if (BN == kPrefillTile) {  // whole tiles: one copy per operand and stage
          bulk_g2s(smem_u32(st + kOffB), b_base + static_cast<int64_t>(b0) * kTileBytes, nblk * kTileBytes, bar, pol);
          bulk_g2s(smem_u32(st + kOffSB), sb_base + static_cast<int64_t>(b0) * kPrefillTile, nblk * BN * 4, bar, pol);
        } else {                   // half tiles: rows [w_half*BN, +BN) of every block
          for (int i = 0; i < nblk; ++i) {
            bulk_g2s(smem_u32(st + kOffB + i * G::kBBytes), b_base + static_cast<int64_t>(b0 + i) * kTileBytes,
                     G::kBBytes, bar, pol);
            bulk_g2s(smem_u32(st + kOffSB + i * BN * 4), sb_base + static_cast<int64_t>(b0 + i) * kPrefillTile,
                     BN * 4, bar, pol);
          }
        }
        issued = s + 1;
      }
      // Never leave with bulk copies in flight into this CTA's shared memory.
      for (int s = max(0, issued - kStages); s < issued; ++s)
        mbar_wait_bounded(smem_u32(&full[s % kStages]), (s / kStages) & 1);
    }
  } else if (warp == 1) {
    // ---- MMA issuer: one tcgen05.mma per K-block into accumulator b % kAcc; blocks go to the
    // epilogue in pairs (2p, 2p + 1), one commit per pair ----
    if (lane == 0) {
      bool ok = true;
      for (int b = 0; b < nb && ok; ++b) {
        const int s = b / kKB, slot = s % kStages, kb = b % kKB, j = b % kAcc, pr = b / 2, P = pr % kPairs;
        if (kb == 0) ok = wait_or_abort(smem_u32(&full[slot]), s / kStages & 1, abort_flag);
        if (ok && b % 2 == 0 && pr >= kPairs)  // the pair kPairs back has been read out
          ok = wait_or_abort(smem_u32(&tempty[P]), ((pr / kPairs) - 1) & 1, abort_flag);
        if (!ok) break;
        tc_fence_after();
        const uint32_t st = smem_u32(smem + slot * G::kStageBytes);
        mma_i8(tmem_base + static_cast<uint32_t>(j * BN), smem_desc(st + kb * kTileBytes),
               smem_desc(st + kOffB + kb * G::kBBytes), G::kIdesc, 0u);
        if (b % 2 == 1 || b == nb - 1) mma_commit(smem_u32(&tfull[P]));
        if (kb == kKB - 1 || b == nb - 1) mma_commit(smem_u32(&empty[slot]));
      }
      // The last stages' release phases (commit + epilogue arrivals) are waited here, so no
      // commit arrival can land after the CTA has exited.
      for (int s = max(0, n_stages - kStages); s < n_stages && ok; ++s)
        ok = wait_or_abort(smem_u32(&empty[s % kStages]), (s / kStages) & 1, abort_flag);
    }
  } else {
    // ---- epilogue: rescale every block's int32 tile into fp32 accumulators ----
    constexpr int kC = G::kCols;           // columns of this warp (32 or 16)
    const int q = warp & 3;                // TMEM lane quarter this warp may access
    const int h = (warp - 2) >> 2;         // column quarter
    const int t_local = q * 32 + lane;     // token row of the tile
    const int c0 = h * kC;                 // first column of this warp
    const int64_t t = m_tile * kBM + t_local;
    uint64_t acc[kC / 2];                  // pairs of fp32 accumulators
#pragma unroll
    for (int i = 0; i < kC / 2; ++i) acc[i] = 0ull;
    // Block kb of the stage at st (its tile in accumulator kb: a stage's kKB blocks go to the kAcc
    // accumulators in order) into the fp32 accumulators; kb is a compile-time constant, so the
    // scale and tensor-memory addresses are fixed offsets.
    const uint32_t tq = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(c0);
    auto rescale = [&](const uint8_t *st, auto kbc, int b) {
      constexpr int kb = decltype(kbc)::value;
      const float dx = reinterpret_cast<const float *>(st + kOffSA)[kb * kPrefillTile + t_local];
      const float4 *dw4 = reinterpret_cast<const float4 *>(st + kOffSB + (kb * BN + c0) * 4);
      const uint64_t dx2 = pk2(dx, dx);
      uint32_t r[kC];
      if constexpr (kC == 32) {
        tmem_ld32(tq + kb * BN, r);
      } else {
        tmem_ld16(tq + kb * BN, r);
      }
      tmem_ld_wait();
      if (DOTS) {
        for (int i = 0; i < kC; ++i) {
          const int64_t nn = n_col0 + c0 + i;
          if (t < p.m && nn < p.n)
            p.dots[(static_cast<int64_t>(kb0 + b) * p.m + t) * p.n + nn] = static_cast<int32_t>(r[i]);
        }
      }
#pragma unroll
      for (int i = 0; i < kC; i += 4) {
        const float4 w = dw4[i / 4];  // same address across the warp: broadcast
        // fmaf((float)I, dw * dx, acc) per lane, two columns per instruction
        const uint64_t s01 = mul2(pk2(w.x, w.y), dx2), s23 = mul2(pk2(w.z, w.w), dx2);
        const uint64_t f01 = cvt2_i2f(r[i], r[i + 1]);
        const uint64_t f23 = cvt2_i2f(r[i + 2], r[i + 3]);
        acc[i / 2] = fma2(f01, s01, acc[i / 2]);
        acc[i / 2 + 1] = fma2(f23, s23, acc[i / 2 + 1]);
      }
    };
    // A pair (kb, kb + 1) of the stage: one wait for both tiles and one release of both
    // accumulators, since these waits, fences and arrivals (not the arithmetic) are most of a
    // warp's chain per block; the two blocks are still added in block order.
    auto pair = [&](const uint8_t *st, int s, auto kbc, int nblk) -> bool {
      constexpr int kb = decltype(kbc)::value;
      const int pr = (s * kKB + kb) / 2, P = pr % kPairs;
      if (!wait_or_abort(smem_u32(&tfull[P]), (pr / kPairs) & 1, abort_flag)) return false;
      tc_fence_after();
      rescale(st, std::integral_constant<int, kb>{}, s * kKB + kb);
      if (kb + 1 < nblk) rescale(st, std::integral_constant<int, kb + 1>{}, s * kKB + kb + 1);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(smem_u32(&tempty[P]));
        if (kb + 2 >= nblk) mbar_arrive(smem_u32(&empty[s % kStages]));
      }
      return true;
    };
    static_assert(kKB == 4 && kAcc == kKB, "a stage's blocks map one to one onto the accumulators");
    bool ok = true;
    for (int s = 0; s < n_stages && ok; ++s) {
      const uint8_t *st = smem + (s % kStages) * G::kStageBytes;
      const int nblk = min(kKB, nb - s * kKB);
      ok = wait_or_abort(smem_u32(&full[s % kStages]), s / kStages & 1, abort_flag);
      if (ok) ok = pair(st, s, std::integral_constant<int, 0>{}, nblk);
      if (ok && nblk > 2) ok = pair(st, s, std::integral_constant<int, 2>{}, nblk);
    }
    if (ok && t < p.m) {
      float *yrow = y_out + t * p.ldy + n_col0 + c0;
      const int64_t n_left = p.n - (n_col0 + c0);
      if (n_left >= kC && (reinterpret_cast<uintptr_t>(yrow) & 15) == 0) {
#pragma unroll
        for (int i = 0; i < kC / 2; i += 2) {
          const float2 a0 = upk2(acc[i]), a1 = upk2(acc[i + 1]);
          *reinterpret_cast<float4 *>(yrow + 2 * i) = make_float4(a0.x, a0.y, a1.x, a1.y);
        }
      } else {
#pragma unroll
        for (int i = 0; i < kC / 2; ++i) {
          const float2 a = upk2(acc[i]);
          if (2 * i < n_left) yrow[2 * i] = a.x;
          if (2 * i + 1 < n_left) yrow[2 * i + 1] = a.y;
        }
      }
    }
  }
  // Every role has finished (or given up).  In the normal path every MMA was consumed by the
  // epilogue; after an abort the MMA thread drains the tensor pipe before TMEM is freed.
  __syncthreads();
  if (warp == 1) {
    if (*abort_flag && lane == 0) {
      mma_commit(smem_u32(drain));
      mbar_wait_bounded(smem_u32(drain), 0);
    }
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, G::kTmemCols);
  }
  if (threadIdx.x == 0 && *abort_flag) status_or(p.status, ST_TIMEOUT);
}

}  // namespace

// ---- host ------------------------------------------------------------------------------------

ugb_status init_prefill_kernels(ugb_ctx *ctx) {
  if (ctx->smem_optin < static_cast<size_t>(Geo<128>::kSmem)) return UGB_EBACKEND;
  for (const void *f : {reinterpret_cast<const void *>(prefill_gemm_kernel<128, false>),
                        reinterpret_cast<const void *>(prefill_gemm_kernel<128, true>)})
    if (cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, Geo<128>::kSmem) != cudaSuccess)
      return UGB_EBACKEND;
  for (const void *f : {reinterpret_cast<const void *>(prefill_gemm_kernel<64, false>),
                        reinterpret_cast<const void *>(prefill_gemm_kernel<64, true>)})
    if (cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, Geo<64>::kSmem) != cudaSuccess)
      return UGB_EBACKEND;
  return UGB_OK;
}

PackedLayout prefill_layout(int64_t rows, int64_t k) {
  PackedLayout p;
  p.tiles = (rows + kPrefillTile - 1) / kPrefillTile;
  p.nb = k / 32;
  p.q_bytes = static_cast<size_t>(p.tiles * p.nb) * kPrefillTileBytes;
  p.bytes = p.q_bytes + static_cast<size_t>(p.tiles * p.nb) * kPrefillTile * sizeof(float);
  return p;
}

namespace {

using Packed = PackedLayout;
inline Packed packed_layout(int64_t rows, int64_t k) { return prefill_layout(rows, k); }

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

ugb_status launch_gemm(ugb_ctx *ctx, cudaStream_t stream, const void *w_packed, const void *x_packed, float *y,
                       int32_t *dots, int64_t m, int64_t n, int64_t k, int64_t ldy, int splits = 1) {
  if (!ctx || !ctx->status) return UGB_ECONTEXT;
  if (m < 1 || n < 1 || k < 32 || k % 32 || ldy < n || k / 32 > (1 << 20)) return UGB_ESHAPE;
  if (!w_packed || !x_packed || !y || !aligned16(w_packed) || !aligned16(x_packed)) return UGB_EALIGN;
  const Packed pw = packed_layout(n, k), px = packed_layout(m, k);
  if (2 * pw.tiles > 65535) return UGB_ESHAPE;
  GemmParams p;
  p.aq = static_cast<const uint8_t *>(x_packed);
  p.as = reinterpret_cast<const float *>(static_cast<const uint8_t *>(x_packed) + px.q_bytes);
  p.bq = static_cast<const uint8_t *>(w_packed);
  p.bs = reinterpret_cast<const float *>(static_cast<const uint8_t *>(w_packed) + pw.q_bytes);
  p.y = y;
  p.ldy = ldy;
  p.m = m;
  p.n = n;
  p.nb = static_cast<int>(k / 32);
  if (splits < 1 || splits > p.nb) return UGB_ESHAPE;
  p.nb_split = (p.nb + splits - 1) / splits;
  splits = (p.nb + p.nb_split - 1) / p.nb_split;  // no split without blocks
  p.y_split = m * ldy;
  p.dots = dots;
  p.status = ctx->status;
  // 64-row CTAs when 128-row tiles would leave SMs idle (twice the CTAs, same packed layout);
  // a split-K launch keeps whole tiles (its splits fill the SMs)
  const bool narrow = splits == 1 && px.tiles * pw.tiles < ctx->sm_count;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(px.tiles), static_cast<unsigned>(narrow ? 2 * pw.tiles : pw.tiles),
                     static_cast<unsigned>(splits));
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = narrow ? Geo<64>::kSmem : Geo<128>::kSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = ctx->pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (p.dots)
    return cuda_status(narrow ? cudaLaunchKernelEx(&cfg, prefill_gemm_kernel<64, true>, p)
                              : cudaLaunchKernelEx(&cfg, prefill_gemm_kernel<128, true>, p));
  return cuda_status(narrow ? cudaLaunchKernelEx(&cfg, prefill_gemm_kernel<64, false>, p)
                            : cudaLaunchKernelEx(&cfg, prefill_gemm_kernel<128, false>, p));
}

}  // namespace

ugb_status launch_prefill_repack(cudaStream_t stream, const uint8_t *w, int64_t n, int64_t k, uint8_t *q_out,
                                 float *s_out) {
  const Packed pw = packed_layout(n, k);
  const int64_t total = pw.tiles * kPrefillTile * pw.nb * 2;
  const int64_t blocks = (total + 255) / 256;
  if (blocks > 0x7fffffff) return UGB_ESHAPE;
  repack_q8_0_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(w, n, static_cast<int>(pw.nb), pw.tiles,
                                                                        q_out, s_out);
  return cuda_status(cudaGetLastError());
}

ugb_status launch_prefill_quant(ugb_ctx *ctx, cudaStream_t stream, const float *x, int64_t m, int64_t k, int64_t ldx,
                                uint8_t *packed) {
  const Packed px = packed_layout(m, k);
  const int64_t warps = px.tiles * kPrefillTile * px.nb;
  const int64_t blocks = (warps + 7) / 8;
  if (blocks > 0x7fffffff) return UGB_ESHAPE;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(blocks));
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = ctx->pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, prefill_quant_kernel, x, m, k, ldx, px.tiles, packed,
                                        reinterpret_cast<float *>(packed + px.q_bytes), ctx->status));
}

ugb_status launch_prefill_gemm(ugb_ctx *ctx, cudaStream_t stream, const void *w_packed, const void *x_packed,
                               float *y, int64_t m, int64_t n, int64_t k, int64_t ldy, int splits) {
  return launch_gemm(ctx, stream, w_packed, x_packed, y, nullptr, m, n, k, ldy, splits);
}

int prefill_gemm_splits(const ugb_ctx *ctx, int64_t m, int64_t n, int64_t k) {
  // Split K while that shortens the launch: waves of whole-tile CTAs x K-blocks per CTA (the
  // per-block rescale bounds each CTA, so its time is proportional to its K-blocks).
  const int64_t tiles = prefill_layout(m, k).tiles * prefill_layout(n, k).tiles, nb = k / 32;
  int best = 1;
  int64_t best_cost = INT64_MAX;
  for (int s = 1; s <= kMaxGemmSplits && s <= nb; ++s) {
    const int64_t waves = (tiles * s + ctx->sm_count - 1) / ctx->sm_count;
    const int64_t cost = waves * ((nb + s - 1) / s);
    if (cost < best_cost) {
      best_cost = cost;
      best = s;
    }
  }
  return best;
}

}  // namespace ugb

using namespace ugb;

extern "C" {

int64_t ugb_prefill_packed_bytes(int64_t rows, int64_t k) {
  if (rows < 1 || k < 32 || k % 32) return -1;
  return static_cast<int64_t>(packed_layout(rows, k).bytes);
}

ugb_status ugb_prefill_repack_q8_0(ugb_ctx *ctx, ugb_stream stream, const void *w_dev, int64_t n, int64_t k,
                                   void *packed_dev) {
  if (!ctx || !ctx->status) return UGB_ECONTEXT;
  if (n < 1 || k < 32 || k % 32) return UGB_ESHAPE;
  if (!w_dev || !packed_dev || !aligned16(packed_dev)) return UGB_EALIGN;
  const Packed pw = packed_layout(n, k);
  uint8_t *q = static_cast<uint8_t *>(packed_dev);
  return launch_prefill_repack(stream, static_cast<const uint8_t *>(w_dev), n, k, q,
                               reinterpret_cast<float *>(q + pw.q_bytes));
}

ugb_status ugb_prefill_quant(ugb_ctx *ctx, ugb_stream stream, const float *x_dev, int64_t m, int64_t k,
                             void *packed_dev) {
  if (!ctx || !ctx->status) return UGB_ECONTEXT;
  if (m < 1 || k < 32 || k % 32) return UGB_ESHAPE;
  if (!x_dev || !packed_dev || !aligned16(packed_dev)) return UGB_EALIGN;
  return launch_prefill_quant(ctx, stream, x_dev, m, k, k, static_cast<uint8_t *>(packed_dev));
}

ugb_status ugb_prefill_gemm_q8_0(ugb_ctx *ctx, ugb_stream stream, const void *w_packed, const void *x_packed,
                                 float *y_dev, int64_t m, int64_t n, int64_t k, int64_t ldy) {
  return launch_gemm(ctx, stream, w_packed, x_packed, y_dev, nullptr, m, n, k, ldy);
}

ugb_status ugb_prefill_block_dots(ugb_ctx *ctx, ugb_stream stream, const void *w_packed, const void *x_packed,
                                  int32_t *dots_dev, float *y_dev, int64_t m, int64_t n, int64_t k) {
  if (!dots_dev) return UGB_EALIGN;
  return launch_gemm(ctx, stream, w_packed, x_packed, y_dev, dots_dev, m, n, k, n);
}

}  // extern "C"
