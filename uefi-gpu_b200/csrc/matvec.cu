// matvec.cu -- HBM-streaming block-quantised matvec for decode (Q8_0 / Q4_K / Q3_K x Q8_1).
//
// Replaces linear_dp4a / qkv_dp4a / gateup_dp4a (gpu_dp4a.cu:32-64) and frontier_matvec
// (frontier_quant.cu:58-66).  Design for sm_100a:
//  * Persistent CTAs (grid = min(row groups, SMs x resident CTAs)), 8 warps each.
//  * Work item = (group of R consecutive rows) x (K chunk).  One elected thread streams the
//    item's R row segments (GGUF bytes, unchanged) and the activation chunk into a stage of
//    a multi-stage shared-memory ring with cp.async.bulk, completing on one mbarrier per
//    stage; weights carry an L2 evict-first hint since each byte is read exactly once.
//  * Warp w owns rows w*RW..w*RW+RW-1 of the group; lane l takes 32-element units l, l+32, ..
//    of the chunk, forms the exact int32 block dot with dp4a and accumulates the scaled term
//    in fp32 registers across chunks.  The row total is a fixed xor-shuffle tree, so results
//    are deterministic run to run.
//  * Every mbarrier wait is bounded; a lost copy sets UGB_STATUS_TIMEOUT and the CTA leaves.
#include <algorithm>
#include <cmath>

#include "formats.cuh"
#include "internal.hpp"

namespace ugb {
namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr uint32_t kBarBytes = 128;  // mbarrier area at the start of dynamic shared memory

struct MvParams {
  const uint8_t *w;
  const uint8_t *w_end;       // w + m * row_bytes
  const uint8_t *w_end16;     // w_end rounded down to 16 bytes
  uint64_t row_bytes;
  int k, m, batch;
  int kc, nch, ngroups;
  uint32_t seg_stride, stage_bytes;
  uint32_t xq_off, xd_off, xs_off, kcb4;
  int stages;
  const uint8_t *xq;
  const float *xd;
  const int *xs;
  int64_t xq_stride, xds_stride;
  float *y;
  int64_t ldy;
  int32_t *dots;
  int64_t dots_ld;
  uint32_t *status;
};

template <int KIND>
__host__ __device__ constexpr uint64_t bytes_of(uint64_t elems) {
  return elems / Fmt<KIND>::kElems * Fmt<KIND>::kBytes;
}

// Issue (or size) the copies of local item t into the stage at `stage`.  Called by one
// thread.  Tail bytes that fall in the last partial 16 bytes of the weight buffer are copied
// with plain loads first (bulk copies need 16-byte aligned ranges and must not read past the
// buffer), then the barrier is armed with the bulk byte count, then the bulk copies go out.
template <int KIND, int NB, int RW>
__device__ void issue_item(const MvParams &p, int t, uint32_t stage, uint32_t bar,
                           uint64_t pol_w, bool weights, bool acts, bool arm) {
  const int j = t / p.nch, c = t - j * p.nch;
  const int g = blockIdx.x + j * gridDim.x;
  constexpr int R = kWarps * RW;
  const int r0 = g * R;
  const int nrows = min(R, p.m - r0);
  const int k0 = c * p.kc;
  const int klen = min(p.kc, p.k - k0);
  const uint64_t seg_off = bytes_of<KIND>(k0), seg_len = bytes_of<KIND>(klen);
  const uint32_t xlen = static_cast<uint32_t>(klen);
  const uint32_t dlen = static_cast<uint32_t>(round_up(klen / 32, 4) * 4);

  if (arm) {
    uint32_t tx = 0;
    for (int r = 0; r < nrows; ++r) {
      const uint8_t *src = p.w + static_cast<uint64_t>(r0 + r) * p.row_bytes + seg_off;
      const uint8_t *a0 = reinterpret_cast<const uint8_t *>(reinterpret_cast<uintptr_t>(src) & ~uintptr_t(15));
      const uint8_t *e = src + seg_len;
      const uint8_t *a1 = reinterpret_cast<const uint8_t *>((reinterpret_cast<uintptr_t>(e) + 15) & ~uintptr_t(15));
      if (e > p.w_end16) {  // only the final segment of the buffer can get here
        const uint8_t *tb = a0 > p.w_end16 ? a0 : p.w_end16;
        for (const uint8_t *b = tb; b < e; ++b)
          sts8(stage + r * p.seg_stride + static_cast<uint32_t>(b - a0), *b);
        a1 = tb;
      }
      tx += static_cast<uint32_t>(a1 - a0);
    }
    tx += NB * (xlen + dlen * (Fmt<KIND>::kNeedsSum ? 2u : 1u));
    mbar_arrive_expect_tx(bar, tx);
  }
  if (weights) {
    for (int r = 0; r < nrows; ++r) {
      const uint8_t *src = p.w + static_cast<uint64_t>(r0 + r) * p.row_bytes + seg_off;
      const uint8_t *a0 = reinterpret_cast<const uint8_t *>(reinterpret_cast<uintptr_t>(src) & ~uintptr_t(15));
      const uint8_t *e = src + seg_len;
      const uint8_t *a1 = reinterpret_cast<const uint8_t *>((reinterpret_cast<uintptr_t>(e) + 15) & ~uintptr_t(15));
      if (e > p.w_end16) a1 = a0 > p.w_end16 ? a0 : p.w_end16;
      if (a1 > a0) bulk_g2s(stage + r * p.seg_stride, a0, static_cast<uint32_t>(a1 - a0), bar, pol_w);
    }
  }
  if (acts) {
    const uint64_t pol_x = policy_evict_last();
    for (int v = 0; v < NB; ++v) {
      bulk_g2s(stage + p.xq_off + v * p.kc, p.xq + v * p.xq_stride + k0, xlen, bar, pol_x);
      bulk_g2s(stage + p.xd_off + v * p.kcb4 * 4, p.xd + v * p.xds_stride + k0 / 32, dlen, bar, pol_x);
      if (Fmt<KIND>::kNeedsSum)
        bulk_g2s(stage + p.xs_off + v * p.kcb4 * 4, p.xs + v * p.xds_stride + k0 / 32, dlen, bar, pol_x);
    }
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <int KIND, int NB, int RW, bool DOTS>
__global__ void __launch_bounds__(kThreads) mv_stream_kernel(const MvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr int R = kWarps * RW;
  const uint32_t bars = smem_u32(smem);
  const uint32_t data = bars + kBarBytes;
  const int my_groups = (p.ngroups - static_cast<int>(blockIdx.x) + static_cast<int>(gridDim.x) - 1) /
                        static_cast<int>(gridDim.x);
  const int T = my_groups * p.nch;

  if (tid == 0) {
    for (int s = 0; s < p.stages; ++s) mbar_init(bars + 8 * s, 1);
    fence_mbar_init();
    const uint64_t pol_w = policy_evict_first();
    const int pre = min(T, p.stages);
    // Weights do not depend on earlier kernels: arm and start them before waiting on the
    // programmatic dependency, then fetch the activations.
    for (int t = 0; t < pre; ++t)
      issue_item<KIND, NB, RW>(p, t, data + (t % p.stages) * p.stage_bytes, bars + 8 * (t % p.stages),
                               pol_w, true, false, true);
    grid_dep_wait();
    for (int t = 0; t < pre; ++t)
      issue_item<KIND, NB, RW>(p, t, data + (t % p.stages) * p.stage_bytes, bars + 8 * (t % p.stages),
                               pol_w, false, true, false);
  }
  grid_dep_wait();
  grid_dep_launch();
  __syncthreads();

  float acc[RW][NB];
#pragma unroll
  for (int rr = 0; rr < RW; ++rr)
#pragma unroll
    for (int v = 0; v < NB; ++v) acc[rr][v] = 0.f;

  for (int t = 0; t < T; ++t) {
    const int s = t % p.stages;
    const uint32_t stage = data + s * p.stage_bytes;
    // Warp-uniform so the shuffles below always see a full warp.
    const bool ok = __all_sync(0xffffffffu, mbar_wait_bounded(bars + 8 * s, (t / p.stages) & 1));
    const int j = t / p.nch, c = t - j * p.nch;
    const int g = blockIdx.x + j * gridDim.x;
    const int r0 = g * R;
    const int nrows = min(R, p.m - r0);
    if (ok) {
      const int k0 = c * p.kc;
      const int nunits = min(p.kc, p.k - k0) / 32;
      const uint64_t seg_off = bytes_of<KIND>(k0);
      uint32_t seg[RW];
#pragma unroll
      for (int rr = 0; rr < RW; ++rr) {
        const int r = warp * RW + rr;
        const uintptr_t src = reinterpret_cast<uintptr_t>(p.w + static_cast<uint64_t>(r0 + r) * p.row_bytes + seg_off);
        seg[rr] = stage + r * p.seg_stride + static_cast<uint32_t>(src & 15);
      }
      for (int u = lane; u < nunits; u += 32) {
        XUnit x[NB];
#pragma unroll
        for (int v = 0; v < NB; ++v)
          load_xunit(stage + p.xq_off + v * p.kc + 32 * u, stage + p.xd_off + (v * p.kcb4 + u) * 4,
                     stage + p.xs_off + (v * p.kcb4 + u) * 4, Fmt<KIND>::kNeedsSum, x[v]);
#pragma unroll
        for (int rr = 0; rr < RW; ++rr) {
          const int r = warp * RW + rr;
          if (r < nrows) {
            WUnit wu;
            load_wunit<KIND>(seg[rr], u, wu);
#pragma unroll
            for (int v = 0; v < NB; ++v) {
              const int isum = unit_isum<KIND>(wu, x[v]);
              if constexpr (DOTS) {
                p.dots[static_cast<int64_t>(r0 + r) * p.dots_ld + k0 / 32 + u] = isum;
              } else {
                acc[rr][v] += unit_term<KIND>(wu, x[v], isum);
              }
            }
          }
        }
      }
      if (!DOTS && c == p.nch - 1) {
#pragma unroll
        for (int rr = 0; rr < RW; ++rr) {
          const int r = warp * RW + rr;
#pragma unroll
          for (int v = 0; v < NB; ++v) {
            const float val = warp_sum(acc[rr][v]);
            acc[rr][v] = 0.f;
            if (lane == 0 && r < nrows) {
              p.y[v * p.ldy + r0 + r] = val;
              if (!isfinite(val)) status_or(p.status, ST_NONFINITE_OUT);
            }
          }
        }
      }
    }
    if (__syncthreads_or(!ok)) {
      if (tid == 0) {
        status_or(p.status, ST_TIMEOUT);
        // Give copies still in flight a bounded chance to land before shared memory is
        // released.
        for (int q = 0; q < p.stages && t + q < T; ++q)
          mbar_wait_bounded(bars + 8 * ((t + q) % p.stages), ((t + q) / p.stages) & 1);
      }
      return;
    }
    if (tid == 0 && t + p.stages < T) {
      const int tn = t + p.stages;
      issue_item<KIND, NB, RW>(p, tn, stage, bars + 8 * s, policy_evict_first(), true, true, true);
    }
  }
}

// ---- host side ------------------------------------------------------------------------------

struct Plan {
  int kc = 0, nch = 0, ngroups = 0, stages = 0;
  uint32_t seg_stride = 0, stage_bytes = 0, xq_off = 0, xd_off = 0, xs_off = 0, kcb4 = 0;
  size_t smem = 0;
};

int gran_elems(uint32_t kind) { return kind == UGB_Q8_0 ? 128 : 256; }
uint64_t elems_to_bytes(uint32_t kind, uint64_t e) {
  switch (kind) {
    case UGB_Q8_0: return bytes_of<UGB_Q8_0>(e);
    case UGB_Q4_K: return bytes_of<UGB_Q4_K>(e);
    default: return bytes_of<UGB_Q3_K>(e);
  }
}

Plan make_plan(uint32_t kind, int64_t k, int64_t m, int nb, int rw) {
  Plan pl;
  const int gran = gran_elems(kind);
  int nch = static_cast<int>((k + 1023) / 1024);
  int kc = static_cast<int>(round_up((k + nch - 1) / nch, gran));
  if (kc > k) kc = static_cast<int>(k);
  nch = static_cast<int>((k + kc - 1) / kc);
  pl.kc = kc;
  pl.nch = nch;
  const int R = kWarps * rw;
  pl.ngroups = static_cast<int>((m + R - 1) / R);
  pl.seg_stride = static_cast<uint32_t>(round_up(elems_to_bytes(kind, kc) + 32, 16));
  pl.kcb4 = static_cast<uint32_t>(round_up(kc / 32, 4));
  const bool need_sum = kind == UGB_Q4_K;
  uint32_t off = R * pl.seg_stride;
  pl.xq_off = off;
  off += nb * kc;
  pl.xd_off = off;
  off += nb * pl.kcb4 * 4;
  pl.xs_off = off;
  if (need_sum) off += nb * pl.kcb4 * 4;
  pl.stage_bytes = static_cast<uint32_t>(round_up(off, 128));
  int stages = static_cast<int>((48 * 1024 + pl.stage_bytes - 1) / pl.stage_bytes);
  stages = std::max(2, std::min(8, stages));
  pl.stages = stages;
  pl.smem = kBarBytes + static_cast<size_t>(stages) * pl.stage_bytes;
  return pl;
}

template <int KIND, int NB, int RW, bool DOTS>
const void *kernel_ptr() {
  return reinterpret_cast<const void *>(&mv_stream_kernel<KIND, NB, RW, DOTS>);
}

const void *select_kernel(uint32_t kind, int nb, bool dots) {
#define UGB_MV_CASE(K)                                                 \
  if (kind == K) {                                                     \
    if (dots) return kernel_ptr<K, 1, 1, true>();                      \
    switch (nb) {                                                      \
      case 1: return kernel_ptr<K, 1, 1, false>();                     \
      case 2: return kernel_ptr<K, 2, 1, false>();                     \
      case 4: return kernel_ptr<K, 4, 1, false>();                     \
      case 8: return kernel_ptr<K, 8, 1, false>();                     \
      default: return nullptr;                                         \
    }                                                                  \
  }
  UGB_MV_CASE(UGB_Q8_0)
  UGB_MV_CASE(UGB_Q4_K)
  UGB_MV_CASE(UGB_Q3_K)
#undef UGB_MV_CASE
  return nullptr;
}

}  // namespace

ugb_status init_matvec_kernels(ugb_ctx *ctx) {
  for (uint32_t kind : {UGB_Q8_0, UGB_Q4_K, UGB_Q3_K}) {
    for (int nb : {1, 2, 4, 8}) {
      const void *f = select_kernel(kind, nb, false);
      if (cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(ctx->smem_optin)) != cudaSuccess)
        return UGB_EBACKEND;
    }
    const void *f = select_kernel(kind, 1, true);
    if (cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(ctx->smem_optin)) != cudaSuccess)
      return UGB_EBACKEND;
  }
  return UGB_OK;
}

ugb_status launch_matvec(ugb_ctx *ctx, cudaStream_t stream, const MatvecArgs &a) {
  const bool dots = a.dots != nullptr;
  // A batch that is not 1, 2, 4 or 8 runs as several launches of those sizes (largest
  // first), each streaming the weights once.
  int64_t done = 0;
  while (done < a.batch) {
    const int64_t rest = a.batch - done;
    const int nb = dots ? 1 : (rest >= 8 ? 8 : rest >= 4 ? 4 : rest >= 2 ? 2 : 1);
    const Plan pl = make_plan(a.kind, a.k, a.m, nb, 1);
    if (pl.smem > ctx->smem_optin) return UGB_ESHAPE;
    const void *f = select_kernel(a.kind, nb, dots);
    if (!f) return UGB_EQUANT;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, f, kThreads, pl.smem) != cudaSuccess ||
        per_sm < 1)
      return UGB_EBACKEND;
    MvParams p{};
    p.w = a.w;
    p.w_end = a.w + a.m * a.row_bytes;
    p.w_end16 = reinterpret_cast<const uint8_t *>(reinterpret_cast<uintptr_t>(p.w_end) & ~uintptr_t(15));
    p.row_bytes = static_cast<uint64_t>(a.row_bytes);
    p.k = static_cast<int>(a.k);
    p.m = static_cast<int>(a.m);
    p.batch = nb;
    p.kc = pl.kc;
    p.nch = pl.nch;
    p.ngroups = pl.ngroups;
    p.seg_stride = pl.seg_stride;
    p.stage_bytes = pl.stage_bytes;
    p.xq_off = pl.xq_off;
    p.xd_off = pl.xd_off;
    p.xs_off = pl.xs_off;
    p.kcb4 = pl.kcb4;
    p.stages = pl.stages;
    p.xq = a.xq + done * a.xl.k;
    p.xd = reinterpret_cast<const float *>(a.xq + a.xl.d_off) + done * a.xl.nbp;
    p.xs = reinterpret_cast<const int *>(a.xq + a.xl.s_off) + done * a.xl.nbp;
    p.xq_stride = a.xl.k;
    p.xds_stride = a.xl.nbp;
    p.y = a.y ? a.y + done * a.ldy : nullptr;
    p.ldy = a.ldy;
    p.dots = a.dots;
    p.dots_ld = a.k / 32;
    p.status = ctx->status;
    const int grid = static_cast<int>(std::min<int64_t>(pl.ngroups, static_cast<int64_t>(ctx->sm_count) * per_sm));

    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = pl.smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = a.pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    void *args[] = {&p};
    if (cudaLaunchKernelExC(&cfg, f, args) != cudaSuccess) return UGB_EBACKEND;
    done += nb;
  }
  return UGB_OK;
}

}  // namespace ugb
