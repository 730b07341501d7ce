// matvec.cu -- HBM-streaming block-quantised matvec for decode (Q8_0 / Q4_K / Q3_K x Q8_1).
//
// Replaces linear_dp4a / qkv_dp4a / gateup_dp4a (gpu_dp4a.cu:32-64) and frontier_matvec
// (frontier_quant.cu:58-66).  Design for sm_100a:
//  * Persistent CTAs, 8 consumer warps + 1 producer warp, coupled only through per-stage
//    full / empty mbarriers (no CTA-wide barrier per item; every wait is bounded and a lost
//    copy sets UGB_STATUS_TIMEOUT instead of hanging).
//  * The producer streams work items -- groups of consecutive rows, in the unchanged GGUF
//    byte layout -- into a multi-stage shared-memory ring with cp.async.bulk (one copy per
//    item when whole rows fit a stage, one per row chunk otherwise), weights carrying an L2
//    evict-first hint since each byte is read once.  The first stages are requested before
//    the programmatic launch dependency resolves, overlapping the previous kernel's tail.
//  * The Q8_1 activation is bulk-copied into shared memory once per CTA.
//  * Consumers:
//    - mv_rows_kernel (batch 1, whole rows): each warp owns RW rows; lane l covers slots
//      l, l+32, ... of the warp's flattened (row, 32-element unit) space, keeps the matching
//      activation units in registers for the whole kernel (every item spans the whole row),
//      and the RW row totals come out of one transposed shuffle tree.  This keeps the
//      per-row instruction overhead small enough to stream at HBM speed.  Its burst form
//      (matrices whose rows fit one CTA per SM) has no producer warp: every item gets its own
//      stage and all copies go out first, at about half an SM, so the next launch becomes
//      resident beside it; it can also quantise an fp32 activation itself (ugb_matvec_f32).
//    - mv_split_kernel (batch 1, rows too long for whole rows per warp): an item's rows are
//      spread over all consumer lanes, partials meet through a named-barrier reduction.
//    - mv_stream_kernel (batches, long rows split into K chunks, int-dot dumps): RW rows per
//      warp share each activation unit read from shared memory, row sums kept in registers
//      across the row's chunks.
//  * Integer block dots are exact (dp4a); the fp32 accumulation order is fixed, so results
//    are deterministic run to run.
#include <algorithm>
#include <cmath>

#include "formats.cuh"
#include "glue.cuh"
#include "internal.hpp"

namespace ugb {
namespace {

constexpr int kWarps = 8;                    // consumer warps per CTA
constexpr int kThreads = kWarps * 32 + 32;   // + one producer warp
constexpr uint32_t kBarBytes = 256;          // mbarriers at the start of dynamic shared memory
constexpr int kMaxStages = 8;
constexpr size_t kXBudget = 100 * 1024;      // activation bytes staged per CTA
constexpr uint32_t kItemTarget = 32 * 1024;  // weight bytes per pipeline stage
constexpr size_t kSmPerKernel = 112 * 1024;  // shared memory one kernel takes per SM
constexpr int kSlots = 4;                    // activation units a lane keeps in registers

constexpr int kMaxSegs = kMaxMatvecSegs;  // matrices sharing one activation in one launch
constexpr int kMaxJobs = kMaxMatvecJobs;  // jobs of one job-table launch

// How a launch maps CTAs to matrices:
//  kSegments -- up to kMaxSegs matrices share one activation; their rows are concatenated and
//               every CTA walks row groups of the whole set (fused Q/K/V, gate/up);
//  kTable    -- up to kMaxSegs independent jobs, each with its own activation and output
//               (the reference's FrontierJob table, frontier_quant.cu:71-93); CTAs
//               [cta0[j], cta0[j+1]) serve job j only;
//  kRouted   -- expert jobs resolved on the device: slot s uses expert ids[s] of a stacked
//               expert tensor (GGUF *_exps, experts contiguous), cpj CTAs per job.
enum MvMode : int { kSegments = 0, kTable = 1, kRouted = 2 };

struct MvParams {
  // Rows [seg_row0[i], seg_row0[i+1]) live in matrix w[i] (the reference's fused QKV /
  // gate-up launches over separate GGUF tensors, gpu_dp4a.cu:53-64).  An item never spans
  // two matrices.  w_end16[i]: end of matrix i rounded down to 16 bytes.
  const uint8_t *w[kMaxSegs];
  const uint8_t *w_end16[kMaxSegs];
  int seg_row0[kMaxSegs];
  int nseg;
  uint64_t row_bytes;
  int k, m;
  int rows;                   // rows per item (8 * rows-per-warp)
  int kc, nch, ngroups;       // K chunk (elements), chunks per row, row groups (items / nch)
  uint32_t seg_stride, stage_bytes;
  int stages;
  uint32_t x_q, x_d, x_s;     // shared offsets of the staged activation arrays
  uint32_t ring;              // shared offset of the weight ring
  uint32_t red;               // shared offset of cross-warp row partials (split kernel)
  const uint8_t *xq;          // Q8_1 buffer: quants [nb][k], scales / sums [nb][nbp]
  const float *xd;
  const int *xs;
  const float *xf;            // burst launches only: fp32 activation quantised by every CTA
  int nbp;
  float *y;
  int64_t ldy;
  int32_t *dots;
  uint32_t *status;
  int mode;                   // MvMode
  // kRouted: job j = (slot s = j / per_slot, matrix i = j % per_slot); expert e = ids[s]
  // (0 <= e < n_total; a slot whose expert another device holds is skipped); weights
  // ebase[i] + (e - expert0) * estride (m rows); activation vector s / x_div of the Q8_1
  // buffer (xq, xd, xs); output y + s * y_slot + i * m.
  const int32_t *ids;
  int per_slot, n_expert, x_div, cpj;
  int expert0, n_total;       // this device holds global experts [expert0, expert0 + n_expert)
  const uint8_t *ebase[2];
  uint64_t estride;
  int64_t y_slot;
};

// kTable launches carry the job table in a larger parameter block of their own, so the
// frequent segment / routed launches keep a small one (a larger block costs launch latency
// on every one of the hundreds of launches of a decode step).
// Job j = matrix jw[j] of jm[j] rows, activation (jxq, jxd, jxs)[j], output jy[j]
// ([batch][jm[j]]), CTAs [cta0[j], cta0[j+1]).
struct MvTable {
  int njobs;
  int jm[kMaxJobs];
  int cta0[kMaxJobs + 1];
  const uint8_t *jw[kMaxJobs];
  const uint8_t *jw_end16[kMaxJobs];
  const uint8_t *jxq[kMaxJobs];
  const float *jxd[kMaxJobs];
  const int *jxs[kMaxJobs];
  float *jy[kMaxJobs];
};
struct MvParamsT : MvParams {
  MvTable t;
};

// What one CTA works on: its index among the CTAs of its matrix (set), that matrix's rows,
// weights (job modes), activation and output.  Rows are global over the segments in
// kSegments mode and local to the job otherwise; y is indexed by that row either way.
struct View {
  bool skip;                  // routed slot of an expert this device does not hold
  int cta, ncta, m, ngroups;
  const uint8_t *w, *w_end16;
  const uint8_t *xq;
  const float *xd;
  const int *xs;
  float *y;
  int64_t ldy;
};

__device__ __forceinline__ const uint8_t *floor16(const uint8_t *p);

// kRouted reads the expert ids the previous kernel wrote: call after grid_dep_wait().
__device__ __forceinline__ View make_view(const MvParams &p);

__device__ __forceinline__ View make_view(const MvParamsT &p) {
  if (p.mode != kTable) return make_view(static_cast<const MvParams &>(p));
  View v;
  v.skip = false;
  const MvTable &t = p.t;
  int j = 0;
  for (int i = 1; i < t.njobs; ++i) j += static_cast<int>(blockIdx.x) >= t.cta0[i] ? 1 : 0;
  v.cta = static_cast<int>(blockIdx.x) - t.cta0[j];
  v.ncta = t.cta0[j + 1] - t.cta0[j];
  v.m = t.jm[j];
  v.ngroups = (v.m + p.rows - 1) / p.rows;
  v.w = t.jw[j];
  v.w_end16 = t.jw_end16[j];
  v.xq = t.jxq[j];
  v.xd = t.jxd[j];
  v.xs = t.jxs[j];
  v.y = t.jy[j];
  v.ldy = v.m;
  return v;
}

__device__ __forceinline__ View make_view(const MvParams &p) {
  View v;
  v.ldy = p.ldy;
  v.skip = false;
  if (p.mode == kSegments) {
    v.cta = blockIdx.x;
    v.ncta = gridDim.x;
    v.m = p.m;
    v.ngroups = p.ngroups;
    v.w = v.w_end16 = nullptr;
    v.xq = p.xq;
    v.xd = p.xd;
    v.xs = p.xs;
    v.y = p.y;
  } else {
    const int j = static_cast<int>(blockIdx.x) / p.cpj;
    v.cta = static_cast<int>(blockIdx.x) - j * p.cpj;
    v.ncta = p.cpj;
    const int s = j / p.per_slot, i = j - s * p.per_slot;
    const int e = p.ids[s];
    if (e < 0 || e >= p.n_total) {  // never index outside the expert tensor
      if (v.cta == 0 && threadIdx.x == 0) status_or(p.status, ST_BADARG);
      v.skip = true;
    }
    const int el = e - p.expert0;
    if (el < 0 || el >= p.n_expert) v.skip = true;
    v.m = p.m;
    v.ngroups = p.ngroups;
    v.w = p.ebase[i] + static_cast<uint64_t>(v.skip ? 0 : el) * p.estride;
    v.w_end16 = floor16(v.w + static_cast<uint64_t>(p.m) * p.row_bytes);
    const int xv = s / p.x_div;
    v.xq = p.xq + static_cast<int64_t>(xv) * p.k;
    v.xd = p.xd + static_cast<int64_t>(xv) * p.nbp;
    v.xs = p.xs + static_cast<int64_t>(xv) * p.nbp;
    v.y = p.y + static_cast<int64_t>(s) * p.y_slot + static_cast<int64_t>(i) * p.m;
  }
  return v;
}

template <int KIND>
__host__ __device__ constexpr uint64_t bytes_of(uint64_t elems) {
  return elems / Fmt<KIND>::kElems * Fmt<KIND>::kBytes;
}

__device__ __forceinline__ const uint8_t *floor16(const uint8_t *p) {
  return reinterpret_cast<const uint8_t *>(reinterpret_cast<uintptr_t>(p) & ~uintptr_t(15));
}
__device__ __forceinline__ const uint8_t *ceil16(const uint8_t *p) {
  return reinterpret_cast<const uint8_t *>((reinterpret_cast<uintptr_t>(p) + 15) & ~uintptr_t(15));
}

// Geometry of item t of this CTA: rows [r0, r0+nrows), K chunk c.  A CTA owns whole row
// groups (g = blockIdx.x, blockIdx.x + gridDim.x, ...) and walks each group's K chunks in
// order, so a row's partial sums stay in the owning warp's registers across its chunks.
struct Item {
  int r0, nrows, c;
};
__device__ __forceinline__ Item item_of(const MvParams &p, const View &v, int t) {
  const int j = p.nch == 1 ? t : t / p.nch;
  const int g = v.cta + j * v.ncta;
  Item it;
  it.c = t - j * p.nch;
  it.r0 = g * p.rows;
  it.nrows = min(p.rows, v.m - it.r0);
  return it;
}

// Items of this CTA: its row groups times the K chunks of each.
__device__ __forceinline__ int items_of(const MvParams &p, const View &v) {
  return (v.ngroups - v.cta + v.ncta - 1) / v.ncta * p.nch;
}

__device__ __forceinline__ int seg_of(const MvParams &p, int row) {
  int s = 0;
#pragma unroll
  for (int i = 1; i < kMaxSegs; ++i) s += (i < p.nseg && row >= p.seg_row0[i]) ? 1 : 0;
  return s;
}

// Address of row `row` (global across the segments, or of the CTA's job).
__device__ __forceinline__ const uint8_t *row_ptr(const MvParams &p, const View &v, int row) {
  if (p.mode != kSegments) return v.w + static_cast<uint64_t>(row) * p.row_bytes;
  const int s = seg_of(p, row);
  return p.w[s] + static_cast<uint64_t>(row - p.seg_row0[s]) * p.row_bytes;
}

// Byte range [a0, a1) a bulk copy may fetch for the span [src, e) of matrix `seg`: 16-byte
// aligned, and never past the last 16-byte boundary of that matrix; the bytes beyond (only in
// a matrix's final span) go through plain loads.
__device__ __forceinline__ void span16(const MvParams &p, const View &v, int seg, const uint8_t *src,
                                       const uint8_t *e, const uint8_t *&a0, const uint8_t *&a1) {
  const uint8_t *end16 = p.mode == kSegments ? p.w_end16[seg] : v.w_end16;
  a0 = floor16(src);
  a1 = ceil16(e);
  if (e > end16) a1 = a0 > end16 ? a0 : end16;
}

// Copies of item t into `stage` (one thread).  When a row chunk is the whole row (nch == 1)
// the item's rows are one contiguous span and one bulk copy fetches all of them.
template <int KIND>
__device__ void issue_item(const MvParams &p, const View &v, int t, uint32_t stage, uint32_t bar, uint64_t pol) {
  const Item it = item_of(p, v, t);
  const int seg = p.mode == kSegments ? seg_of(p, it.r0) : 0;
  const uint8_t *first = row_ptr(p, v, it.r0);
  const uint64_t seg_off = bytes_of<KIND>(static_cast<uint64_t>(it.c) * p.kc);
  const uint64_t seg_len = bytes_of<KIND>(min(p.kc, p.k - it.c * p.kc));
  const int spans = p.nch == 1 ? 1 : it.nrows;
  uint32_t tx = 0;
  for (int r = 0; r < spans; ++r) {
    const uint8_t *src = first + static_cast<uint64_t>(r) * p.row_bytes + seg_off;
    const uint8_t *e = p.nch == 1 ? first + static_cast<uint64_t>(it.nrows) * p.row_bytes : src + seg_len;
    const uint8_t *a0, *a1;
    span16(p, v, seg, src, e, a0, a1);
    const uint32_t dst = stage + r * p.seg_stride;
    for (const uint8_t *b = a1; b < e; ++b) sts8(dst + static_cast<uint32_t>(b - a0), *b);
    tx += static_cast<uint32_t>(a1 - a0);
  }
  mbar_arrive_expect_tx(bar, tx);
  for (int r = 0; r < spans; ++r) {
    const uint8_t *src = first + static_cast<uint64_t>(r) * p.row_bytes + seg_off;
    const uint8_t *e = p.nch == 1 ? first + static_cast<uint64_t>(it.nrows) * p.row_bytes : src + seg_len;
    const uint8_t *a0, *a1;
    span16(p, v, seg, src, e, a0, a1);
    if (a1 > a0) bulk_g2s(stage + r * p.seg_stride, a0, static_cast<uint32_t>(a1 - a0), bar, pol);
  }
}

// Shared prologue: barriers, programmatic-launch hand-off, the producer warp's whole life,
// and the activation staging.  Returns false in the producer warp (which is done), true in
// consumer warps once the activation is in shared memory (ok = false if that copy timed out).
template <int KIND, int NB>
__device__ __forceinline__ bool prologue(const MvParams &p, const View &v, uint32_t base, int T, bool &ok) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t full = base, empty = base + 64, xbar = base + 128;
  const uint32_t ring = base + p.ring;
  constexpr bool kSum = Fmt<KIND>::kNeedsSum;
  const uint32_t xq_bytes = static_cast<uint32_t>(p.k), xd_bytes = static_cast<uint32_t>(p.nbp) * 4;
  const int pre = min(T, p.stages);
  grid_dep_launch();  // the next kernel may become resident beside this one and start its own copies
  if (tid == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(full + 8 * s, 1);
      mbar_init(empty + 8 * s, kWarps);
    }
    mbar_init(xbar, 1);
    fence_mbar_init();
    // Weights do not depend on earlier kernels: the first stages are requested before anything
    // else, and before the programmatic dependency resolves.  The copy engine takes them one
    // after another, so the sooner the first is issued, the sooner HBM is busy.
    const uint64_t pol_w = policy_evict_first();
    for (int t = 0; t < pre; ++t) issue_item<KIND>(p, v, t, ring + t * p.stage_bytes, full + 8 * t, pol_w);
  }
  __syncthreads();
  if (warp == kWarps) {
    if (lane == 0) {
      // then the activation, once for the CTA, and the items that wait for a free stage
      grid_dep_wait();
      mbar_arrive_expect_tx(xbar, NB * (xq_bytes + xd_bytes * (kSum ? 2u : 1u)));
      const uint64_t pol_x = policy_evict_last();
      for (int b = 0; b < NB; ++b) {
        bulk_g2s(base + p.x_q + b * xq_bytes, v.xq + static_cast<int64_t>(b) * p.k, xq_bytes, xbar, pol_x);
        bulk_g2s(base + p.x_d + b * xd_bytes, v.xd + static_cast<int64_t>(b) * p.nbp, xd_bytes, xbar, pol_x);
        if (kSum) bulk_g2s(base + p.x_s + b * xd_bytes, v.xs + static_cast<int64_t>(b) * p.nbp, xd_bytes, xbar, pol_x);
      }
      const uint64_t pol_w = policy_evict_first();
      for (int t = pre; t < T; ++t) {
        const int s = t % p.stages;
        if (!mbar_wait_bounded(empty + 8 * s, ((t / p.stages) - 1) & 1)) {
          status_or(p.status, ST_TIMEOUT);
          break;
        }
        issue_item<KIND>(p, v, t, ring + s * p.stage_bytes, full + 8 * s, pol_w);
      }
    }
    return false;
  }
  grid_dep_wait();  // consumers read the activation and write y only after the dependency
  ok = __all_sync(0xffffffffu, mbar_wait_bounded(xbar, 0));
  if (!ok && lane == 0) status_or(p.status, ST_TIMEOUT);
  return true;
}

// Prologue of a burst launch (no producer warp): every item of the CTA has a stage of its own,
// so all weight copies go out at once, first thing, and nothing is ever released.  Thread 0
// requests the weights while thread 32 waits for the dependency and stages the activation.
template <int KIND>
__device__ __forceinline__ bool prologue_burst(const MvParams &p, const View &v, uint32_t base, int T, bool &ok) {
  const int tid = threadIdx.x, lane = tid & 31;
  const uint32_t full = base, xbar = base + 128;
  constexpr bool kSum = Fmt<KIND>::kNeedsSum;
  grid_dep_launch();  // the next kernel may become resident beside this one and start its copies
  if (tid == 0) {
    for (int t = 0; t < T; ++t) mbar_init(full + 8 * t, 1);
    mbar_init(xbar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (tid == 0) {
    const uint64_t pol_w = policy_evict_first();
    for (int t = 0; t < T; ++t) issue_item<KIND>(p, v, t, base + p.ring + t * p.stage_bytes, full + 8 * t, pol_w);
  } else if (tid == 32 && p.xf == nullptr) {
    const uint32_t xq_bytes = static_cast<uint32_t>(p.k), xd_bytes = static_cast<uint32_t>(p.nbp) * 4;
    grid_dep_wait();
    mbar_arrive_expect_tx(xbar, xq_bytes + xd_bytes * (kSum ? 2u : 1u));
    const uint64_t pol_x = policy_evict_last();
    bulk_g2s(base + p.x_q, v.xq, xq_bytes, xbar, pol_x);
    bulk_g2s(base + p.x_d, v.xd, xd_bytes, xbar, pol_x);
    if (kSum) bulk_g2s(base + p.x_s, v.xs, xd_bytes, xbar, pol_x);
  }
  grid_dep_wait();  // the activation is read and y written only after the dependency
  if (p.xf != nullptr) {
    // The fp32 activation, quantised into shared memory by every CTA: quant_q8_1_kernel's
    // arithmetic bit for bit (glue.cuh), eight blocks per warp at a time, loads first.
    constexpr int kQB = 8;
    const int warp = tid >> 5, nb = p.k / 32;
    uint8_t *smem = reinterpret_cast<uint8_t *>(__cvta_shared_to_generic(base));
    int8_t *q = reinterpret_cast<int8_t *>(smem + p.x_q);
    float *d = reinterpret_cast<float *>(smem + p.x_d);
    int32_t *sm = reinterpret_cast<int32_t *>(smem + p.x_s);
    bool bad = false;
    for (int b0 = warp; b0 < nb; b0 += kWarps * kQB) {
      float xv[kQB];
      int bb[kQB];
      bool live[kQB];
#pragma unroll
      for (int i = 0; i < kQB; ++i) {
        bb[i] = b0 + i * kWarps;
        live[i] = bb[i] < nb;
        xv[i] = p.xf[static_cast<int64_t>(live[i] ? bb[i] : b0) * 32 + lane];
      }
      bad |= quant_blocks<kQB>(xv, bb, live, lane, q, d, sm);
    }
    if (bad && lane == 0) status_or(p.status, ST_NONFINITE_IN);
    __syncthreads();
    ok = true;
    return true;
  }
  ok = __all_sync(0xffffffffu, mbar_wait_bounded(xbar, 0));
  if (!ok && lane == 0) status_or(p.status, ST_TIMEOUT);
  return true;
}

// Wait for stage s of item t; false (and the status bit) if it never arrives.
__device__ __forceinline__ bool wait_stage(const MvParams &p, uint32_t full, int t, int lane) {
  const bool ok = __all_sync(0xffffffffu, mbar_wait_bounded(full + 8 * (t % p.stages), (t / p.stages) & 1));
  if (!ok && lane == 0) status_or(p.status, ST_TIMEOUT);
  return ok;
}

// Hand stage s back to the producer.  Every read of it has completed (the values were
// consumed by the arithmetic before this point); a relaxed arrive avoids waiting for this
// thread's earlier global stores.
__device__ __forceinline__ void release_stage(uint32_t empty, int s, int lane) {
  __syncwarp();
  if (lane == 0) mbar_arrive_relaxed(empty + 8 * s);
}

// Batch-1, whole-row consumer (see the file comment).  RW rows per warp, 8 * RW per item.
// BURST: the launch gives every item of a CTA its own stage (one CTA per SM, about half its
// shared memory and registers), so there is no producer warp and no stage reuse, and the next
// kernel in the stream fits beside this one and streams its own weights meanwhile.
template <int KIND, int RW, int J, class P, bool BURST>
__global__ void __launch_bounds__(BURST ? kWarps * 32 : kThreads, 2) mv_rows_kernel(const P p) {
  static_assert(J >= 2 && J <= kSlots, "2 to kSlots register slots");
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t base = smem_u32(smem);
  const uint32_t full = base, empty = base + 64;
  const uint32_t ring = base + p.ring;
  if (p.mode == kRouted) grid_dep_wait();  // the expert ids come from the previous kernel
  const View v = make_view(p);
  if (v.skip) return;  // nothing staged or issued yet
  const int T = items_of(p, v);
  bool ok = true;
  if constexpr (BURST) {
    prologue_burst<KIND>(p, v, base, T, ok);
  } else {
    if (!prologue<KIND, 1>(p, v, base, T, ok)) return;
  }

  // Slot j of this lane is flat index f = lane + 32 j of the warp's RW x U (row, unit) space.
  // Its row offset inside an item, its unit and its activation unit are fixed for the kernel.
  const int U = p.k / 32;
  const int total = RW * U;
  uint32_t srow_off[J];
  int sunit[J], srow[J];
  XUnit xr[J];
#pragma unroll
  for (int j = 0; j < J; ++j) {
    const int f = lane + 32 * j;
    const bool valid = f < total;
    const int r = valid ? f / U : 0;
    const int u = valid ? f - r * U : 0;
    srow[j] = valid ? r : RW;  // RW matches no row: the slot adds nothing
    sunit[j] = u;
    srow_off[j] = static_cast<uint32_t>((warp * RW + r) * p.row_bytes);
    load_xunit(base + p.x_q + 32 * u, base + p.x_d + 4 * u, base + p.x_s + 4 * u,
               Fmt<KIND>::kNeedsSum, xr[j]);
  }

  // The slot dots of one item (staged at `stage`) and the row totals of an item's group.
  auto item_acc = [&](uint32_t stage, float (&acc)[J]) {
#pragma unroll
    for (int j = 0; j + 1 < J; j += 2) {
      acc[j] = acc[j + 1] = 0.f;
      if (j * 32 < total) {  // warp-uniform
        WUnit wa, wb;
        load_wunit<KIND>(stage + srow_off[j], sunit[j], wa);
        load_wunit<KIND>(stage + srow_off[j + 1], sunit[j + 1], wb);
        const int ia = unit_isum<KIND>(wa, xr[j]);
        const int ib = unit_isum<KIND>(wb, xr[j + 1]);
        acc[j] = unit_term<KIND>(wa, xr[j], ia);
        acc[j + 1] = unit_term<KIND>(wb, xr[j + 1], ib);
      }
    }
    if constexpr (J % 2 == 1) {  // odd slot count: the last slot alone
      constexpr int j = J - 1;
      acc[j] = 0.f;
      if (j * 32 < total) {
        WUnit wa;
        load_wunit<KIND>(stage + srow_off[j], sunit[j], wa);
        acc[j] = unit_term<KIND>(wa, xr[j], unit_isum<KIND>(wa, xr[j]));
      }
    }
  };
  auto item_out = [&](const Item &it, const float (&acc)[J], bool live) {
    float rs[RW];
#pragma unroll
    for (int r = 0; r < RW; ++r) {
      rs[r] = 0.f;
#pragma unroll
      for (int j = 0; j < J; ++j) rs[r] += srow[j] == r ? acc[j] : 0.f;
    }
    float tot;
    if (reduce_rows<RW>(rs, lane, tot) && live) {
      const int rr = warp * RW + lane / (32 / RW);
      if (rr < it.nrows) {
        v.y[it.r0 + rr] = tot;
        if (!isfinite(tot)) status_or(p.status, ST_NONFINITE_OUT);
      }
    }
  };
  // The item's rows are one span fetched from floor16(first row).
  auto stage_of = [&](int t, const Item &it) {
    return ring + (t % p.stages) * p.stage_bytes +
           static_cast<uint32_t>(reinterpret_cast<uintptr_t>(row_ptr(p, v, it.r0)) & 15);
  };

  if constexpr (BURST) {
    // Items two at a time: every item is already requested, and the two groups' dependency
    // chains (shared-memory loads, dp4a, the shuffle tree) interleave.  With an odd count the
    // last pair repeats its first item and drops the copy.
    for (int t = 0; ok && t < T; t += 2) {
      const bool two = t + 1 < T;
      const int t1 = two ? t + 1 : t;
      ok = wait_stage(p, full, t, lane) && wait_stage(p, full, t1, lane);
      if (!ok) break;
      const Item i0 = item_of(p, v, t), i1 = item_of(p, v, t1);
      float a0[J], a1[J];
      item_acc(stage_of(t, i0), a0);
      item_acc(stage_of(t1, i1), a1);
      item_out(i0, a0, true);
      item_out(i1, a1, two);
    }
  } else {
    for (int t = 0; ok && t < T; ++t) {
      ok = wait_stage(p, full, t, lane);
      if (!ok) break;
      const Item it = item_of(p, v, t);
      float acc[J];
      item_acc(stage_of(t, it), acc);
      release_stage(empty, t % p.stages, lane);
      item_out(it, acc, true);
    }
  }
}

// Batch-1 consumer for rows too long to give each warp whole rows: an item of R rows is
// spread over all 256 consumer lanes (flat index f = warp * 32 + lane + 256 j of the item's
// R x U (row, unit) space), activation units again held in registers.  Each warp reduces its
// share of the R rows; the per-warp partials meet in shared memory (double-buffered by item
// parity) and warp 0 adds them in warp order.  The one named barrier per item also ANDs the
// warps' wait results, so a timed-out stage makes every consumer warp stop together.
template <int KIND, int R, int J, class P>
__global__ void __launch_bounds__(kThreads, 1) mv_split_kernel(const P p) {
  static_assert(J % 2 == 0 && J <= kSlots, "slots are processed in pairs");
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t base = smem_u32(smem);
  const uint32_t full = base, empty = base + 64;
  const uint32_t ring = base + p.ring;
  if (p.mode == kRouted) grid_dep_wait();  // the expert ids come from the previous kernel
  const View v = make_view(p);
  if (v.skip) return;  // nothing staged or issued yet
  const int T = items_of(p, v);
  bool ok = true;
  if (!prologue<KIND, 1>(p, v, base, T, ok)) return;

  const int U = p.k / 32;
  const int total = R * U;
  uint32_t srow_off[J];
  int sunit[J], srow[J];
  XUnit xr[J];
#pragma unroll
  for (int j = 0; j < J; ++j) {
    const int f = warp * 32 + lane + kWarps * 32 * j;
    const bool valid = f < total;
    const int r = valid ? f / U : 0;
    const int u = valid ? f - r * U : 0;
    srow[j] = valid ? r : R;  // R matches no row: the slot adds nothing
    sunit[j] = u;
    srow_off[j] = static_cast<uint32_t>(r * p.row_bytes);
    load_xunit(base + p.x_q + 32 * u, base + p.x_d + 4 * u, base + p.x_s + 4 * u,
               Fmt<KIND>::kNeedsSum, xr[j]);
  }
  float *red = reinterpret_cast<float *>(smem + p.red);

  for (int t = 0; t < T; ++t) {
    const int s = t % p.stages;
    const bool mine = __all_sync(0xffffffffu, mbar_wait_bounded(full + 8 * s, (t / p.stages) & 1));
    const Item it = item_of(p, v, t);
    float rs[R];
#pragma unroll
    for (int r = 0; r < R; ++r) rs[r] = 0.f;
    if (mine) {
      const uint32_t stage = ring + s * p.stage_bytes +
          static_cast<uint32_t>(reinterpret_cast<uintptr_t>(row_ptr(p, v, it.r0)) & 15);
      float acc[J];
#pragma unroll
      for (int j = 0; j < J; j += 2) {
        acc[j] = acc[j + 1] = 0.f;
        if ((warp * 32 + kWarps * 32 * j) < total) {  // warp-uniform
          WUnit wa, wb;
          load_wunit<KIND>(stage + srow_off[j], sunit[j], wa);
          load_wunit<KIND>(stage + srow_off[j + 1], sunit[j + 1], wb);
          acc[j] = unit_term<KIND>(wa, xr[j], unit_isum<KIND>(wa, xr[j]));
          acc[j + 1] = unit_term<KIND>(wb, xr[j + 1], unit_isum<KIND>(wb, xr[j + 1]));
        }
      }
      release_stage(empty, s, lane);
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int j = 0; j < J; ++j) rs[r] += srow[j] == r ? acc[j] : 0.f;
    }
    float tot;
    const bool owner = reduce_rows<R>(rs, lane, tot);
    if (owner) red[((t & 1) * kWarps + warp) * 4 + lane / (32 / R)] = tot;
    uint32_t all;
    asm volatile(
        "{\n\t.reg .pred pi, po;\n\tsetp.ne.u32 pi, %1, 0;\n\t"
        "bar.red.and.pred po, 1, %2, pi;\n\tselp.u32 %0, 1, 0, po;\n\t}"
        : "=r"(all)
        : "r"(mine ? 1u : 0u), "r"(kWarps * 32)
        : "memory");
    if (!all) {
      if (!mine && lane == 0) status_or(p.status, ST_TIMEOUT);
      break;
    }
    if (warp == 0 && lane < R && lane < it.nrows) {
      float sum = 0.f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) sum += red[((t & 1) * kWarps + w) * 4 + lane];
      v.y[it.r0 + lane] = sum;
      if (!isfinite(sum)) status_or(p.status, ST_NONFINITE_OUT);
    }
  }
}

// General consumer: NB activation vectors, rows of any length (K chunks), or int-dot dumps
// (DOTS).  Warp w owns rows w * RW .. w * RW + RW - 1 of every item (8 * RW rows per item);
// lane l takes 32-element units l, l+32, ... of the chunk.  The NB activation units of a unit
// are read from shared memory once and serve all RW rows: with batches those reads, not the
// weights, are what the shared-memory bandwidth goes to.
template <int KIND, int NB, bool DOTS, class P, int RW>
__global__ void __launch_bounds__(kThreads, 1) mv_stream_kernel(const P p) {
  static_assert(!DOTS || (NB == 1 && RW == 1), "block dots are dumped one row per warp");
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t base = smem_u32(smem);
  const uint32_t full = base, empty = base + 64;
  const uint32_t ring = base + p.ring;
  if (p.mode == kRouted) grid_dep_wait();  // the expert ids come from the previous kernel
  const View v = make_view(p);
  if (v.skip) return;  // nothing staged or issued yet
  const int T = items_of(p, v);
  bool ok = true;
  if (!prologue<KIND, NB>(p, v, base, T, ok)) return;
  constexpr bool kSum = Fmt<KIND>::kNeedsSum;
  const uint32_t xq_bytes = static_cast<uint32_t>(p.k), xd_bytes = static_cast<uint32_t>(p.nbp) * 4;

  float acc[RW][NB];
#pragma unroll
  for (int r = 0; r < RW; ++r)
#pragma unroll
    for (int b = 0; b < NB; ++b) acc[r][b] = 0.f;

  for (int t = 0; ok && t < T; ++t) {
    const int s = t % p.stages;
    ok = wait_stage(p, full, t, lane);
    if (!ok) break;
    const uint32_t stage = ring + s * p.stage_bytes;
    const Item it = item_of(p, v, t);
    const int k0 = it.c * p.kc;
    if (warp * RW < it.nrows) {
      const int nunits = min(p.kc, p.k - k0) / 32;
      const uint64_t seg_off = bytes_of<KIND>(static_cast<uint64_t>(k0));
      const uint8_t *row0 = row_ptr(p, v, it.r0);
      uint32_t seg[RW];
#pragma unroll
      for (int r = 0; r < RW; ++r) {
        const int rr = warp * RW + r;
        const uint8_t *row = row0 + static_cast<uint64_t>(rr) * p.row_bytes + seg_off;
        if (p.nch == 1) {
          seg[r] = stage + static_cast<uint32_t>(row - floor16(row0));
        } else {
          seg[r] = stage + rr * p.seg_stride + static_cast<uint32_t>(reinterpret_cast<uintptr_t>(row) & 15);
        }
      }
      for (int u = lane; u < nunits; u += 32) {
        const int ug = k0 / 32 + u;  // unit index within the whole row
        XUnit x[NB];
#pragma unroll
        for (int b = 0; b < NB; ++b)
          load_xunit(base + p.x_q + b * xq_bytes + 32 * ug, base + p.x_d + b * xd_bytes + 4 * ug,
                     base + p.x_s + b * xd_bytes + 4 * ug, kSum, x[b]);
#pragma unroll
        for (int r = 0; r < RW; ++r) {
          if (warp * RW + r < it.nrows) {  // warp-uniform
            WUnit wu;
            load_wunit<KIND, false>(seg[r], u, wu);
#pragma unroll
            for (int b = 0; b < NB; ++b) {
              const int isum = unit_isum<KIND>(wu, x[b]);
              if constexpr (DOTS) {
                p.dots[static_cast<int64_t>(it.r0 + warp) * (p.k / 32) + ug] = isum;
              } else {
                acc[r][b] += unit_term<KIND>(wu, x[b], isum);
              }
            }
          }
        }
      }
    }
    release_stage(empty, s, lane);
    if (!DOTS && it.c == p.nch - 1) {
#pragma unroll
      for (int r = 0; r < RW; ++r) {
        const int rr = warp * RW + r;
#pragma unroll
        for (int b = 0; b < NB; ++b) {
          const float val = warp_sum(acc[r][b]);
          acc[r][b] = 0.f;
          if (lane == 0 && rr < it.nrows) {
            v.y[b * v.ldy + it.r0 + rr] = val;
            if (!isfinite(val)) status_or(p.status, ST_NONFINITE_OUT);
          }
        }
      }
    }
  }
}

// ---- host side ------------------------------------------------------------------------------

uint64_t elems_to_bytes(uint32_t kind, uint64_t e) {
  switch (kind) {
    case UGB_Q8_0: return bytes_of<UGB_Q8_0>(e);
    case UGB_Q4_K: return bytes_of<UGB_Q4_K>(e);
    case UGB_Q3_K: return bytes_of<UGB_Q3_K>(e);
    case UGB_Q6_K: return bytes_of<UGB_Q6_K>(e);
    case UGB_IQ3_XXS: return bytes_of<UGB_IQ3_XXS>(e);
    case UGB_IQ4_NL: return bytes_of<UGB_IQ4_NL>(e);
    default: return bytes_of<UGB_IQ4_XS>(e);
  }
}

// The configurations' formats get every kernel form; the reference's other formats (Q6_K,
// IQ3_XXS, IQ4_NL, IQ4_XS) go through the streaming kernel, which serves every batch, the job
// table and the routed experts alike.
bool all_forms(uint32_t kind) { return kind == UGB_Q8_0 || kind == UGB_Q4_K || kind == UGB_Q3_K; }

size_t x_bytes(uint32_t kind, int64_t k, int nb) {
  const size_t nbp = round_up(static_cast<uint64_t>(k / 32), 4);
  return static_cast<size_t>(nb) * (static_cast<size_t>(k) + nbp * 4 * (kind == UGB_Q4_K ? 2 : 1));
}

struct Plan {
  bool rows_kernel = false;   // mv_rows_kernel
  bool burst = false;         // its burst form (every item of a CTA staged at once)
  int burst_stages = 0;       // items per CTA when the rows kernel can run as a burst (0: cannot)
  bool split = false;         // mv_split_kernel (neither: mv_stream_kernel)
  int rw = 1, slots = 2;      // rows per warp (rows kernel) or per item (split kernel), and
                              // register slots per lane
  int rows = kWarps, kc = 0, nch = 1, ngroups = 0, stages = 2, ctas_per_sm = 1;
  uint32_t seg_stride = 0, stage_bytes = 0, x_q = 0, x_d = 0, x_s = 0, red = 0, ring = 0;
  size_t smem = 0;
};

Plan make_plan(uint32_t kind, int64_t k, int64_t m, int nb, bool dots, size_t smem_optin, int sm_count) {
  Plan pl;
  const uint64_t rb = elems_to_bytes(kind, static_cast<uint64_t>(k));
  const int64_t units = k / 32;
  // Batch 1, whole rows: the rows kernel with the largest rows-per-warp whose item fits a
  // stage and whose slots fit the register budget.
  if (nb == 1 && !dots && all_forms(kind)) {
    for (int rw : {4, 2, 1}) {
      const int64_t slots = (rw * units + 31) / 32;
      if (rb * kWarps * rw <= kItemTarget && slots <= kSlots) {
        pl.rows_kernel = true;
        pl.rw = rw;
        pl.slots = slots <= 2 ? 2 : static_cast<int>(slots);  // 2, 3 or 4
        break;
      }
    }
    // Rows too long for that: spread an item of R rows over all consumer lanes (the largest
    // R whose item fits a stage and whose slots fit the registers).
    for (int r : {4, 2, 1}) {
      if (pl.rows_kernel || pl.split) break;
      const int64_t slots = (r * units + kWarps * 32 - 1) / (kWarps * 32);
      if (rb * r <= kItemTarget && slots <= kSlots) {
        pl.split = true;
        pl.rw = r;
        pl.slots = slots <= 2 ? 2 : 4;
      }
    }
  }
  if (!pl.rows_kernel && !pl.split && !dots && nb > 1) {
    // Batches: two rows per warp share each activation unit read from shared memory, when
    // that still leaves a row group for every SM (four ran slower: 168 registers and spills
    // at batch 8).
    if ((m + 2 * kWarps - 1) / (2 * kWarps) >= sm_count) pl.rw = 2;
  }
  pl.rows = pl.split ? pl.rw : kWarps * pl.rw;
  auto size_items = [&](uint64_t target) {
    if (rb * pl.rows <= target) {
      pl.kc = static_cast<int>(k);
      pl.nch = 1;
      pl.seg_stride = 0;
      pl.stage_bytes = static_cast<uint32_t>(round_up(rb * pl.rows + 32, 128));
    } else {
      // K chunks sized so the item's row chunks fill about one stage.
      // chunk starts keep x arrays 16B aligned and fall on block boundaries
      const int gran = (kind == UGB_Q8_0 || kind == UGB_IQ4_NL) ? 128 : 256;
      const int nch = static_cast<int>((rb * pl.rows + target - 1) / target);
      pl.kc = static_cast<int>(round_up((k + nch - 1) / nch, gran));
      pl.nch = static_cast<int>((k + pl.kc - 1) / pl.kc);
      pl.seg_stride = static_cast<uint32_t>(round_up(elems_to_bytes(kind, pl.kc) + 32, 16));
      pl.stage_bytes = static_cast<uint32_t>(round_up(static_cast<uint64_t>(pl.rows) * pl.seg_stride, 128));
    }
  };
  // Batches take stages twice as large where two still fit beside the activations: whole rows
  // of the 3584-wide matrices in one copy, and row chunks twice as long otherwise (every chunk
  // of every row is a copy of its own, and short copies do not keep HBM busy).
  const bool batch_stream = !pl.rows_kernel && !pl.split && !dots && nb > 1;
  size_items(batch_stream ? 2 * kItemTarget : kItemTarget);
  pl.ngroups = static_cast<int>((m + pl.rows - 1) / pl.rows);
  const size_t nbp = round_up(static_cast<uint64_t>(k / 32), 4);
  uint32_t off = kBarBytes;
  pl.x_q = off;
  off += static_cast<uint32_t>(round_up(static_cast<uint64_t>(nb) * k, 16));
  pl.x_d = off;
  off += static_cast<uint32_t>(nb * nbp * 4);
  pl.x_s = off;  // sums: read by Q4_K only, but always allocated (the fused quantiser writes them)
  off += static_cast<uint32_t>(nb * nbp * 4);
  pl.red = static_cast<uint32_t>(round_up(off, 16));
  off = pl.red + 2 * kWarps * 4 * 4;
  pl.ring = static_cast<uint32_t>(round_up(off, 128));
  if (batch_stream && pl.ring + 2 * static_cast<size_t>(pl.stage_bytes) > smem_optin) {
    size_items(kItemTarget);
    pl.ngroups = static_cast<int>((m + pl.rows - 1) / pl.rows);
  }
  // One kernel takes at most about half an SM's shared memory (kSmPerKernel over its resident
  // CTAs), so the next kernel in the stream can become resident beside it and prefetch its
  // weights under programmatic dependent launch.
  pl.ctas_per_sm = pl.ring + 2 * static_cast<size_t>(pl.stage_bytes) <= kSmPerKernel / 2 ? 2 : 1;
  const size_t budget = std::max<size_t>(kSmPerKernel / pl.ctas_per_sm, pl.ring + 2 * pl.stage_bytes);
  int stages = static_cast<int>((budget - pl.ring) / pl.stage_bytes);
  stages = std::max(2, std::min(kMaxStages, stages));
  while (stages > 2 && pl.ring + static_cast<size_t>(stages) * pl.stage_bytes > smem_optin) --stages;
  pl.stages = stages;
  pl.smem = pl.ring + static_cast<size_t>(stages) * pl.stage_bytes;
  // The burst form: one CTA per SM holding all of its whole-row items at once, within
  // kSmPerKernel so the next kernel fits beside it.
  if (pl.rows_kernel && pl.nch == 1) {
    const int64_t per_cta = (pl.ngroups + sm_count - 1) / sm_count;
    if (per_cta <= kMaxStages && pl.ring + static_cast<size_t>(per_cta) * pl.stage_bytes <= kSmPerKernel)
      pl.burst_stages = static_cast<int>(per_cta);
  }
  return pl;
}

template <int KIND, class P>
const void *rows_kernel_ptr(int rw, int slots, bool burst) {
#define UGB_RK(RW, J)                                                                                 \
  if (rw == RW && slots == J)                                                                         \
    return burst ? reinterpret_cast<const void *>(&mv_rows_kernel<KIND, RW, J, P, true>)              \
                 : reinterpret_cast<const void *>(&mv_rows_kernel<KIND, RW, J, P, false>);
  UGB_RK(1, 2) UGB_RK(1, 3) UGB_RK(1, 4)
  UGB_RK(2, 2) UGB_RK(2, 3) UGB_RK(2, 4)
  UGB_RK(4, 2) UGB_RK(4, 3) UGB_RK(4, 4)
#undef UGB_RK
  return nullptr;
}

template <int KIND, class P>
const void *split_kernel_ptr(int r, int slots) {
#define UGB_SK(R, J) if (r == R && slots == J) return reinterpret_cast<const void *>(&mv_split_kernel<KIND, R, J, P>);
  UGB_SK(1, 2) UGB_SK(1, 4)
  UGB_SK(2, 2) UGB_SK(2, 4)
  UGB_SK(4, 2) UGB_SK(4, 4)
#undef UGB_SK
  return nullptr;
}

template <int KIND, class P>
const void *stream_kernel_ptr(int nb, bool dots, int rw) {
  if (dots) return rw == 1 ? reinterpret_cast<const void *>(&mv_stream_kernel<KIND, 1, true, P, 1>) : nullptr;
#define UGB_SK2(NB)                                                                             \
  case NB:                                                                                      \
    return rw == 2 ? reinterpret_cast<const void *>(&mv_stream_kernel<KIND, NB, false, P, 2>)   \
                   : reinterpret_cast<const void *>(&mv_stream_kernel<KIND, NB, false, P, 1>);
  switch (nb) {
    UGB_SK2(1) UGB_SK2(2) UGB_SK2(4) UGB_SK2(8)
    default: return nullptr;
  }
#undef UGB_SK2
}

template <int KIND, class P>
const void *select_stream(const Plan &pl, int nb, bool dots) {
  return pl.rows_kernel || pl.split ? nullptr : stream_kernel_ptr<KIND, P>(nb, dots, pl.rw);
}

template <int KIND, class P>
const void *select_for(const Plan &pl, int nb, bool dots) {
  return pl.rows_kernel ? rows_kernel_ptr<KIND, P>(pl.rw, pl.slots, pl.burst)
         : pl.split     ? split_kernel_ptr<KIND, P>(pl.rw, pl.slots)
                        : stream_kernel_ptr<KIND, P>(nb, dots, pl.rw);
}

// The kernel instance for a plan; `table` picks the instances that take the job table.
const void *select_kernel(uint32_t kind, const Plan &pl, int nb, bool dots, bool table = false) {
  if (table && dots) return nullptr;
  switch (kind) {
    case UGB_Q8_0: return table ? select_for<UGB_Q8_0, MvParamsT>(pl, nb, dots) : select_for<UGB_Q8_0, MvParams>(pl, nb, dots);
    case UGB_Q4_K: return table ? select_for<UGB_Q4_K, MvParamsT>(pl, nb, dots) : select_for<UGB_Q4_K, MvParams>(pl, nb, dots);
    case UGB_Q3_K: return table ? select_for<UGB_Q3_K, MvParamsT>(pl, nb, dots) : select_for<UGB_Q3_K, MvParams>(pl, nb, dots);
#define UGB_STREAM_ONLY(K) \
    case K: return table ? select_stream<K, MvParamsT>(pl, nb, dots) : select_stream<K, MvParams>(pl, nb, dots);
    UGB_STREAM_ONLY(UGB_Q6_K) UGB_STREAM_ONLY(UGB_IQ3_XXS) UGB_STREAM_ONLY(UGB_IQ4_NL) UGB_STREAM_ONLY(UGB_IQ4_XS)
#undef UGB_STREAM_ONLY
    default: return nullptr;
  }
}

ugb_status allow_smem(const void *f, size_t bytes) {
  return cuda_status(cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes)));
}

}  // namespace

ugb_status init_matvec_kernels(ugb_ctx *ctx) {
  for (uint32_t kind : {UGB_Q6_K, UGB_IQ3_XXS, UGB_IQ4_NL, UGB_IQ4_XS}) {
    Plan pl;
    for (int rw : {1, 2}) {
      pl.rw = rw;
      for (int nb : {1, 2, 4, 8})
        for (bool table : {false, true})
          if (allow_smem(select_kernel(kind, pl, nb, false, table), ctx->smem_optin) != UGB_OK) return UGB_EBACKEND;
    }
    pl.rw = 1;
    if (allow_smem(select_kernel(kind, pl, 1, true), ctx->smem_optin) != UGB_OK) return UGB_EBACKEND;
  }
  for (uint32_t kind : {UGB_Q8_0, UGB_Q4_K, UGB_Q3_K}) {
    Plan pl;
    for (int rw : {1, 2, 4})
      for (int j : {2, 3, 4}) {
        pl.rows_kernel = true;
        pl.rw = rw;
        pl.slots = j;
        for (bool table : {false, true}) {
          pl.rows_kernel = true;
          pl.split = false;
          pl.burst = true;
          if (allow_smem(select_kernel(kind, pl, 1, false, table), ctx->smem_optin) != UGB_OK) return UGB_EBACKEND;
          pl.burst = false;
          if (allow_smem(select_kernel(kind, pl, 1, false, table), ctx->smem_optin) != UGB_OK) return UGB_EBACKEND;
          if (j == 3) continue;  // the split kernel takes 2 or 4 slots
          pl.rows_kernel = false;
          pl.split = true;
          if (allow_smem(select_kernel(kind, pl, 1, false, table), ctx->smem_optin) != UGB_OK) return UGB_EBACKEND;
        }
        pl.split = false;
      }
    pl.rows_kernel = false;
    for (int rw : {1, 2}) {
      pl.rw = rw;
      for (int nb : {1, 2, 4, 8})
        for (bool table : {false, true})
          if (allow_smem(select_kernel(kind, pl, nb, false, table), ctx->smem_optin) != UGB_OK) return UGB_EBACKEND;
    }
    pl.rw = 1;
    if (allow_smem(select_kernel(kind, pl, 1, true), ctx->smem_optin) != UGB_OK) return UGB_EBACKEND;
  }
  return UGB_OK;
}

ugb_status launch_matvec(ugb_ctx *ctx, cudaStream_t stream, const MatvecArgs &a_in) {
  MatvecArgs a = a_in;
  const int mode = a.ids ? kRouted : a.njobs > 0 ? kTable : kSegments;
  if (mode == kTable) {
    if (a.njobs > kMaxJobs) return UGB_ESHAPE;
    a.nseg = a.njobs;
    a.m = 0;
    for (int i = 0; i < a.njobs; ++i) a.m = std::max(a.m, a.seg_rows[i]);
  } else if (mode == kRouted) {
    if (a.batch != 1 || a.per_slot < 1 || a.per_slot > 2 || a.n_slots < 1 || a.n_expert < 1 || a.x_div < 1)
      return UGB_ESHAPE;
    a.nseg = 1;
  } else if (a.nseg > kMaxSegs) {
    return UGB_ESHAPE;
  } else if (a.nseg == 0) {
    a.nseg = 1;
    a.ws[0] = a.w;
    a.seg_rows[0] = a.m;
  }
  const bool dots = a.dots != nullptr;
  if (dots && mode != kSegments) return UGB_ESHAPE;
  if (a.xf) {
    // Quantise inside the matvec when it runs as one batch-1 burst, else as a launch of its own.
    const Plan pl = make_plan(a.kind, a.k, a.m, 1, dots, ctx->smem_optin, ctx->sm_count);
    const bool fused = mode == kSegments && a.nseg <= 1 && a.batch == 1 && !dots && pl.burst_stages > 0;
    if (!fused) {
      const ugb_status st = launch_quant_q8_1(ctx, stream, a.xf, const_cast<uint8_t *>(a.xq), a.k, a.batch, a.pdl);
      if (st != UGB_OK) return st;
      MatvecArgs b = a;
      b.xf = nullptr;
      return launch_matvec(ctx, stream, b);
    }
  }
  // A batch runs as launches of 8, 4, 2 or 1 vectors (largest first) whose staged
  // activations fit kXBudget; each launch streams the weights once.
  int64_t done = 0;
  while (done < a.batch) {
    const int64_t rest = a.batch - done;
    if (mode == kSegments && !dots && rest >= 5) {  // Q4_K batches of 5..8 on the tensor cores
      bool used = false;
      const ugb_status st = launch_matvec_tc(ctx, stream, a, done, static_cast<int>(std::min<int64_t>(rest, 8)), &used);
      if (st != UGB_OK) return st;
      if (used) {
        done += std::min<int64_t>(rest, 8);
        continue;
      }
    }
    int nb = dots ? 1 : (rest >= 8 ? 8 : rest >= 4 ? 4 : rest >= 2 ? 2 : 1);
    while (nb > 1 && x_bytes(a.kind, a.k, nb) > kXBudget) nb /= 2;
    Plan pl = make_plan(a.kind, a.k, a.m, nb, dots, ctx->smem_optin, ctx->sm_count);
    if (mode == kSegments && pl.burst_stages > 0) {
      // every CTA's items staged at once: grid = min(groups, SMs), at most burst_stages each
      pl.burst = true;
      pl.stages = pl.burst_stages;
      pl.ctas_per_sm = 1;
      pl.smem = pl.ring + static_cast<size_t>(pl.stages) * pl.stage_bytes;
    }
    if (pl.smem > ctx->smem_optin) return UGB_ESHAPE;
    const void *f = select_kernel(a.kind, pl, nb, dots, mode == kTable);
    if (!f) return UGB_EQUANT;
    const int threads = pl.burst ? kWarps * 32 : kThreads;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, f, threads, pl.smem) != cudaSuccess ||
        per_sm < 1)
      return UGB_EBACKEND;
    per_sm = std::min(per_sm, pl.ctas_per_sm);
    // Items must not straddle two matrices: every matrix but the last must hold whole items,
    // otherwise the matrices go out as separate launches.
    bool whole = true;
    for (int i = 0; i + 1 < a.nseg; ++i) whole = whole && a.seg_rows[i] % pl.rows == 0;
    if (mode == kSegments && a.nseg > 1 && !whole) {
      int64_t row0 = 0;
      for (int i = 0; i < a.nseg; ++i) {
        MatvecArgs one = a;
        one.nseg = 1;
        one.w = a.ws[i];
        one.ws[0] = a.ws[i];
        one.m = one.seg_rows[0] = a.seg_rows[i];
        if (a.y) one.y = a.y + row0;
        if (a.dots) one.dots = a.dots + row0 * (a.k / 32);
        const ugb_status st = launch_matvec(ctx, stream, one);
        if (st != UGB_OK) return st;
        row0 += a.seg_rows[i];
      }
      return UGB_OK;
    }
    MvParamsT pt{};
    MvParams &p = pt;
    p.nseg = mode == kTable ? 1 : a.nseg;
    if (mode != kTable) {
      int64_t row0 = 0;
      for (int i = 0; i < a.nseg; ++i) {
        p.w[i] = a.ws[i];
        p.w_end16[i] = reinterpret_cast<const uint8_t *>(
            reinterpret_cast<uintptr_t>(a.ws[i] + a.seg_rows[i] * a.row_bytes) & ~uintptr_t(15));
        p.seg_row0[i] = static_cast<int>(row0);
        row0 += a.seg_rows[i];
      }
    }
    p.row_bytes = static_cast<uint64_t>(a.row_bytes);
    p.k = static_cast<int>(a.k);
    p.m = static_cast<int>(a.m);
    p.rows = pl.rows;
    p.kc = pl.kc;
    p.nch = pl.nch;
    p.ngroups = pl.ngroups;
    p.seg_stride = pl.seg_stride;
    p.stage_bytes = pl.stage_bytes;
    p.stages = pl.stages;
    p.x_q = pl.x_q;
    p.x_d = pl.x_d;
    p.x_s = pl.x_s;
    p.ring = pl.ring;
    p.red = pl.red;
    p.xq = a.xq + done * a.xl.k;
    p.xd = reinterpret_cast<const float *>(a.xq + a.xl.d_off) + done * a.xl.nbp;
    p.xs = reinterpret_cast<const int *>(a.xq + a.xl.s_off) + done * a.xl.nbp;
    p.xf = a.xf;  // only ever set for a batch-1 burst (checked above)
    p.nbp = static_cast<int>(a.xl.nbp);
    p.y = a.y ? a.y + done * a.ldy : nullptr;
    p.ldy = a.ldy;
    p.dots = a.dots;
    p.status = ctx->status;
    p.mode = mode;
    const int64_t budget = static_cast<int64_t>(ctx->sm_count) * per_sm;
    int grid = static_cast<int>(std::min<int64_t>(pl.ngroups, budget));
    if (mode == kTable) {
      // CTAs per job in proportion to its row groups (at least one, at most one per group).
      int64_t groups = 0;
      for (int i = 0; i < a.njobs; ++i) groups += (a.seg_rows[i] + pl.rows - 1) / pl.rows;
      MvTable &t = pt.t;
      t.njobs = a.njobs;
      int c = 0;
      for (int i = 0; i < a.njobs; ++i) {
        const int64_t g = (a.seg_rows[i] + pl.rows - 1) / pl.rows;
        t.jm[i] = static_cast<int>(a.seg_rows[i]);
        t.cta0[i] = c;
        c += static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(g, budget * g / std::max<int64_t>(1, groups))));
        t.jw[i] = a.ws[i];
        t.jw_end16[i] = reinterpret_cast<const uint8_t *>(
            reinterpret_cast<uintptr_t>(a.ws[i] + a.seg_rows[i] * a.row_bytes) & ~uintptr_t(15));
        t.jxq[i] = a.jx[i] + done * a.xl.k;
        t.jxd[i] = reinterpret_cast<const float *>(a.jx[i] + a.xl.d_off) + done * a.xl.nbp;
        t.jxs[i] = reinterpret_cast<const int *>(a.jx[i] + a.xl.s_off) + done * a.xl.nbp;
        t.jy[i] = a.jy[i] + done * a.seg_rows[i];
      }
      t.cta0[a.njobs] = c;
      grid = c;
    } else if (mode == kRouted) {
      const int jobs = a.n_slots * a.per_slot;
      p.ids = a.ids;
      p.per_slot = a.per_slot;
      p.n_expert = a.n_expert;
      p.expert0 = a.expert0;
      p.n_total = a.n_total;
      p.x_div = a.x_div;
      p.ebase[0] = a.ebase[0];
      p.ebase[1] = a.ebase[1];
      p.estride = a.estride;
      p.y_slot = a.y_slot;
      p.cpj = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(pl.ngroups, budget / jobs)));
      grid = p.cpj * jobs;
    }

    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(threads);  // 8 consumer warps (+ 1 producer warp unless a burst)
    cfg.dynamicSmemBytes = pl.smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = a.pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    void *args[] = {mode == kTable ? static_cast<void *>(&pt) : static_cast<void *>(&p)};
    if (cudaLaunchKernelExC(&cfg, f, args) != cudaSuccess) return UGB_EBACKEND;
    done += nb;
  }
  return UGB_OK;
}

}  // namespace ugb
