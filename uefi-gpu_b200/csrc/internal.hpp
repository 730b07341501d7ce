// internal.hpp -- host-side declarations shared by the .cu files of libugb.
#pragma once
#include <cstddef>
#include <cstdint>
#include <mutex>
#include <cuda_runtime.h>

#include "../../include/ugb.h"

struct ugb_ctx {
  int device = 0;
  int sm_count = 0;
  size_t smem_optin = 0;        // max dynamic shared memory per block
  uint32_t *status = nullptr;   // device status word
  uint32_t *status_host = nullptr;  // pinned mirror for ugb_status_read
  // Workspace of the host-buffer entry points (x staging, xq, y staging).
  void *work = nullptr;
  size_t work_bytes = 0;
  float *pinned = nullptr;      // pinned host staging for ugb_linear
  size_t pinned_bytes = 0;
  bool pdl = false;             // programmatic dependent launch for every kernel
  // K-split workspace of the tensor-core batched matvec (mv_tc.cu): chunk partials and one
  // ticket per 128-row tile (zero between launches).  Launches that use it are ordered on one
  // stream, as every launch of a decode step is.
  float *mv_part = nullptr;
  size_t mv_part_floats = 0;
  uint32_t *mv_tickets = nullptr;
  size_t mv_ntickets = 0;
  std::mutex mu;
};

namespace ugb {

inline ugb_status cuda_status(cudaError_t e) { return e == cudaSuccess ? UGB_OK : UGB_EBACKEND; }

// Q8_1 activation layout (see ugb.h ugb_q8act_bytes).
struct Q8Act {
  int64_t k = 0, batch = 0, nbp = 0;
  size_t d_off = 0, s_off = 0, bytes = 0;
};
Q8Act q8act_layout(int64_t k, int64_t batch);

constexpr int kMaxMatvecSegs = 4;   // matrices sharing one activation in one matvec launch
constexpr int kMaxMatvecJobs = 32;  // independent jobs of one job-table launch

// Streaming matvec launch description.
struct MatvecArgs {
  uint32_t kind = 0;
  const uint8_t *w = nullptr;    // single matrix (nseg == 0), or:
  const uint8_t *ws[kMaxMatvecJobs] = {};  // matrices of seg_rows[i] rows, y rows concatenated
  int64_t seg_rows[kMaxMatvecJobs] = {};    // (up to kMaxMatvecSegs segments, or the jobs)
  int nseg = 0;
  int64_t row_bytes = 0, k = 0, m = 0;
  const uint8_t *xq = nullptr;   // Q8_1 buffer
  Q8Act xl;                      // its layout
  // fp32 activation ([batch][k]) to quantise first, or null.  A batch-1 burst launch quantises
  // it itself (every CTA, into shared memory); otherwise it is quantised into xq (then a
  // scratch buffer of layout xl) by a launch of its own.
  const float *xf = nullptr;
  float *y = nullptr;            // [batch][ldy]
  int64_t ldy = 0;
  int64_t batch = 1;
  int32_t *dots = nullptr;       // debug: block dots instead of y
  bool pdl = false;              // launch with programmatic stream serialisation
  // Job table (njobs > 0): job i = matrix ws[i] of seg_rows[i] rows with its own Q8_1
  // activation jx[i] (layout xl, `batch` vectors) and output jy[i] ([batch][seg_rows[i]]).
  int njobs = 0;
  const uint8_t *jx[kMaxMatvecJobs] = {};
  float *jy[kMaxMatvecJobs] = {};
  // Routed experts (ids set; batch 1): slot s < n_slots, matrix i < per_slot uses expert
  // ids[s] of the stacked tensor ebase[i] (n_expert experts of m rows, estride bytes apart,
  // global ids from expert0; other ids < n_total are another device's and are skipped),
  // activation vector s / x_div of xq (layout xl) and writes y + s * y_slot + i * m.
  const int32_t *ids = nullptr;
  int n_slots = 0, per_slot = 1, n_expert = 0, x_div = 1;
  int expert0 = 0, n_total = 0;  // held experts are global ids [expert0, expert0 + n_expert)
  const uint8_t *ebase[2] = {};
  uint64_t estride = 0;
  int64_t y_slot = 0;
};

ugb_status launch_matvec(ugb_ctx *ctx, cudaStream_t stream, const MatvecArgs &a);
ugb_status launch_quant_q8_1(ugb_ctx *ctx, cudaStream_t stream, const float *x, uint8_t *xq,
                             int64_t k, int64_t batch, bool pdl);
ugb_status launch_fill_synthetic(ugb_ctx *ctx, cudaStream_t stream, uint32_t kind, uint8_t *w,
                                 int64_t k, int64_t m, uint64_t seed);
ugb_status init_matvec_kernels(ugb_ctx *ctx);
// Tensor-core form of a Q4_K batch launch (vectors [done, done + nb)); *used is false when the
// launch does not qualify and the dp4a kernels must serve it.
ugb_status launch_matvec_tc(ugb_ctx *ctx, cudaStream_t stream, const MatvecArgs &a, int64_t done, int nb,
                            bool *used);
ugb_status init_matvec_tc_kernels(ugb_ctx *ctx);

// Collectives of a sharded decode step (comm.cu).
ugb_status comm_allreduce_sum_f32(ugb_comm *c, float *buf, size_t n, cudaStream_t stream);
ugb_status comm_allreduce_max_u64(ugb_comm *c, unsigned long long *buf, size_t n, cudaStream_t stream);
int comm_world(const ugb_comm *c);

// Entry-point prologue: a live context, and its device made current for this thread.
ugb_status check_ctx(ugb_ctx *ctx);
// Synchronise `stream`, return the context's device status bits (and clear them) as a status
// code: TIMEOUT, then NONFINITE, then BADARG (as UGB_ESHAPE).
ugb_status read_status_bits(ugb_ctx *ctx, cudaStream_t stream, uint32_t *bits);

// Kinds the matvec kernels read: Q8_0, Q3_K, Q4_K, Q6_K, IQ3_XXS, IQ4_NL, IQ4_XS.
inline bool matvec_kind(uint32_t kind) {
  return kind == UGB_Q8_0 || kind == UGB_Q3_K || kind == UGB_Q4_K || kind == UGB_Q6_K || kind == UGB_IQ3_XXS ||
         kind == UGB_IQ4_NL || kind == UGB_IQ4_XS;
}

// Validation shared by entry points: kind supported by the matvec kernels, k a multiple of
// its block, row_bytes consistent.
ugb_status check_weights(uint32_t kind, const void *w, int64_t row_bytes, int64_t k, int64_t m);

}  // namespace ugb
