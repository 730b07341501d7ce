// moe.cu -- the MoE expert path: the job-table matvec (the reference's FrontierJob launch),
// top-k routing, the device-routed expert SwiGLU and the weighted combine.
//
// Reference: frontier_multi_matvec + FrontierJob (kernels/frontier_quant.cu:68-93), its host
// packer (frontier_dispatch.rs:11-31), and Forward::ffn (frontier_forward.rs:164-199): router
// matvec, softmax (:47-51), top-k by descending probability with ties to the lower id (:167),
// weights renormalised by the top-k sum (:168, :193), gate/up per selected expert in one
// batched launch, SiLU(gate) * up, down per expert in a second launch, and the combine
// out += w * value in rank order with a separate fp32 multiply and add (frontier_cpu_axpy.rs).
//
// B200 form: the expert weights stay stacked as in the GGUF file ([expert][rows][row_bytes]);
// routing writes expert ids to device memory and the routed matvec resolves each (token, rank)
// slot's matrix on the device, so a whole MoE layer is a fixed launch sequence that a CUDA
// graph can replay.  Under expert parallelism each device holds a contiguous range of
// experts; slots routed elsewhere are skipped (their weights are never read) and the combine
// sums only the held experts' terms, leaving the cross-device sum to one all-reduce.
#include <cmath>

#include "common.cuh"
#include "decode.hpp"
#include "internal.hpp"

namespace ugb {
namespace {

constexpr int kRouteMax = 4096;  // experts a router may score

// One warp per token: softmax over the n experts' logits, then top_k rounds of argmax
// (highest probability, lowest id on ties), weights = p / (sum of the chosen p in rank order).
// A non-finite logit or a zero sum gives ids -1 / weights 0 and the non-finite status bit.
__global__ void __launch_bounds__(32) moe_route_kernel(const float *__restrict__ logits, int n, int top_k,
                                                       int32_t *__restrict__ ids, float *__restrict__ weights,
                                                       uint32_t *status) {
  grid_dep_launch();
  grid_dep_wait();
  __shared__ float prob[kRouteMax];
  const int lane = threadIdx.x;
  const float *l = logits + static_cast<int64_t>(blockIdx.x) * n;
  float mx = -INFINITY;
  bool fin = true;
  for (int e = lane; e < n; e += 32) {
    const float v = l[e];
    fin = fin && isfinite(v);
    mx = fmaxf(mx, v);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  fin = __all_sync(0xffffffffu, fin);
  for (int e = lane; e < n; e += 32) prob[e] = expf(l[e] - mx);
  __syncwarp();
  // the reference sums in index order (frontier_forward.rs:49): one lane, sequentially
  float sum = 0.f;
  if (lane == 0)
    for (int e = 0; e < n; ++e) sum += prob[e];
  sum = __shfl_sync(0xffffffffu, sum, 0);
  int32_t *out_ids = ids + static_cast<int64_t>(blockIdx.x) * top_k;
  float *out_w = weights + static_cast<int64_t>(blockIdx.x) * top_k;
  if (!fin || !(sum > 0.f) || !isfinite(sum)) {
    for (int r = lane; r < top_k; r += 32) {
      out_ids[r] = -1;
      out_w[r] = 0.f;
    }
    if (lane == 0) status_or(status, ST_NONFINITE_IN);
    return;
  }
  for (int e = lane; e < n; e += 32) prob[e] = prob[e] / sum;
  __syncwarp();
  float top = 0.f, chosen_p = 0.f;  // lane r keeps rank r's probability (top_k <= 32)
  for (int r = 0; r < top_k; ++r) {
    float bp = -1.f;
    int bid = 0x7fffffff;
    for (int e = lane; e < n; e += 32) {
      const float v = prob[e];
      if (v > bp) {  // e ascends within a lane: strict > keeps the lowest id among equals
        bp = v;
        bid = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float op = __shfl_xor_sync(0xffffffffu, bp, o);
      const int oid = __shfl_xor_sync(0xffffffffu, bid, o);
      if (op > bp || (op == bp && oid < bid)) {
        bp = op;
        bid = oid;
      }
    }
    if (lane == 0) {
      top += bp;  // rank order, as the reference's sum over ids[..k]
      out_ids[r] = bid;
      prob[bid] = -1.f;  // taken
    }
    if (lane == r) chosen_p = bp;
    __syncwarp();
  }
  top = __shfl_sync(0xffffffffu, top, 0);
  if (lane < top_k) out_w[lane] = chosen_p / top;  // frontier_forward.rs:193 scores[id] / sum
}

// h = silu(g) * u of every slot's gate/up outputs (gu[s] = [gate F ; up F]), block-32
// quantised into vector s of a Q8_1 buffer; slots of experts this device does not hold get
// zero quants and scales.  One warp per (32-block, slot).
__global__ void __launch_bounds__(256) moe_silu_quant_kernel(const float *__restrict__ gu, int ff,
                                                             const int32_t *__restrict__ ids, int expert0,
                                                             int n_local, uint8_t *__restrict__ hq, size_t d_off,
                                                             size_t s_off, int nbp, uint32_t *status) {
  grid_dep_launch();
  grid_dep_wait();
  const int lane = threadIdx.x & 31;
  const int b = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int s = blockIdx.y;
  if (b >= nbp) return;
  int8_t *q = reinterpret_cast<int8_t *>(hq) + static_cast<int64_t>(s) * ff;
  float *d = reinterpret_cast<float *>(hq + d_off) + static_cast<int64_t>(s) * nbp;
  int32_t *sm = reinterpret_cast<int32_t *>(hq + s_off) + static_cast<int64_t>(s) * nbp;
  const int el = ids[s] - expert0;
  const bool held = el >= 0 && el < n_local;
  if (b >= ff / 32 || !held) {
    if (b < ff / 32) q[b * 32 + lane] = 0;
    if (lane == 0) {
      d[b] = 0.f;
      sm[b] = 0;
    }
    return;
  }
  const float *g = gu + static_cast<int64_t>(s) * 2 * ff;
  const float gv = g[b * 32 + lane], uv = g[ff + b * 32 + lane];
  const float h = (gv / (1.0f + expf(-gv))) * uv;
  const bool fin = isfinite(h);
  float a = fin ? fabsf(h) : 0.f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
  const float inv = a > 0.f ? 127.0f / a : 0.0f;
  int qi = fin ? __float2int_rn(h * inv) : 0;
  qi = max(-127, min(127, qi));
  q[b * 32 + lane] = static_cast<int8_t>(qi);
  const int total = __reduce_add_sync(0xffffffffu, qi);
  const bool bad = __any_sync(0xffffffffu, !fin);
  if (lane == 0) {
    d[b] = a / 127.0f;
    sm[b] = total;
    if (bad) status_or(status, ST_NONFINITE_IN);
  }
}

// out[t][i] (=|+=) sum over ranks r of w[t][r] * v[t][r][i], in rank order with a separate
// multiply and add (frontier_cpu_axpy.rs); ranks whose expert this device does not hold (or
// whose id is -1) are left out.
__global__ void __launch_bounds__(256) moe_combine_kernel(const float *__restrict__ values,
                                                          const float *__restrict__ w,
                                                          const int32_t *__restrict__ ids, int top_k, int d,
                                                          int expert0, int n_local, int accumulate,
                                                          float *__restrict__ out, uint32_t *status) {
  grid_dep_launch();
  grid_dep_wait();
  const int t = blockIdx.y;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= d) return;
  float acc = accumulate ? out[static_cast<int64_t>(t) * d + i] : 0.f;
  for (int r = 0; r < top_k; ++r) {
    const int el = ids[t * top_k + r] - expert0;
    if (el < 0 || el >= n_local) continue;
    acc = __fadd_rn(acc, __fmul_rn(w[t * top_k + r], values[(static_cast<int64_t>(t) * top_k + r) * d + i]));
  }
  out[static_cast<int64_t>(t) * d + i] = acc;
  if (!isfinite(acc)) status_or(status, ST_NONFINITE_OUT);
}

}  // namespace
}  // namespace ugb

// ---- host ------------------------------------------------------------------------------------

using namespace ugb;

namespace {

template <typename... KArgs, typename... Args>
ugb_status launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, cudaStream_t s, bool pdl, Args... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...));
}

bool aligned16(uint64_t p) { return (p & 15) == 0; }

struct MoeLayout {
  int64_t slots = 0;
  size_t gu = 0, hq = 0, values = 0, bytes = 0;  // offsets in the workspace
  Q8Act hl;
};

MoeLayout moe_layout(int64_t hidden, int64_t ffn, int64_t top_k, int64_t batch) {
  MoeLayout l;
  l.slots = top_k * batch;
  l.hl = q8act_layout(ffn, l.slots);
  l.gu = 0;
  l.hq = round_up(static_cast<uint64_t>(l.slots * 2 * ffn) * 4, 256);
  l.values = l.hq + round_up(l.hl.bytes, 256);
  l.bytes = l.values + round_up(static_cast<uint64_t>(l.slots * hidden) * 4, 256);
  return l;
}

}  // namespace

namespace ugb {

ugb_status launch_moe_route(ugb_ctx *ctx, cudaStream_t stream, bool pdl, const float *logits, int n_expert,
                            int top_k, int batch, int32_t *ids, float *weights) {
  return launch_pdl(moe_route_kernel, dim3(static_cast<unsigned>(batch)), dim3(32), stream, pdl, logits, n_expert,
                    top_k, ids, weights, ctx->status);
}

// gate/up of every held slot (two routed matrices per slot sharing the token's activation) ->
// SiLU*up quant -> down (one routed matrix per slot on its own activation) -> combine.
ugb_status launch_moe_experts(ugb_ctx *ctx, cudaStream_t stream, const ugb_moe_args &m) {
  const int64_t rb_in = ugb_row_bytes(m.kind, m.hidden), rb_ff = ugb_row_bytes(m.kind, m.ffn);
  const MoeLayout l = moe_layout(m.hidden, m.ffn, m.top_k, m.batch);
  uint8_t *ws = static_cast<uint8_t *>(m.workspace);
  float *gu = reinterpret_cast<float *>(ws + l.gu);
  uint8_t *hq = ws + l.hq;
  float *values = reinterpret_cast<float *>(ws + l.values);
  const int slots = static_cast<int>(l.slots);
  MatvecArgs a;
  a.kind = m.kind;
  a.k = m.hidden;
  a.m = m.ffn;
  a.row_bytes = rb_in;
  a.xq = static_cast<const uint8_t *>(m.xq);
  a.xl = q8act_layout(m.hidden, m.batch);
  a.y = gu;
  a.pdl = true;
  a.ids = m.ids;
  a.n_slots = slots;
  a.per_slot = 2;
  a.n_expert = static_cast<int>(m.n_expert);
  a.expert0 = static_cast<int>(m.expert0);
  a.n_total = static_cast<int>(m.n_expert_total);
  a.x_div = static_cast<int>(m.top_k);
  a.ebase[0] = static_cast<const uint8_t *>(m.gate);
  a.ebase[1] = static_cast<const uint8_t *>(m.up);
  a.estride = static_cast<uint64_t>(rb_in) * m.ffn;
  a.y_slot = 2 * m.ffn;
  ugb_status st = launch_matvec(ctx, stream, a);
  if (st != UGB_OK) return st;
  st = launch_pdl(moe_silu_quant_kernel, dim3(static_cast<unsigned>((l.hl.nbp + 7) / 8), static_cast<unsigned>(slots)),
                  dim3(256), stream, true, gu, static_cast<int>(m.ffn), m.ids, static_cast<int>(m.expert0),
                  static_cast<int>(m.n_expert), hq, l.hl.d_off, l.hl.s_off, static_cast<int>(l.hl.nbp), ctx->status);
  if (st != UGB_OK) return st;
  MatvecArgs b = a;
  b.k = m.ffn;
  b.m = m.hidden;
  b.row_bytes = rb_ff;
  b.xq = hq;
  b.xl = l.hl;
  b.y = values;
  b.per_slot = 1;
  b.x_div = 1;
  b.ebase[0] = static_cast<const uint8_t *>(m.down);
  b.ebase[1] = nullptr;
  b.estride = static_cast<uint64_t>(rb_ff) * m.hidden;
  b.y_slot = m.hidden;
  st = launch_matvec(ctx, stream, b);
  if (st != UGB_OK) return st;
  return launch_pdl(moe_combine_kernel, dim3(static_cast<unsigned>((m.hidden + 255) / 256), static_cast<unsigned>(m.batch)),
                    dim3(256), stream, true, static_cast<const float *>(values), m.weights, m.ids,
                    static_cast<int>(m.top_k), static_cast<int>(m.hidden), static_cast<int>(m.expert0),
                    static_cast<int>(m.n_expert), m.accumulate, m.out, ctx->status);
}

}  // namespace ugb

extern "C" {

ugb_status ugb_matvec_jobs(ugb_ctx *ctx, ugb_stream stream, const ugb_job *jobs, int count, int64_t batch) {
  if (!ctx || !ctx->status) return UGB_ECONTEXT;
  if (!jobs || count < 1 || count > UGB_MAX_JOBS || batch < 1 || batch > UGB_MAX_BATCH) return UGB_ESHAPE;
  // frontier_dispatch.rs:14-27: every job well-formed, no two outputs overlapping
  for (int i = 0; i < count; ++i) {
    const ugb_job &j = jobs[i];
    if (j.n == 0 || j.m == 0 || j.n > UGB_MAX_K) return UGB_ESHAPE;
    const int64_t rb = ugb_row_bytes(j.kind, j.n);
    if (rb == -1) return UGB_EQUANT;
    if (rb < 0 || static_cast<uint64_t>(rb) != j.row_bytes) return UGB_ESHAPE;
    if (!j.weights || !j.input || !j.output) return UGB_EALIGN;
    if (!aligned16(j.weights) || !aligned16(j.input)) return UGB_EALIGN;
    const ugb_status st = check_weights(j.kind, reinterpret_cast<const void *>(j.weights), rb, j.n, j.m);
    if (st != UGB_OK) return st;
    const uint64_t end = j.output + static_cast<uint64_t>(batch) * j.m * 4;
    for (int p = 0; p < i; ++p) {
      const uint64_t pend = jobs[p].output + static_cast<uint64_t>(batch) * jobs[p].m * 4;
      if (j.output < pend && jobs[p].output < end) return UGB_ESHAPE;
    }
  }
  std::lock_guard<std::mutex> lock(ctx->mu);
  // One launch per (kind, n) group, jobs in table order within it.
  bool done[UGB_MAX_JOBS] = {};
  for (int i = 0; i < count; ++i) {
    if (done[i]) continue;
    MatvecArgs a;
    a.kind = jobs[i].kind;
    a.k = jobs[i].n;
    a.row_bytes = jobs[i].row_bytes;
    a.xl = q8act_layout(a.k, batch);
    a.batch = batch;
    a.pdl = ctx->pdl;
    for (int j = i; j < count; ++j) {
      if (done[j] || jobs[j].kind != a.kind || jobs[j].n != static_cast<uint32_t>(a.k)) continue;
      done[j] = true;
      const int q = a.njobs++;
      a.ws[q] = reinterpret_cast<const uint8_t *>(jobs[j].weights);
      a.seg_rows[q] = jobs[j].m;
      a.jx[q] = reinterpret_cast<const uint8_t *>(jobs[j].input);
      a.jy[q] = reinterpret_cast<float *>(jobs[j].output);
    }
    const ugb_status st = launch_matvec(ctx, stream, a);
    if (st != UGB_OK) return st;
  }
  return UGB_OK;
}

ugb_status ugb_moe_route(ugb_ctx *ctx, ugb_stream stream, const float *logits_dev, int64_t n_expert,
                         int64_t top_k, int64_t batch, int32_t *ids_dev, float *weights_dev) {
  if (!ctx || !ctx->status) return UGB_ECONTEXT;
  if (n_expert < 1 || n_expert > kRouteMax || top_k < 1 || top_k > 32 || top_k > n_expert || batch < 1 ||
      batch > 65535)
    return UGB_ESHAPE;
  if (!logits_dev || !ids_dev || !weights_dev) return UGB_EALIGN;
  return launch_moe_route(ctx, stream, ctx->pdl, logits_dev, static_cast<int>(n_expert), static_cast<int>(top_k),
                          static_cast<int>(batch), ids_dev, weights_dev);
}

size_t ugb_moe_workspace_bytes(int64_t hidden, int64_t ffn, int64_t top_k, int64_t batch) {
  if (hidden < 32 || ffn < 32 || top_k < 1 || batch < 1) return 0;
  return moe_layout(hidden, ffn, top_k, batch).bytes;
}

ugb_status ugb_moe_combine(ugb_ctx *ctx, ugb_stream stream, const float *values_dev, const float *weights_dev,
                           const int32_t *ids_dev, int64_t top_k, int64_t d, int64_t batch, int64_t expert0,
                           int64_t n_local, int accumulate, float *out_dev) {
  if (!ctx || !ctx->status) return UGB_ECONTEXT;
  if (top_k < 1 || top_k > 32 || d < 1 || batch < 1 || batch > 65535 || n_local < 0 || expert0 < 0)
    return UGB_ESHAPE;
  if (!values_dev || !weights_dev || !ids_dev || !out_dev) return UGB_EALIGN;
  return launch_pdl(moe_combine_kernel, dim3(static_cast<unsigned>((d + 255) / 256), static_cast<unsigned>(batch)),
                    dim3(256), stream, ctx->pdl, values_dev, weights_dev, ids_dev, static_cast<int>(top_k),
                    static_cast<int>(d), static_cast<int>(expert0), static_cast<int>(n_local), accumulate, out_dev,
                    ctx->status);
}

ugb_status ugb_moe_experts(ugb_ctx *ctx, ugb_stream stream, const ugb_moe_args *m) {
  if (!ctx || !ctx->status) return UGB_ECONTEXT;
  if (!m) return UGB_ESHAPE;
  if (m->hidden < 32 || m->ffn < 32 || m->hidden > UGB_MAX_K || m->ffn > UGB_MAX_K || m->top_k < 1 ||
      m->top_k > 32 || m->batch < 1 || m->batch > 256 || m->n_expert < 1 || m->expert0 < 0 ||
      m->n_expert_total < m->expert0 + m->n_expert)
    return UGB_ESHAPE;
  const int64_t rb_in = ugb_row_bytes(m->kind, m->hidden), rb_ff = ugb_row_bytes(m->kind, m->ffn);
  if (!matvec_kind(m->kind)) return UGB_EQUANT;
  if (rb_in < 0 || rb_ff < 0) return UGB_ESHAPE;
  if (!m->gate || !m->up || !m->down || !m->xq || !m->ids || !m->weights || !m->out || !m->workspace)
    return UGB_EALIGN;
  if (m->workspace_bytes < moe_layout(m->hidden, m->ffn, m->top_k, m->batch).bytes ||
      (reinterpret_cast<uintptr_t>(m->workspace) & 255))
    return UGB_ESHAPE;
  for (const void *w : {m->gate, m->up, m->down})
    if ((reinterpret_cast<uintptr_t>(w) & 15) != 0) return UGB_EALIGN;
  std::lock_guard<std::mutex> lock(ctx->mu);
  return launch_moe_experts(ctx, stream, *m);
}

}  // extern "C"
