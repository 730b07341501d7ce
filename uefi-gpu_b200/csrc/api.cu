// api.cu -- the extern "C" boundary of libugb (include/ugb.h): validation, context, status.
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <new>
#include <vector>

#include "common.cuh"
#include "internal.hpp"
#include "decode.hpp"
#include "prefill.hpp"

namespace ugb {

ugb_status check_weights(uint32_t kind, const void *w, int64_t row_bytes, int64_t k, int64_t m) {
  if (!matvec_kind(kind)) return UGB_EQUANT;
  if (k <= 0 || k > UGB_MAX_K || m <= 0 || m > (int64_t{1} << 31) - 64) return UGB_ESHAPE;
  const int64_t rb = ugb_row_bytes(kind, k);
  if (rb < 0 || rb != row_bytes) return UGB_ESHAPE;
  if (!w || (reinterpret_cast<uintptr_t>(w) & 15) != 0) return UGB_EALIGN;
  return UGB_OK;
}

ugb_status check_ctx(ugb_ctx *ctx) {
  if (!ctx || !ctx->status) return UGB_ECONTEXT;
  if (cudaSetDevice(ctx->device) != cudaSuccess) return UGB_EBACKEND;
  return UGB_OK;
}

ugb_status read_status_bits(ugb_ctx *ctx, cudaStream_t stream, uint32_t *bits) {
  // The status word is cleared even when the read-back fails, so no bits leak into the next call.
  const bool copied = cudaMemcpyAsync(ctx->status_host, ctx->status, 4, cudaMemcpyDeviceToHost, stream) == cudaSuccess;
  const bool cleared = cudaMemsetAsync(ctx->status, 0, 4, stream) == cudaSuccess;
  if (cudaStreamSynchronize(stream) != cudaSuccess || !copied || !cleared) return UGB_EBACKEND;
  const uint32_t b = *ctx->status_host;
  if (bits) *bits = b;
  if (b & ST_TIMEOUT) {
    // A launch that gave up may have left tile tickets of the tensor-core matvec's K split
    // partly counted (mv_tc.cu); clear them so the next launches count from zero.
    if (ctx->mv_tickets &&
        (cudaMemsetAsync(ctx->mv_tickets, 0, ctx->mv_ntickets * 4, stream) != cudaSuccess ||
         cudaStreamSynchronize(stream) != cudaSuccess))
      return UGB_EBACKEND;
    return UGB_ETIMEOUT;
  }
  if (b & (ST_NONFINITE_IN | ST_NONFINITE_OUT)) return UGB_ENONFINITE;
  if (b & ST_BADARG) return UGB_ESHAPE;
  return UGB_OK;
}

namespace {

bool aligned16(const void *p) { return p && (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Grow the host-buffer workspace to at least `bytes` (device) and `pinned` (host).
ugb_status reserve(ugb_ctx *ctx, size_t bytes, size_t pinned) {
  if (bytes > ctx->work_bytes) {
    if (ctx->work) {
      cudaDeviceSynchronize();
      cudaFree(ctx->work);
      ctx->work = nullptr;
      ctx->work_bytes = 0;
    }
    const size_t want = round_up(bytes, 1 << 20);
    if (cudaMalloc(&ctx->work, want) != cudaSuccess) return UGB_EBACKEND;
    ctx->work_bytes = want;
  }
  if (pinned > ctx->pinned_bytes) {
    if (ctx->pinned) {
      cudaDeviceSynchronize();
      cudaFreeHost(ctx->pinned);
      ctx->pinned = nullptr;
      ctx->pinned_bytes = 0;
    }
    const size_t want = round_up(pinned, 1 << 16);
    if (cudaMallocHost(reinterpret_cast<void **>(&ctx->pinned), want) != cudaSuccess) return UGB_EBACKEND;
    ctx->pinned_bytes = want;
  }
  return UGB_OK;
}

}  // namespace
}  // namespace ugb

using namespace ugb;

extern "C" {

ugb_status ugb_init(int device, ugb_ctx **out) {
  if (!out) return UGB_ECONTEXT;
  *out = nullptr;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) return UGB_EBACKEND;
  if (cudaSetDevice(device) != cudaSuccess) return UGB_EBACKEND;
  ugb_ctx *ctx = new (std::nothrow) ugb_ctx();
  if (!ctx) return UGB_EBACKEND;
  ctx->device = device;
  int v = 0;
  cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device);
  ctx->sm_count = v;
  cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
  ctx->smem_optin = static_cast<size_t>(v);
  if (cudaMalloc(&ctx->status, 4) != cudaSuccess || cudaMemset(ctx->status, 0, 4) != cudaSuccess ||
      cudaMallocHost(reinterpret_cast<void **>(&ctx->status_host), 4) != cudaSuccess) {
    ugb_destroy(ctx);
    return UGB_EBACKEND;
  }
  ctx->mv_part_floats = size_t(1) << 20;  // 4 MB: 1024 tile chunks of 8 x 128 partials
  ctx->mv_ntickets = 4096;
  if (cudaMalloc(reinterpret_cast<void **>(&ctx->mv_part), ctx->mv_part_floats * 4) != cudaSuccess ||
      cudaMalloc(reinterpret_cast<void **>(&ctx->mv_tickets), ctx->mv_ntickets * 4) != cudaSuccess ||
      cudaMemset(ctx->mv_tickets, 0, ctx->mv_ntickets * 4) != cudaSuccess) {
    ugb_destroy(ctx);
    return UGB_EBACKEND;
  }
  ugb_status st = init_matvec_kernels(ctx);
  if (st == UGB_OK) st = init_matvec_tc_kernels(ctx);
  if (st == UGB_OK) st = init_decode_kernels(ctx);
  if (st == UGB_OK) st = init_prefill_kernels(ctx);
  if (st == UGB_OK) st = init_prefill_step_kernels(ctx);
  if (st != UGB_OK) {
    ugb_destroy(ctx);
    return st;
  }
  *out = ctx;
  return UGB_OK;
}

ugb_status ugb_destroy(ugb_ctx *ctx) {
  if (!ctx) return UGB_ECONTEXT;
  cudaSetDevice(ctx->device);
  cudaDeviceSynchronize();
  if (ctx->status) cudaFree(ctx->status);
  if (ctx->status_host) cudaFreeHost(ctx->status_host);
  if (ctx->work) cudaFree(ctx->work);
  if (ctx->mv_part) cudaFree(ctx->mv_part);
  if (ctx->mv_tickets) cudaFree(ctx->mv_tickets);
  if (ctx->pinned) cudaFreeHost(ctx->pinned);
  delete ctx;
  return UGB_OK;
}

const char *ugb_status_string(ugb_status s) {
  switch (s) {
    case UGB_OK: return "ok";
    case UGB_ESHAPE: return "shape";
    case UGB_ENONFINITE: return "non-finite";
    case UGB_ETIMEOUT: return "timeout";
    case UGB_EBACKEND: return "backend";
    case UGB_EALIGN: return "alignment";
    case UGB_EQUANT: return "quant kind";
    case UGB_ECONTEXT: return "context";
  }
  return "unknown";
}

ugb_status ugb_status_read(ugb_ctx *ctx, ugb_stream stream, uint32_t *bits) {
  ugb_status st = check_ctx(ctx);
  if (st != UGB_OK) return st;
  std::lock_guard<std::mutex> lock(ctx->mu);
  return read_status_bits(ctx, stream, bits);
}

int64_t ugb_row_bytes(uint32_t kind, int64_t n) {
  // frontier_core.rs:54-57, plus ggml's Q4_K / Q3_K.
  int64_t block, bytes;
  switch (kind) {
    case 0: block = 1; bytes = 4; break;      // F32
    case 8: block = 32; bytes = 34; break;    // Q8_0
    case 11: block = 256; bytes = 110; break; // Q3_K
    case 12: block = 256; bytes = 144; break; // Q4_K
    case 14: block = 256; bytes = 210; break; // Q6_K
    case 18: block = 256; bytes = 98; break;  // IQ3_XXS
    case 20: block = 32; bytes = 18; break;   // IQ4_NL
    case 23: block = 256; bytes = 136; break; // IQ4_XS
    case 30: block = 1; bytes = 2; break;     // BF16
    default: return -1;
  }
  if (n <= 0 || n % block != 0) return -2;
  return n / block * bytes;
}

size_t ugb_q8act_bytes(int64_t k, int64_t batch) {
  if (k <= 0 || k % 32 || batch <= 0) return 0;
  return q8act_layout(k, batch).bytes;
}
size_t ugb_q8act_scale_offset(int64_t k, int64_t batch) {
  if (k <= 0 || k % 32 || batch <= 0) return 0;
  return q8act_layout(k, batch).d_off;
}
size_t ugb_q8act_sum_offset(int64_t k, int64_t batch) {
  if (k <= 0 || k % 32 || batch <= 0) return 0;
  return q8act_layout(k, batch).s_off;
}

ugb_status ugb_quant_q8_1(ugb_ctx *ctx, ugb_stream stream, const float *x_dev, void *xq_dev,
                          int64_t k, int64_t batch) {
  ugb_status st = check_ctx(ctx);
  if (st != UGB_OK) return st;
  if (k <= 0 || k % 32 || k > UGB_MAX_K || batch <= 0 || batch > 65536) return UGB_ESHAPE;
  if (!x_dev || (reinterpret_cast<uintptr_t>(x_dev) & 3) || !aligned16(xq_dev)) return UGB_EALIGN;
  return launch_quant_q8_1(ctx, stream, x_dev, static_cast<uint8_t *>(xq_dev), k, batch, ctx->pdl);
}

ugb_status ugb_matvec(ugb_ctx *ctx, ugb_stream stream, uint32_t kind, const void *w_dev,
                      int64_t row_bytes, const void *xq_dev, float *y_dev, int64_t k, int64_t m,
                      int64_t batch) {
  ugb_status st = check_ctx(ctx);
  if (st != UGB_OK) return st;
  st = check_weights(kind, w_dev, row_bytes, k, m);
  if (st != UGB_OK) return st;
  if (batch <= 0 || batch > UGB_MAX_BATCH) return UGB_ESHAPE;
  if (!aligned16(xq_dev) || !y_dev || (reinterpret_cast<uintptr_t>(y_dev) & 3)) return UGB_EALIGN;
  MatvecArgs a;
  a.kind = kind;
  a.w = static_cast<const uint8_t *>(w_dev);
  a.row_bytes = row_bytes;
  a.k = k;
  a.m = m;
  a.xq = static_cast<const uint8_t *>(xq_dev);
  a.xl = q8act_layout(k, batch);
  a.y = y_dev;
  a.ldy = m;
  a.batch = batch;
  a.pdl = ctx->pdl;
  return launch_matvec(ctx, stream, a);
}

ugb_status ugb_matvec_f32(ugb_ctx *ctx, ugb_stream stream, uint32_t kind, const void *w_dev,
                          int64_t row_bytes, const float *x_dev, void *xq_scratch, float *y_dev,
                          int64_t k, int64_t m, int64_t batch) {
  ugb_status st = check_ctx(ctx);
  if (st != UGB_OK) return st;
  st = check_weights(kind, w_dev, row_bytes, k, m);
  if (st != UGB_OK) return st;
  if (batch <= 0 || batch > UGB_MAX_BATCH) return UGB_ESHAPE;
  if (!x_dev || (reinterpret_cast<uintptr_t>(x_dev) & 3) || !aligned16(xq_scratch) || !y_dev ||
      (reinterpret_cast<uintptr_t>(y_dev) & 3))
    return UGB_EALIGN;
  MatvecArgs a;
  a.kind = kind;
  a.w = static_cast<const uint8_t *>(w_dev);
  a.row_bytes = row_bytes;
  a.k = k;
  a.m = m;
  a.xf = x_dev;
  a.xq = static_cast<const uint8_t *>(xq_scratch);
  a.xl = q8act_layout(k, batch);
  a.y = y_dev;
  a.ldy = m;
  a.batch = batch;
  a.pdl = ctx->pdl;
  return launch_matvec(ctx, stream, a);
}

ugb_status ugb_matvec_multi(ugb_ctx *ctx, ugb_stream stream, uint32_t kind,
                            const void *const *w_devs, const int64_t *rows, int count,
                            int64_t row_bytes, const void *xq_dev, float *y_dev, int64_t k,
                            int64_t batch) {
  ugb_status st = check_ctx(ctx);
  if (st != UGB_OK) return st;
  if (!w_devs || !rows || count < 1 || count > 4) return UGB_ESHAPE;
  if (batch <= 0 || batch > UGB_MAX_BATCH) return UGB_ESHAPE;
  if (!aligned16(xq_dev) || !y_dev || (reinterpret_cast<uintptr_t>(y_dev) & 3)) return UGB_EALIGN;
  MatvecArgs a;
  int64_t total = 0;
  for (int i = 0; i < count; ++i) {
    st = check_weights(kind, w_devs[i], row_bytes, k, rows[i]);
    if (st != UGB_OK) return st;
    a.ws[i] = static_cast<const uint8_t *>(w_devs[i]);
    a.seg_rows[i] = rows[i];
    total += rows[i];
  }
  if (total > (int64_t{1} << 31) - 64) return UGB_ESHAPE;
  a.nseg = count;
  a.kind = kind;
  a.w = a.ws[0];
  a.row_bytes = row_bytes;
  a.k = k;
  a.m = total;
  a.xq = static_cast<const uint8_t *>(xq_dev);
  a.xl = q8act_layout(k, batch);
  a.y = y_dev;
  a.ldy = total;
  a.batch = batch;
  a.pdl = ctx->pdl;
  return launch_matvec(ctx, stream, a);
}

ugb_status ugb_block_dots(ugb_ctx *ctx, ugb_stream stream, uint32_t kind, const void *w_dev,
                          int64_t row_bytes, const void *xq_dev, int32_t *out_dev, int64_t k,
                          int64_t m) {
  ugb_status st = check_ctx(ctx);
  if (st != UGB_OK) return st;
  st = check_weights(kind, w_dev, row_bytes, k, m);
  if (st != UGB_OK) return st;
  if (!aligned16(xq_dev) || !out_dev || (reinterpret_cast<uintptr_t>(out_dev) & 3)) return UGB_EALIGN;
  MatvecArgs a;
  a.kind = kind;
  a.w = static_cast<const uint8_t *>(w_dev);
  a.row_bytes = row_bytes;
  a.k = k;
  a.m = m;
  a.xq = static_cast<const uint8_t *>(xq_dev);
  a.xl = q8act_layout(k, 1);
  a.batch = 1;
  a.dots = out_dev;
  return launch_matvec(ctx, stream, a);
}

ugb_status ugb_fill_synthetic(ugb_ctx *ctx, ugb_stream stream, uint32_t kind, void *w_dev,
                              int64_t k, int64_t m, uint64_t seed) {
  ugb_status st = check_ctx(ctx);
  if (st != UGB_OK) return st;
  st = check_weights(kind, w_dev, ugb_row_bytes(kind, k), k, m);
  if (st != UGB_OK) return st;
  return launch_fill_synthetic(ctx, stream, kind, static_cast<uint8_t *>(w_dev), k, m, seed);
}

ugb_status ugb_set_pdl(ugb_ctx *ctx, int enable) {
  if (!ctx) return UGB_ECONTEXT;
  ctx->pdl = enable != 0;
  return UGB_OK;
}

struct ugb_graph {
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
};

ugb_status ugb_graph_begin(ugb_ctx *ctx, ugb_stream stream) {
  ugb_status st = check_ctx(ctx);
  if (st != UGB_OK) return st;
  if (!stream) return UGB_ECONTEXT;  // the legacy default stream cannot be captured
  return cuda_status(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal));
}

ugb_status ugb_graph_end(ugb_ctx *ctx, ugb_stream stream, ugb_graph **out) {
  ugb_status st = check_ctx(ctx);
  if (st != UGB_OK) return st;
  if (!out) return UGB_ECONTEXT;
  *out = nullptr;
  ugb_graph *g = new (std::nothrow) ugb_graph();
  if (!g) return UGB_EBACKEND;
  if (cudaStreamEndCapture(stream, &g->graph) != cudaSuccess) {
    delete g;
    return UGB_EBACKEND;
  }
  if (cudaGraphInstantiate(&g->exec, g->graph, 0) != cudaSuccess) {
    cudaGraphDestroy(g->graph);
    delete g;
    return UGB_EBACKEND;
  }
  *out = g;
  return UGB_OK;
}

ugb_status ugb_graph_launch(ugb_graph *graph, ugb_stream stream) {
  if (!graph || !graph->exec) return UGB_ECONTEXT;
  return cuda_status(cudaGraphLaunch(graph->exec, stream));
}

ugb_status ugb_graph_kernels(const ugb_graph *g, int64_t *count) {
  if (!g || !g->graph || !count) return UGB_ECONTEXT;
  size_t n = 0;
  if (cudaGraphGetNodes(g->graph, nullptr, &n) != cudaSuccess) return UGB_EBACKEND;
  std::vector<cudaGraphNode_t> nodes(n);
  if (n && cudaGraphGetNodes(g->graph, nodes.data(), &n) != cudaSuccess) return UGB_EBACKEND;
  int64_t k = 0;
  for (size_t i = 0; i < n; ++i) {
    cudaGraphNodeType t;
    if (cudaGraphNodeGetType(nodes[i], &t) != cudaSuccess) return UGB_EBACKEND;
    k += t == cudaGraphNodeTypeKernel ? 1 : 0;
  }
  *count = k;
  return UGB_OK;
}

ugb_status ugb_graph_destroy(ugb_graph *graph) {
  if (!graph) return UGB_ECONTEXT;
  if (graph->exec) cudaGraphExecDestroy(graph->exec);
  if (graph->graph) cudaGraphDestroy(graph->graph);
  delete graph;
  return UGB_OK;
}

ugb_status ugb_linear(ugb_ctx *ctx, ugb_stream stream, uint32_t kind, const void *w_dev,
                      int64_t row_bytes, const float *x_host, float *y_host, int64_t k,
                      int64_t m) {
  ugb_status st = check_ctx(ctx);
  if (st != UGB_OK) return st;
  st = check_weights(kind, w_dev, row_bytes, k, m);
  if (st != UGB_OK) return st;
  if (!x_host || !y_host) return UGB_EALIGN;
  std::lock_guard<std::mutex> lock(ctx->mu);
  // x -> device, quant_act, matvec, y -> host (the reference's Gpu::matvec round trip).
  const Q8Act xl = q8act_layout(k, 1);
  const size_t x_off = 0, xq_off = round_up(k * 4, 256), y_off = xq_off + round_up(xl.bytes, 256);
  st = reserve(ctx, y_off + round_up(m * 4, 256), static_cast<size_t>(k + m) * 4);
  if (st != UGB_OK) return st;
  uint8_t *base = static_cast<uint8_t *>(ctx->work);
  float *x_dev = reinterpret_cast<float *>(base + x_off);
  uint8_t *xq = base + xq_off;
  float *y_dev = reinterpret_cast<float *>(base + y_off);
  std::memcpy(ctx->pinned, x_host, static_cast<size_t>(k) * 4);
  if (cudaMemcpyAsync(x_dev, ctx->pinned, k * 4, cudaMemcpyHostToDevice, stream) != cudaSuccess)
    return UGB_EBACKEND;
  MatvecArgs a;  // quant_act fused into the matvec where it runs as a burst (else xq first)
  a.kind = kind;
  a.w = static_cast<const uint8_t *>(w_dev);
  a.row_bytes = row_bytes;
  a.k = k;
  a.m = m;
  a.xf = x_dev;
  a.xq = xq;
  a.xl = xl;
  a.y = y_dev;
  a.ldy = m;
  a.batch = 1;
  st = launch_matvec(ctx, stream, a);
  if (st != UGB_OK) return st;
  float *y_pin = ctx->pinned + k;
  if (cudaMemcpyAsync(y_pin, y_dev, m * 4, cudaMemcpyDeviceToHost, stream) != cudaSuccess)
    return UGB_EBACKEND;
  st = read_status_bits(ctx, stream, nullptr);  // synchronises the stream
  if (st != UGB_OK) return st;
  std::memcpy(y_host, y_pin, static_cast<size_t>(m) * 4);
  return UGB_OK;
}

}  // extern "C"
