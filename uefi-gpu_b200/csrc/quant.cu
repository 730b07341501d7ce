// quant.cu -- block-32 activation quantiser (fp32 -> Q8_1: int8 quants, f32 scale, int32 sum).
//
// Replaces quant_act (gpu_dp4a.cu:23-31) and the arithmetic of prefill_quant
// (gpu_prefill.cu:111-123): one warp per 32-block, a = max|x| by xor-shuffle, d = a/127,
// q = clamp(rint(x * (127/a)), -127, 127) with IEEE division and round-half-even conversion,
// so every quant and scale is bit-identical to the reference CPU form (gpu_prefill.rs:105-106).
#include <cmath>

#include "common.cuh"
#include "internal.hpp"

namespace ugb {
namespace {

__global__ void __launch_bounds__(256) quant_q8_1_kernel(const float *__restrict__ x,
                                                          uint8_t *__restrict__ xq, int64_t k,
                                                          int64_t batch, int nbp, size_t d_off,
                                                          size_t s_off, uint32_t *status) {
  // Let the consumer launch (and prefetch its weights) now; it waits for this grid to finish
  // before it reads the quantised activation.
  grid_dep_launch();
  grid_dep_wait();
  const int lane = threadIdx.x & 31;
  const int64_t gw = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (gw >= batch * nbp) return;
  const int64_t v = gw / nbp;
  const int b = static_cast<int>(gw - v * nbp);
  float *d = reinterpret_cast<float *>(xq + d_off);
  int32_t *s = reinterpret_cast<int32_t *>(xq + s_off);
  if (b >= k / 32) {  // padding entries of the scale / sum rows
    if (lane == 0) {
      d[v * nbp + b] = 0.f;
      s[v * nbp + b] = 0;
    }
    return;
  }
  const float val = x[v * k + b * 32 + lane];
  const bool fin = isfinite(val);
  float a = fin ? fabsf(val) : 0.f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
  const float inv = a > 0.f ? 127.0f / a : 0.0f;
  int qi = fin ? __float2int_rn(val * inv) : 0;
  qi = max(-127, min(127, qi));
  reinterpret_cast<int8_t *>(xq)[v * k + b * 32 + lane] = static_cast<int8_t>(qi);
  const int sum = __reduce_add_sync(0xffffffffu, qi);
  const bool bad = __any_sync(0xffffffffu, !fin);
  if (lane == 0) {
    d[v * nbp + b] = a / 127.0f;
    s[v * nbp + b] = sum;
    if (bad) status_or(status, ST_NONFINITE_IN);
  }
}

}  // namespace

Q8Act q8act_layout(int64_t k, int64_t batch) {
  Q8Act l;
  l.k = k;
  l.batch = batch;
  l.nbp = static_cast<int64_t>(round_up(static_cast<uint64_t>(k / 32), 4));
  l.d_off = round_up(static_cast<uint64_t>(batch * k), 256);
  const size_t vec = round_up(static_cast<uint64_t>(batch * l.nbp * 4), 256);
  l.s_off = l.d_off + vec;
  l.bytes = l.s_off + vec;
  return l;
}

ugb_status launch_quant_q8_1(ugb_ctx *ctx, cudaStream_t stream, const float *x, uint8_t *xq,
                             int64_t k, int64_t batch, bool pdl) {
  const Q8Act l = q8act_layout(k, batch);
  const int64_t warps = batch * l.nbp;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>((warps + 7) / 8));
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int nbp = static_cast<int>(l.nbp);
  size_t d_off = l.d_off, s_off = l.s_off;
  uint32_t *status = ctx->status;
  void *args[] = {&x, &xq, &k, &batch, &nbp, &d_off, &s_off, &status};
  return cuda_status(cudaLaunchKernelExC(&cfg, reinterpret_cast<const void *>(&quant_q8_1_kernel), args));
}

}  // namespace ugb
