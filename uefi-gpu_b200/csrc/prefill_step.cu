// prefill_step.cu -- the glue of a whole-prompt prefill around the tcgen05 INT8 GEMMs: the
// token embedding, per-token RMSNorm, bias + RoPE with the KV-cache write, causal attention over
// the prompt, and SiLU * up.  The decoder (decoder.cu, ugb_decoder_prefill) runs them with the
// GEMMs of prefill.cu as the reference's prefill graph does (gpu_prefill.rs:122-150; kernels
// prefill_embedding / prefill_resnorm / prefill_rope / prefill_attention / silu_mul,
// gpu_prefill.cu:60-101), for n tokens at positions pos0 .. pos0 + n - 1 of sequence 0.
//
// Arithmetic kept from the decode step (and so from the reference): the same RMSNorm formula,
// RoPE over the pairs (i, i + 64) from the decoder's table, scores q.k / sqrt(128) with an exact
// expf softmax, SiLU(g) * u.  Attention is computed in fp32 on the CUDA cores, with an online
// (running max) softmax over 64-position chunks of the cache.
#include <cfloat>
#include <cmath>

#include "common.cuh"
#include "decode.hpp"
#include "glue.cuh"
#include "prefill.hpp"

namespace ugb {
namespace {

constexpr int kHD = kHeadDim;

// x[t] = the Q8_0 embedding row of tokens[t] (embedding_q8 / prefill_embedding,
// gpu_prefill.cu:60-64).  One CTA per token.
__global__ void __launch_bounds__(256) pf_embed_kernel(const uint8_t *__restrict__ tok_embd,
                                                       const int32_t *__restrict__ tokens, int embd, int vocab,
                                                       float *__restrict__ x, uint32_t *status) {
  const int t = blockIdx.x;
  int tok = tokens[t];
  if (tok < 0 || tok >= vocab) {
    if (threadIdx.x == 0) status_or(status, ST_BADARG);
    tok = 0;
  }
  const uint8_t *row = tok_embd + static_cast<uint64_t>(tok) * (embd / 32) * 34;
  float *xt = x + static_cast<int64_t>(t) * embd;
  for (int i = threadIdx.x; i < embd; i += blockDim.x) {
    const uint8_t *blk = row + (i / 32) * 34;
    const uint32_t h = blk[0] | (static_cast<uint32_t>(blk[1]) << 8);
    xt[i] = half_bits_to_float(h) * static_cast<float>(static_cast<int8_t>(blk[2 + (i & 31)]));
  }
}

// Token t = blockIdx.x: x[t] += dx[t] (when dx is given); y[t] = x[t] * (1/sqrt(mean(x^2) +
// eps)) * w (prefill_resnorm, gpu_prefill.cu:65-72).  The sum of squares is the decode kernel's
// fixed-order tree.
__global__ void __launch_bounds__(512) pf_rmsnorm_kernel(float *__restrict__ x, const float *__restrict__ dx,
                                                         const float *__restrict__ w, int n, float eps,
                                                         float *__restrict__ y, uint32_t *status) {
  __shared__ float part[32];
  const int t = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float *xt = x + static_cast<int64_t>(t) * n;
  const float *dxt = dx ? dx + static_cast<int64_t>(t) * n : nullptr;
  float *yt = y + static_cast<int64_t>(t) * n;
  float ss = 0.f;
  for (int i = tid; i < n; i += blockDim.x) {
    float v = xt[i];
    if (dxt) {
      v += dxt[i];
      xt[i] = v;
    }
    ss += v * v;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (lane == 0) part[warp] = ss;
  __syncthreads();
  if (warp == 0) {
    float s = lane < (blockDim.x >> 5) ? part[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) part[0] = s;
  }
  __syncthreads();
  const float scale = 1.0f / sqrtf(part[0] / static_cast<float>(n) + eps);
  bool bad = false;
  for (int i = tid; i < n; i += blockDim.x) {
    const float v = xt[i] * scale * w[i];
    bad |= !isfinite(v);
    yt[i] = v;
  }
  if (__any_sync(0xffffffffu, bad) && lane == 0) status_or(status, ST_NONFINITE_IN);
}

// Thread (token t = blockIdx.x, pair j of head-pair slot): the query and key heads get their
// bias and rotation (rope_bias / prefill_rope, gpu_prefill.cu:73-81), the rotated query goes to
// q, the rotated key and the biased value into the cache at position pos0 + t (rounded to fp16
// in an fp16 cache).
template <typename KV>
__global__ void __launch_bounds__(256) pf_rope_kv_kernel(PrefillAttn a) {
  const int t = blockIdx.x;
  const int pos = a.pos0 + t;
  const int qr = a.n_head * kHD, kr = a.n_kv * kHD;
  const float *row = a.qkv + static_cast<int64_t>(t) * a.ld;
  const float2 *rope = a.rope + static_cast<size_t>(pos) * (kHD / 2);
  const int pairs = (a.n_head + a.n_kv) * (kHD / 2);
  KV *kc = static_cast<KV *>(a.kcache), *vc = static_cast<KV *>(a.vcache);
  for (int i = threadIdx.x; i < pairs + kr; i += blockDim.x) {
    if (i < pairs) {
      const int h = i / (kHD / 2), j = i % (kHD / 2);
      const bool is_q = h < a.n_head;
      const int r0 = is_q ? h * kHD + j : qr + (h - a.n_head) * kHD + j;
      const float b0 = a.bias ? a.bias[r0] : 0.f, b1 = a.bias ? a.bias[r0 + kHD / 2] : 0.f;
      const float u = row[r0] + b0, v = row[r0 + kHD / 2] + b1;
      const float2 cs = rope[j];
      const float lo = u * cs.x - v * cs.y, hi = u * cs.y + v * cs.x;
      if (is_q) {
        float *q = a.q + static_cast<int64_t>(t) * qr + h * kHD;
        q[j] = lo;
        q[j + kHD / 2] = hi;
      } else {
        KV *k = kc + (static_cast<size_t>(h - a.n_head) * a.n_ctx + pos) * kHD;
        KvIO<KV>::store(k + j, lo);
        KvIO<KV>::store(k + j + kHD / 2, hi);
      }
    } else {
      const int e = i - pairs, kvh = e / kHD, d = e % kHD;
      const int r = qr + kr + e;
      KvIO<KV>::store(vc + (static_cast<size_t>(kvh) * a.n_ctx + pos) * kHD + d, row[r] + (a.bias ? a.bias[r] : 0.f));
    }
  }
}

// Causal attention of query head h = blockIdx.y for the kQT prompt tokens of tile blockIdx.x
// over the cache positions [0, pos0 + t] of each (prefill_attention, gpu_prefill.cu:82-101;
// fused_attention's arithmetic).  The cache is read in 64-position chunks into shared memory
// as fp32; each query row keeps a running max m, a running sum l and its output o, rescaled by
// exp(m_old - m_new) when a chunk raises the max.  Threads: 16 per query row; thread (r, c)
// scores keys c, c + 16, c + 32, c + 48 of the chunk and owns output dims 8c .. 8c + 7.
constexpr int kQT = 16;   // query tokens per CTA
constexpr int kKC = 64;   // cache positions per chunk
constexpr int kPadK = kHD + 1;
// shared memory: queries [kQT][kHD], keys [kKC][kPadK], values [kKC][kHD], probabilities [kQT][kKC]
constexpr size_t kAttnSmem = sizeof(float) * (kQT * kHD + kKC * kPadK + kKC * kHD + kQT * kKC);
static_assert((kQT * kHD + kKC * kPadK) % 4 == 0, "values must start 16-byte aligned");

template <typename KV>
__global__ void __launch_bounds__(256) pf_attention_kernel(PrefillAttn a) {
  extern __shared__ __align__(16) float sm[];
  float(*qs)[kHD] = reinterpret_cast<float(*)[kHD]>(sm);
  float(*ks)[kPadK] = reinterpret_cast<float(*)[kPadK]>(sm + kQT * kHD);
  float(*vs)[kHD] = reinterpret_cast<float(*)[kHD]>(sm + kQT * kHD + kKC * kPadK);
  float(*ps)[kKC] = reinterpret_cast<float(*)[kKC]>(sm + kQT * kHD + kKC * kPadK + kKC * kHD);
  const int tid = threadIdx.x, r = tid >> 4, c = tid & 15;
  const int t0 = blockIdx.x * kQT, h = blockIdx.y;
  const int G = a.n_head / a.n_kv, kvh = h / G;
  const int qr = a.n_head * kHD;
  const int t = t0 + r;                       // this thread's query token
  const bool live = t < a.n;
  const int my_pos = a.pos0 + min(t, a.n - 1);  // its position (the last token's for padding rows)
  const int last = a.pos0 + min(t0 + kQT, a.n) - 1;  // the tile's last query position
  for (int i = tid; i < kQT * kHD; i += blockDim.x) {
    const int rr = i / kHD, d = i % kHD;
    const int tt = min(t0 + rr, a.n - 1);
    qs[rr][d] = a.q[static_cast<int64_t>(tt) * qr + h * kHD + d];
  }
  const KV *kc = static_cast<const KV *>(a.kcache) + static_cast<size_t>(kvh) * a.n_ctx * kHD;
  const KV *vc = static_cast<const KV *>(a.vcache) + static_cast<size_t>(kvh) * a.n_ctx * kHD;
  const float inv_sqrt = 1.0f / sqrtf(static_cast<float>(kHD));
  float m = -FLT_MAX, l = 0.f, o[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i] = 0.f;
  for (int p0 = 0; p0 <= last; p0 += kKC) {
    const int np = min(kKC, last + 1 - p0);
    __syncthreads();  // the previous chunk is consumed (and qs written, for the first)
    for (int i = tid; i < kKC * (kHD / 4); i += blockDim.x) {
      const int pp = i / (kHD / 4), d = (i % (kHD / 4)) * 4;
      float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
      if (pp < np) {
        kv = KvIO<KV>::load4(kc + static_cast<size_t>(p0 + pp) * kHD + d);
        vv = KvIO<KV>::load4(vc + static_cast<size_t>(p0 + pp) * kHD + d);
      }
      ks[pp][d] = kv.x;
      ks[pp][d + 1] = kv.y;
      ks[pp][d + 2] = kv.z;
      ks[pp][d + 3] = kv.w;
      *reinterpret_cast<float4 *>(&vs[pp][d]) = vv;
    }
    __syncthreads();
    float s[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) s[j] = 0.f;
#pragma unroll 8
    for (int d = 0; d < kHD; ++d) {
      const float qv = qs[r][d];
#pragma unroll
      for (int j = 0; j < 4; ++j) s[j] += qv * ks[c + 16 * j][d];
    }
    float cmax = -FLT_MAX;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int pp = c + 16 * j;
      s[j] = (pp < np && p0 + pp <= my_pos) ? s[j] * inv_sqrt : -FLT_MAX;  // causal mask
      cmax = fmaxf(cmax, s[j]);
    }
#pragma unroll
    for (int off = 8; off > 0; off >>= 1) cmax = fmaxf(cmax, __shfl_xor_sync(0xffffffffu, cmax, off));
    const float m_new = fmaxf(m, cmax);  // finite: position 0 is never masked
    const float resc = expf(m - m_new);
    float csum = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float e = s[j] == -FLT_MAX ? 0.f : expf(s[j] - m_new);
      ps[r][c + 16 * j] = e;
      csum += e;
    }
#pragma unroll
    for (int off = 8; off > 0; off >>= 1) csum += __shfl_xor_sync(0xffffffffu, csum, off);
    l = l * resc + csum;
    m = m_new;
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] *= resc;
    for (int pp = 0; pp < np; ++pp) {
      const float pv = ps[r][pp];
      const float4 v0 = *reinterpret_cast<const float4 *>(&vs[pp][8 * c]);
      const float4 v1 = *reinterpret_cast<const float4 *>(&vs[pp][8 * c + 4]);
      o[0] += pv * v0.x;
      o[1] += pv * v0.y;
      o[2] += pv * v0.z;
      o[3] += pv * v0.w;
      o[4] += pv * v1.x;
      o[5] += pv * v1.y;
      o[6] += pv * v1.z;
      o[7] += pv * v1.w;
    }
  }
  if (live) {
    const float inv = 1.0f / l;
    float *out = a.out + static_cast<int64_t>(t) * qr + h * kHD + 8 * c;
    *reinterpret_cast<float4 *>(out) = make_float4(o[0] * inv, o[1] * inv, o[2] * inv, o[3] * inv);
    *reinterpret_cast<float4 *>(out + 4) = make_float4(o[4] * inv, o[5] * inv, o[6] * inv, o[7] * inv);
  }
}

// h[t][i] = SiLU(g) * u of the gate / up GEMM rows (silu_mul of the prefill graph).
__global__ void __launch_bounds__(256) pf_silu_kernel(const float *__restrict__ gu, int64_t ld, int n_ff,
                                                      float *__restrict__ h) {
  const int t = blockIdx.y;
  const float *row = gu + static_cast<int64_t>(t) * ld;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n_ff; i += gridDim.x * blockDim.x) {
    const float g = row[i], u = row[n_ff + i];
    h[static_cast<int64_t>(t) * n_ff + i] = (g / (1.0f + expf(-g))) * u;
  }
}

}  // namespace

ugb_status launch_pf_embed(cudaStream_t s, const uint8_t *tok_embd, const int32_t *tokens, int n, int embd, int vocab,
                           float *x, uint32_t *status) {
  pf_embed_kernel<<<n, 256, 0, s>>>(tok_embd, tokens, embd, vocab, x, status);
  return cuda_status(cudaGetLastError());
}

ugb_status launch_pf_rmsnorm(cudaStream_t s, float *x, const float *dx, const float *w, int n, int embd, float eps,
                             float *y, uint32_t *status) {
  pf_rmsnorm_kernel<<<n, 512, 0, s>>>(x, dx, w, embd, eps, y, status);
  return cuda_status(cudaGetLastError());
}

ugb_status launch_pf_rope_kv(cudaStream_t s, const PrefillAttn &a) {
  if (a.kv16)
    pf_rope_kv_kernel<__half><<<a.n, 256, 0, s>>>(a);
  else
    pf_rope_kv_kernel<float><<<a.n, 256, 0, s>>>(a);
  return cuda_status(cudaGetLastError());
}

ugb_status init_prefill_step_kernels(ugb_ctx *ctx) {
  if (ctx->smem_optin < kAttnSmem) return UGB_EBACKEND;
  if (cudaFuncSetAttribute(pf_attention_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(kAttnSmem)) != cudaSuccess)
    return UGB_EBACKEND;
  return cuda_status(cudaFuncSetAttribute(pf_attention_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          static_cast<int>(kAttnSmem)));
}

ugb_status launch_pf_attention(cudaStream_t s, const PrefillAttn &a) {
  const dim3 grid((a.n + kQT - 1) / kQT, a.n_head);
  if (a.kv16)
    pf_attention_kernel<__half><<<grid, 256, kAttnSmem, s>>>(a);
  else
    pf_attention_kernel<float><<<grid, 256, kAttnSmem, s>>>(a);
  return cuda_status(cudaGetLastError());
}

ugb_status launch_pf_silu(cudaStream_t s, const float *gu, int64_t ld, int n, int n_ff, float *h) {
  const dim3 grid((n_ff + 255) / 256, n);
  pf_silu_kernel<<<grid, 256, 0, s>>>(gu, ld, n_ff, h);
  return cuda_status(cudaGetLastError());
}

}  // namespace ugb
