// decode.cu -- the per-token glue around the quantised matvecs of a Qwen2-style decoder, for a
// batch of up to 8 sequences decoded together.
//
// The reference runs the same steps as separate kernels in its prebuilt decode command list
// (gpu_graph.rs:139-162): fused_resnorm -> quant_act -> qkv_dp4a -> rope_bias ->
// fused_attention -> quant_act -> linear(o) -> fused_resnorm -> quant_act -> gateup_dp4a ->
// quant_act -> linear(down), then the output head and greedy_tiles/greedy_finish.  Here each
// glue step also produces the Q8_1 activation its consumer needs, attention is split over the
// context (flash-decoding), and greedy selection is one atomicMax on an order-preserving
// (value, id) key.  Every kernel takes part in programmatic dependent launch: it lets the next
// kernel start, then waits for its own inputs.  Sequence b of a batch is a grid dimension.
#include <algorithm>
#include <cfloat>
#include <cmath>

#include "common.cuh"
#include "decode.hpp"
#include "glue.cuh"

namespace ugb {
namespace {

// Vector b of a Q8_1 buffer of length-n vectors: (quants, scales, sums).
struct Q8View {
  int8_t *q;
  float *d;
  int32_t *s;
};
__device__ __forceinline__ Q8View q8_vec(uint8_t *buf, int n, size_t d_off, size_t s_off, int nbp, int b) {
  Q8View v;
  v.q = reinterpret_cast<int8_t *>(buf) + static_cast<int64_t>(b) * n;
  v.d = reinterpret_cast<float *>(buf + d_off) + static_cast<int64_t>(b) * nbp;
  v.s = reinterpret_cast<int32_t *>(buf + s_off) + static_cast<int64_t>(b) * nbp;
  return v;
}

// ---- embedding --------------------------------------------------------------------------

// Sequence b = blockIdx.x: its token is the previous step's greedy choice when there is one,
// else the host-provided token; x[b] = dequantised Q8_0 embedding row (embedding_q8,
// gpu_embedding.cu:3-9; frontier_core.rs:79).  When the keys are set the shared position
// advances (sequence 0's CTA moves it); a position that would run past the KV cache is pinned
// to its last slot and flagged, so no later kernel of the step indexes outside the cache.
// The keys are cleared by the next kernel, after every sequence has read its own.
__global__ void __launch_bounds__(512) embed_kernel(const uint8_t *__restrict__ tok_embd, int embd, int vocab,
                                                    int n_ctx, DecodeState *state, float *__restrict__ x,
                                                    uint32_t *status) {
  grid_dep_launch();
  grid_dep_wait();
  const int b = blockIdx.x;
  __shared__ int tok_s;
  if (threadIdx.x == 0) {
    const unsigned long long key = state->key[b];
    int tok = key != 0 ? static_cast<int>(key_id(key)) : state->token[b];
    if (b == 0) {
      int pos = state->pos + (key != 0 ? 1 : 0);
      if (pos < 0 || pos >= n_ctx) {
        status_or(status, ST_BADARG);
        pos = pos < 0 ? 0 : n_ctx - 1;
      }
      state->pos = pos;
    }
    if (tok < 0 || tok >= vocab) {
      status_or(status, ST_BADARG);
      tok = 0;
    }
    state->token[b] = tok;
    tok_s = tok;
  }
  __syncthreads();
  const uint8_t *row = tok_embd + static_cast<uint64_t>(tok_s) * (embd / 32) * 34;
  float *xb = x + static_cast<int64_t>(b) * embd;
  for (int i = threadIdx.x; i < embd; i += blockDim.x) {
    const uint8_t *blk = row + (i / 32) * 34;
    const uint32_t h = blk[0] | (static_cast<uint32_t>(blk[1]) << 8);
    xb[i] = half_bits_to_float(h) * static_cast<float>(static_cast<int8_t>(blk[2 + (i & 31)]));
  }
}

// ---- residual add + RMSNorm + quant -----------------------------------------------------

// Sequence b = blockIdx.x: x += dx (when dx is given); y = x * (1/sqrt(mean(x^2) + eps)) * w;
// xq[b] = Q8_1(y).  One CTA of 1024 threads per sequence; the sum of squares is a fixed-order
// tree (fused_resnorm, gpu_fused.cu:28-35; llm.rs:323-327 on the CPU).  With clear_keys set
// (the first norm of a step) the CTA also clears its sequence's greedy key, which the
// embedding kernel has consumed by now.
__global__ void __launch_bounds__(1024) rmsnorm_quant_kernel(float *__restrict__ x, const float *__restrict__ dx,
                                                             const float *__restrict__ w, int n, float eps,
                                                             uint8_t *__restrict__ xq, size_t d_off, size_t s_off,
                                                             int nbp, DecodeState *clear_keys, uint32_t *status,
                                                             float *__restrict__ pre) {
  grid_dep_launch();
  grid_dep_wait();
  __shared__ float part[32];
  const int b = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (clear_keys && tid == 0) clear_keys->key[b] = 0;
  float *xb = x + static_cast<int64_t>(b) * n;
  const float *dxb = dx ? dx + static_cast<int64_t>(b) * n : nullptr;
  float ss = 0.f;
  for (int i = tid; i < n; i += blockDim.x) {
    float v = xb[i];
    if (dxb) {
      v += dxb[i];
      xb[i] = v;
    }
    ss += v * v;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (lane == 0) part[warp] = ss;
  __syncthreads();
  if (warp == 0) {
    float t = lane < (blockDim.x >> 5) ? part[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (lane == 0) part[0] = t;
  }
  __syncthreads();
  const float scale = 1.0f / sqrtf(part[0] / static_cast<float>(n) + eps);
  const Q8View v = q8_vec(xq, n, d_off, s_off, nbp, b);
  bool bad = false;
  const int nb = n / 32;
  for (int blk = warp; blk < nb; blk += blockDim.x >> 5) {
    const int i = blk * 32 + lane;
    const float y = xb[i] * scale * w[i];
    if (pre) pre[static_cast<int64_t>(b) * n + i] = y;
    bad |= quant_block(y, lane, v.q, v.d, v.s, blk);
  }
  for (int blk = nb + tid; blk < nbp; blk += blockDim.x) {
    v.d[blk] = 0.f;
    v.s[blk] = 0;
  }
  if (bad && lane == 0) status_or(status, ST_NONFINITE_IN);
}

// ---- SiLU(gate) * up + quant ------------------------------------------------------------

// h = (g / (1 + exp(-g))) * u per element (gateup_dp4a epilogue, gpu_dp4a.cu:63), quantised
// per 32-block; gu[b] holds [gate rows ; up rows] of sequence b = blockIdx.y.  One warp per
// block.
__global__ void __launch_bounds__(256) silu_quant_kernel(const float *__restrict__ gu, int n_ff,
                                                         uint8_t *__restrict__ hq, size_t d_off, size_t s_off,
                                                         int nbp, uint32_t *status, float *__restrict__ pre) {
  grid_dep_launch();
  grid_dep_wait();
  const int lane = threadIdx.x & 31;
  const int blk = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int b = blockIdx.y;
  const Q8View v = q8_vec(hq, n_ff, d_off, s_off, nbp, b);
  const int nb = n_ff / 32;
  if (blk >= nbp) return;
  if (blk >= nb) {
    if (lane == 0) {
      v.d[blk] = 0.f;
      v.s[blk] = 0;
    }
    return;
  }
  const float *g = gu + static_cast<int64_t>(b) * 2 * n_ff;
  const float gv = g[blk * 32 + lane], uv = g[n_ff + blk * 32 + lane];
  const float h = (gv / (1.0f + expf(-gv))) * uv;
  if (pre) pre[static_cast<int64_t>(b) * n_ff + blk * 32 + lane] = h;
  if (quant_block(h, lane, v.q, v.d, v.s, blk) && lane == 0) status_or(status, ST_NONFINITE_IN);
}

// ---- attention ------------------------------------------------------------------------------

// Flash-decoding over one KV head (blockIdx.x) and one context chunk of kAttnChunk positions
// (blockIdx.y) of sequence b = blockIdx.z: the G query heads of the group get their bias and
// RoPE (rope_bias, gpu_ops.cu:9-20: a = v0*c - v1*s, b = v0*s + v1*c over pairs
// (i, i + HD/2)), the chunk holding `pos` also biases, rotates and stores the new key and
// value (fp32 cache as the reference keeps it, gpu_attention.cu:1, or fp16), and every chunk writes
// unnormalised partials (max, sum of exp, exp-weighted V) for the combine step.  Scores are
// q.k / sqrt(HD) with an exact expf softmax (fused_attention, gpu_attention.cu:2-26;
// llm.rs:358-368).
// Batch-1 form: keys and values converted to fp32 as they are staged, one accumulator per dot.
// With few CTAs (one sequence: n_kv x chunks) it measured faster than the form below (C5 batch 1:
// 181.2 vs 172.1 tok/s, A/B on one box); with a batch the form below fits twice the CTAs per SM
// and wins (C4 batch 8: attention 30.8 -> 20.2 us per launch).
// Flash-decoding over one KV head (blockIdx.x) and one context chunk of kAttnChunk positions
// (blockIdx.y) of sequence b = blockIdx.z: the G query heads of the group get their bias and
// RoPE (rope_bias, gpu_ops.cu:9-20: a = v0*c - v1*s, b = v0*s + v1*c over pairs
// (i, i + HD/2)), the chunk holding `pos` also biases, rotates and stores the new key and
// value (fp32 cache as the reference keeps it, gpu_attention.cu:1, or fp16), and every chunk writes
// unnormalised partials (max, sum of exp, exp-weighted V) for the combine step.  Scores are
// q.k / sqrt(HD) with an exact expf softmax (fused_attention, gpu_attention.cu:2-26;
// llm.rs:358-368).
template <int HD, typename KV>
__global__ void __launch_bounds__(256) attn_partial_f32_kernel(AttnParams a) {
  extern __shared__ __align__(16) float sm[];
  const int G = a.n_head / a.n_kv;
  float *q_s = sm;                          // [G][HD] (raw, then rotated)
  float *r_s = q_s + G * HD;                // [G][HD] raw q before rotation
  float *ks = r_s + G * HD;                 // [CH][HD + 1]
  float *vs = ks + kAttnChunk * (HD + 1);   // [CH][HD]
  float *ps = vs + kAttnChunk * HD;         // [G][CH]
  float *kn = ps + G * kAttnChunk;          // [2][HD] new key / value (raw)
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int kvh = blockIdx.x, sp = blockIdx.y, b = blockIdx.z;
  grid_dep_launch();
  grid_dep_wait();
  const int pos = a.state->pos;
  const int t0 = sp * kAttnChunk;
  const size_t part = (static_cast<size_t>(b) * a.n_kv + kvh) * a.n_split + sp;
  float *pm = a.part_m + part * G;
  float *pl = a.part_l + part * G;
  float *po = a.part_o + part * G * HD;
  if (pos < 0 || pos >= a.n_ctx) {  // the embedding step pins pos; this is a second guard
    if (tid == 0 && sp == 0 && kvh == 0 && b == 0) status_or(a.status, ST_BADARG);
    return;
  }
  if (t0 > pos) return;  // the combine step only reads chunks <= pos / kAttnChunk
  const int nt = min(kAttnChunk, pos + 1 - t0);
  const int qrows = a.n_head * HD, kvrows = a.n_kv * HD;
  const float *qkv = a.qkv + static_cast<int64_t>(b) * (qrows + 2 * kvrows);
  const float2 *rope = a.rope + static_cast<size_t>(pos) * (HD / 2);
  const bool has_new = pos < t0 + kAttnChunk;
  for (int i = tid; i < G * HD; i += blockDim.x) {
    const int row = (kvh * G) * HD + i;
    r_s[i] = qkv[row] + (a.bias ? a.bias[row] : 0.f);
  }
  if (has_new) {
    for (int i = tid; i < 2 * HD; i += blockDim.x) {
      const int row = qrows + (i < HD ? 0 : kvrows) + kvh * HD + (i % HD);
      kn[i] = qkv[row] + (a.bias ? a.bias[row] : 0.f);
    }
  }
  __syncthreads();
  for (int i = tid; i < G * HD; i += blockDim.x) {
    const int dd = i % HD, base = i - dd, j = dd % (HD / 2);
    const float2 cs = rope[j];
    const float v0 = r_s[base + j], v1 = r_s[base + j + HD / 2];
    q_s[i] = dd < HD / 2 ? v0 * cs.x - v1 * cs.y : v0 * cs.y + v1 * cs.x;
  }
  KV *kcache = static_cast<KV *>(a.kcache) + static_cast<int64_t>(b) * a.cache_seq;
  KV *vcache = static_cast<KV *>(a.vcache) + static_cast<int64_t>(b) * a.cache_seq;
  const size_t cache_head = (static_cast<size_t>(kvh) * a.n_ctx) * HD;
  if (has_new && tid < HD) {
    const int j = tid % (HD / 2);
    const float2 cs = rope[j];
    const float v0 = kn[j], v1 = kn[j + HD / 2];
    // the new row takes part as the cache holds it (rounded to fp16 in an fp16 cache)
    const float k = KvIO<KV>::round(tid < HD / 2 ? v0 * cs.x - v1 * cs.y : v0 * cs.y + v1 * cs.x);
    const float v = KvIO<KV>::round(kn[HD + tid]);
    KvIO<KV>::store(kcache + cache_head + static_cast<size_t>(pos) * HD + tid, k);
    KvIO<KV>::store(vcache + cache_head + static_cast<size_t>(pos) * HD + tid, v);
    ks[(pos - t0) * (HD + 1) + tid] = k;
    vs[(pos - t0) * HD + tid] = v;
  }
  const int n_old = has_new ? nt - 1 : nt;
  {
    const KV *kc = kcache + cache_head + static_cast<size_t>(t0) * HD;
    const KV *vc = vcache + cache_head + static_cast<size_t>(t0) * HD;
    for (int i = tid; i < n_old * (HD / 4); i += blockDim.x) {
      const int t = i / (HD / 4), dd = (i - t * (HD / 4)) * 4;
      const float4 kv = KvIO<KV>::load4(kc + 4 * i), vv = KvIO<KV>::load4(vc + 4 * i);
      float *kd = ks + t * (HD + 1) + dd;
      kd[0] = kv.x;
      kd[1] = kv.y;
      kd[2] = kv.z;
      kd[3] = kv.w;
      *reinterpret_cast<float4 *>(vs + t * HD + dd) = vv;
    }
  }
  __syncthreads();
  const float inv_sqrt = 1.0f / sqrtf(static_cast<float>(HD));
  for (int i = tid; i < G * nt; i += blockDim.x) {
    const int g = i / nt, t = i - g * nt;
    const float *qg = q_s + g * HD, *kt = ks + t * (HD + 1);
    float dot = 0.f;
#pragma unroll 8
    for (int dd = 0; dd < HD; ++dd) dot += qg[dd] * kt[dd];
    ps[g * kAttnChunk + t] = dot * inv_sqrt;
  }
  __syncthreads();
  if (warp < G) {
    float mx = -FLT_MAX;
    for (int t = lane; t < nt; t += 32) mx = fmaxf(mx, ps[warp * kAttnChunk + t]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.f;
    for (int t = lane; t < nt; t += 32) {
      const float e = expf(ps[warp * kAttnChunk + t] - mx);
      ps[warp * kAttnChunk + t] = e;
      sum += e;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) {
      pm[warp] = mx;
      pl[warp] = sum;
    }
  }
  __syncthreads();
  for (int i = tid; i < G * HD; i += blockDim.x) {
    const int g = i / HD, dd = i - g * HD;
    float acc = 0.f;
    for (int t = 0; t < nt; ++t) acc += ps[g * kAttnChunk + t] * vs[t * HD + dd];
    po[i] = acc;
  }
}

// Keys and values stay in shared memory in the cache's element type (an fp16 cache takes half the
// space, so twice the CTAs fit an SM); key rows are padded to an odd word count, so the lanes of
// a warp (consecutive positions) read distinct banks.
template <typename KV>
struct AttnSmem {
  static constexpr int kKeyStride = sizeof(KV) == 2 ? kHeadDim + 2 : kHeadDim + 1;  // elements
};

template <int HD, typename KV>
__global__ void __launch_bounds__(256) attn_partial_kernel(AttnParams a) {
  extern __shared__ __align__(16) float sm[];
  constexpr int KS = AttnSmem<KV>::kKeyStride;
  const int G = a.n_head / a.n_kv;
  float *q_s = sm;                          // [G][HD] (raw, then rotated)
  float *r_s = q_s + G * HD;                // [G][HD] raw q before rotation
  KV *ks = reinterpret_cast<KV *>(r_s + G * HD);  // [CH][KS]
  KV *vs = ks + kAttnChunk * KS;            // [CH][HD]
  float *ps = reinterpret_cast<float *>(vs + kAttnChunk * HD);  // [G][CH]
  float *kn = ps + G * kAttnChunk;          // [2][HD] new key / value (raw)
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int kvh = blockIdx.x, sp = blockIdx.y, b = blockIdx.z;
  grid_dep_launch();
  grid_dep_wait();
  const int pos = a.state->pos;
  const int t0 = sp * kAttnChunk;
  const size_t part = (static_cast<size_t>(b) * a.n_kv + kvh) * a.n_split + sp;
  float *pm = a.part_m + part * G;
  float *pl = a.part_l + part * G;
  float *po = a.part_o + part * G * HD;
  if (pos < 0 || pos >= a.n_ctx) {  // the embedding step pins pos; this is a second guard
    if (tid == 0 && sp == 0 && kvh == 0 && b == 0) status_or(a.status, ST_BADARG);
    return;
  }
  if (t0 > pos) return;  // the combine step only reads chunks <= pos / kAttnChunk
  const int nt = min(kAttnChunk, pos + 1 - t0);
  const int qrows = a.n_head * HD, kvrows = a.n_kv * HD;
  const float *qkv = a.qkv + static_cast<int64_t>(b) * (qrows + 2 * kvrows);
  const float2 *rope = a.rope + static_cast<size_t>(pos) * (HD / 2);
  const bool has_new = pos < t0 + kAttnChunk;
  for (int i = tid; i < G * HD; i += blockDim.x) {
    const int row = (kvh * G) * HD + i;
    r_s[i] = qkv[row] + (a.bias ? a.bias[row] : 0.f);
  }
  if (has_new) {
    for (int i = tid; i < 2 * HD; i += blockDim.x) {
      const int row = qrows + (i < HD ? 0 : kvrows) + kvh * HD + (i % HD);
      kn[i] = qkv[row] + (a.bias ? a.bias[row] : 0.f);
    }
  }
  __syncthreads();
  for (int i = tid; i < G * HD; i += blockDim.x) {
    const int dd = i % HD, base = i - dd, j = dd % (HD / 2);
    const float2 cs = rope[j];
    const float v0 = r_s[base + j], v1 = r_s[base + j + HD / 2];
    q_s[i] = dd < HD / 2 ? v0 * cs.x - v1 * cs.y : v0 * cs.y + v1 * cs.x;
  }
  KV *kcache = static_cast<KV *>(a.kcache) + static_cast<int64_t>(b) * a.cache_seq;
  KV *vcache = static_cast<KV *>(a.vcache) + static_cast<int64_t>(b) * a.cache_seq;
  const size_t cache_head = (static_cast<size_t>(kvh) * a.n_ctx) * HD;
  if (has_new && tid < HD) {
    const int j = tid % (HD / 2);
    const float2 cs = rope[j];
    const float v0 = kn[j], v1 = kn[j + HD / 2];
    // the new row takes part as the cache holds it (rounded to fp16 in an fp16 cache)
    const float k = KvIO<KV>::round(tid < HD / 2 ? v0 * cs.x - v1 * cs.y : v0 * cs.y + v1 * cs.x);
    const float v = KvIO<KV>::round(kn[HD + tid]);
    KvIO<KV>::store(kcache + cache_head + static_cast<size_t>(pos) * HD + tid, k);
    KvIO<KV>::store(vcache + cache_head + static_cast<size_t>(pos) * HD + tid, v);
    KvIO<KV>::store(ks + (pos - t0) * KS + tid, k);  // exact: k and v are already rounded
    KvIO<KV>::store(vs + (pos - t0) * HD + tid, v);
  }
  const int n_old = has_new ? nt - 1 : nt;
  {
    const KV *kc = kcache + cache_head + static_cast<size_t>(t0) * HD;
    const KV *vc = vcache + cache_head + static_cast<size_t>(t0) * HD;
    for (int i = tid; i < n_old * (HD / 4); i += blockDim.x) {
      const int t = i / (HD / 4), dd = (i - t * (HD / 4)) * 4;
      KV *kd = ks + t * KS + dd;
      if constexpr (sizeof(KV) == 2) {  // 8 bytes each; key rows are 4-byte aligned
        const uint2 kv = *reinterpret_cast<const uint2 *>(kc + 4 * i), vv = *reinterpret_cast<const uint2 *>(vc + 4 * i);
        reinterpret_cast<uint32_t *>(kd)[0] = kv.x;
        reinterpret_cast<uint32_t *>(kd)[1] = kv.y;
        *reinterpret_cast<uint2 *>(vs + t * HD + dd) = vv;
      } else {
        const float4 kv = KvIO<KV>::load4(kc + 4 * i), vv = KvIO<KV>::load4(vc + 4 * i);
        kd[0] = kv.x;
        kd[1] = kv.y;
        kd[2] = kv.z;
        kd[3] = kv.w;
        *reinterpret_cast<float4 *>(vs + t * HD + dd) = vv;
      }
    }
  }
  __syncthreads();
  const float inv_sqrt = 1.0f / sqrtf(static_cast<float>(HD));
  // Scores: one (query head, position) per thread; four partial sums shorten the FMA chain.
  for (int i = tid; i < G * nt; i += blockDim.x) {
    const int g = i / nt, t = i - g * nt;
    const float *qg = q_s + g * HD;
    const KV *kt = ks + t * KS;
    float d0 = 0.f, d1 = 0.f, d2 = 0.f, d3 = 0.f;
#pragma unroll 8
    for (int dd = 0; dd < HD; dd += 4) {
      const float4 q4 = *reinterpret_cast<const float4 *>(qg + dd);  // same address across the warp
      float k0, k1, k2, k3;
      if constexpr (sizeof(KV) == 2) {
        const float2 a01 = __half22float2(*reinterpret_cast<const __half2 *>(kt + dd));
        const float2 a23 = __half22float2(*reinterpret_cast<const __half2 *>(kt + dd + 2));
        k0 = a01.x, k1 = a01.y, k2 = a23.x, k3 = a23.y;
      } else {
        k0 = kt[dd], k1 = kt[dd + 1], k2 = kt[dd + 2], k3 = kt[dd + 3];
      }
      d0 = fmaf(q4.x, k0, d0);
      d1 = fmaf(q4.y, k1, d1);
      d2 = fmaf(q4.z, k2, d2);
      d3 = fmaf(q4.w, k3, d3);
    }
    ps[g * kAttnChunk + t] = ((d0 + d1) + (d2 + d3)) * inv_sqrt;
  }
  __syncthreads();
  if (warp < G) {
    float mx = -FLT_MAX;
    for (int t = lane; t < nt; t += 32) mx = fmaxf(mx, ps[warp * kAttnChunk + t]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.f;
    for (int t = lane; t < nt; t += 32) {
      const float e = expf(ps[warp * kAttnChunk + t] - mx);
      ps[warp * kAttnChunk + t] = e;
      sum += e;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) {
      pm[warp] = mx;
      pl[warp] = sum;
    }
  }
  __syncthreads();
  // Probability-weighted values: one (query head, dimension) per thread, four partial sums.
  for (int i = tid; i < G * HD; i += blockDim.x) {
    const int g = i / HD, dd = i - g * HD;
    const float *pg = ps + g * kAttnChunk;
    const KV *vd = vs + dd;
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
    int t = 0;
    for (; t + 4 <= nt; t += 4) {
      const float4 p4 = *reinterpret_cast<const float4 *>(pg + t);  // same address across the warp
      a0 = fmaf(p4.x, KvIO<KV>::load(vd + t * HD), a0);
      a1 = fmaf(p4.y, KvIO<KV>::load(vd + (t + 1) * HD), a1);
      a2 = fmaf(p4.z, KvIO<KV>::load(vd + (t + 2) * HD), a2);
      a3 = fmaf(p4.w, KvIO<KV>::load(vd + (t + 3) * HD), a3);
    }
    for (; t < nt; ++t) a0 = fmaf(pg[t], KvIO<KV>::load(vd + t * HD), a0);
    po[i] = (a0 + a1) + (a2 + a3);
  }
}

// Combine the chunk partials of query head blockIdx.x of sequence blockIdx.y (log-sum-exp)
// and quantise the head's HD outputs into the Q8_1 input of the output projection.
template <int HD>
__global__ void __launch_bounds__(HD) attn_combine_quant_kernel(AttnParams a, uint8_t *__restrict__ xq,
                                                                size_t d_off, size_t s_off, int nbp,
                                                                float *__restrict__ pre) {
  grid_dep_launch();
  grid_dep_wait();
  const int G = a.n_head / a.n_kv;
  const int h = blockIdx.x, b = blockIdx.y, kvh = h / G, g = h - kvh * G;
  const int dd = threadIdx.x, lane = dd & 31;
  const int pos = a.state->pos;
  const int ns = (pos >= 0 && pos < a.n_ctx) ? pos / kAttnChunk + 1 : 0;  // 0: flagged upstream
  const size_t part0 = (static_cast<size_t>(b) * a.n_kv + kvh) * a.n_split;
  float mx = -FLT_MAX;
  for (int sp = 0; sp < ns; ++sp) mx = fmaxf(mx, a.part_m[(part0 + sp) * G + g]);
  float l = 0.f, o = 0.f;
  for (int sp = 0; sp < ns; ++sp) {
    const size_t ps = part0 + sp;
    const float e = expf(a.part_m[ps * G + g] - mx);
    l += e * a.part_l[ps * G + g];
    o += e * a.part_o[(ps * G + g) * HD + dd];
  }
  const float v = ns ? o / l : 0.f;
  if (pre) pre[(static_cast<int64_t>(b) * a.n_head + h) * HD + dd] = v;
  const Q8View q = q8_vec(xq, a.n_head * HD, d_off, s_off, nbp, b);
  const int blk = (h * HD + dd) / 32;
  if (quant_block(v, lane, q.q, q.d, q.s, blk) && lane == 0) status_or(a.status, ST_NONFINITE_IN);
}

// ---- greedy ----------------------------------------------------------------------------------

// The largest logit of sequence blockIdx.y (lowest id on ties; ids offset by id0 when this
// device holds a slice of the vocabulary) into the state's greedy key (greedy_tiles /
// greedy_finish, gpu_greedy.cu:13-27).  Non-finite logits are reported by the head matvec.
__global__ void __launch_bounds__(256) argmax_kernel(const float *__restrict__ logits, int n, int id0,
                                                     DecodeState *state) {
  grid_dep_launch();
  grid_dep_wait();
  __shared__ unsigned long long part[8];
  const int b = blockIdx.y;
  const float *lb = logits + static_cast<int64_t>(b) * n;
  uint64_t best = 0;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const float v = lb[i];
    if (isfinite(v)) best = max(best, greedy_key(v, static_cast<uint32_t>(id0 + i)));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) best = max(best, static_cast<uint64_t>(__shfl_xor_sync(0xffffffffu, best, o)));
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < 8; ++w) best = max(best, static_cast<uint64_t>(part[w]));
    atomicMax(&state->key[b], static_cast<unsigned long long>(best));
  }
}

}  // namespace
}  // namespace ugb

namespace ugb {
namespace {

template <typename... KArgs, typename... Args>
ugb_status launch_ex(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                     bool pdl, Args... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...));
}

}  // namespace

size_t attn_partial_f32_smem(int group) {
  return sizeof(float) * (2 * group * kHeadDim + kAttnChunk * (kHeadDim + 1) + kAttnChunk * kHeadDim +
                          group * kAttnChunk + 2 * kHeadDim);
}

size_t attn_partial_smem(int group, bool kv16) {
  const size_t kv = kv16 ? sizeof(__half) * kAttnChunk * (AttnSmem<__half>::kKeyStride + kHeadDim)
                         : sizeof(float) * kAttnChunk * (AttnSmem<float>::kKeyStride + kHeadDim);
  return sizeof(float) * (2 * group * kHeadDim + group * kAttnChunk + 2 * kHeadDim) + kv;
}

ugb_status init_decode_kernels(ugb_ctx *ctx) {
  const int f32_smem = static_cast<int>(std::min<size_t>(ctx->smem_optin, attn_partial_f32_smem(8)));
  if (cudaFuncSetAttribute(attn_partial_f32_kernel<kHeadDim, float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           f32_smem) != cudaSuccess ||
      cudaFuncSetAttribute(attn_partial_f32_kernel<kHeadDim, __half>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           f32_smem) != cudaSuccess)
    return UGB_EBACKEND;
  if (cudaFuncSetAttribute(attn_partial_kernel<kHeadDim, float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(std::min<size_t>(ctx->smem_optin, attn_partial_smem(8, false)))) !=
      cudaSuccess)
    return UGB_EBACKEND;
  return cuda_status(cudaFuncSetAttribute(
      attn_partial_kernel<kHeadDim, __half>, cudaFuncAttributeMaxDynamicSharedMemorySize,
      static_cast<int>(std::min<size_t>(ctx->smem_optin, attn_partial_smem(8, true)))));
}

ugb_status launch_embed(cudaStream_t s, bool pdl, const uint8_t *tok_embd, int embd, int vocab, int n_ctx,
                        int batch, DecodeState *state, float *x, uint32_t *status) {
  return launch_ex(embed_kernel, dim3(batch), dim3(512), 0, s, pdl, tok_embd, embd, vocab, n_ctx, state, x, status);
}

ugb_status launch_rmsnorm_quant(cudaStream_t s, bool pdl, float *x, const float *dx, const float *w, int n,
                                int batch, float eps, uint8_t *xq, DecodeState *clear_keys, uint32_t *status,
                                float *pre) {
  const Q8Act l = q8act_layout(n, batch);
  return launch_ex(rmsnorm_quant_kernel, dim3(batch), dim3(1024), 0, s, pdl, x, dx, w, n, eps, xq, l.d_off,
                   l.s_off, static_cast<int>(l.nbp), clear_keys, status, pre);
}

ugb_status launch_silu_quant(cudaStream_t s, bool pdl, const float *gu, int n_ff, int batch, uint8_t *hq,
                             uint32_t *status, float *pre) {
  const Q8Act l = q8act_layout(n_ff, batch);
  const int warps = static_cast<int>(l.nbp);
  return launch_ex(silu_quant_kernel, dim3((warps + 7) / 8, batch), dim3(256), 0, s, pdl, gu, n_ff, hq, l.d_off,
                   l.s_off, warps, status, pre);
}

ugb_status launch_attention(cudaStream_t s, bool pdl, const AttnParams &a, int batch, uint8_t *xq, float *pre) {
  const int group = a.n_head / a.n_kv;
  const dim3 grid(a.n_kv, a.n_split, batch);
  ugb_status st;
  if (batch == 1) {  // few CTAs: the fp32-staging form (see attn_partial_f32_kernel)
    st = a.kv16 ? launch_ex(attn_partial_f32_kernel<kHeadDim, __half>, grid, dim3(256), attn_partial_f32_smem(group),
                            s, pdl, a)
                : launch_ex(attn_partial_f32_kernel<kHeadDim, float>, grid, dim3(256), attn_partial_f32_smem(group),
                            s, pdl, a);
  } else {
    st = a.kv16 ? launch_ex(attn_partial_kernel<kHeadDim, __half>, grid, dim3(256), attn_partial_smem(group, true), s,
                            pdl, a)
                : launch_ex(attn_partial_kernel<kHeadDim, float>, grid, dim3(256), attn_partial_smem(group, false), s,
                            pdl, a);
  }
  if (st != UGB_OK) return st;
  const Q8Act l = q8act_layout(static_cast<int64_t>(a.n_head) * kHeadDim, batch);
  return launch_ex(attn_combine_quant_kernel<kHeadDim>, dim3(a.n_head, batch), dim3(kHeadDim), 0, s, pdl, a, xq,
                   l.d_off, l.s_off, static_cast<int>(l.nbp), pre);
}

ugb_status launch_argmax(cudaStream_t s, bool pdl, const float *logits, int n, int batch, int id0,
                         DecodeState *state, int sm_count) {
  const int blocks = std::max(1, std::min(sm_count / std::max(1, batch), (n + 255) / 256));
  return launch_ex(argmax_kernel, dim3(blocks, batch), dim3(256), 0, s, pdl, logits, n, id0, state);
}

}  // namespace ugb
