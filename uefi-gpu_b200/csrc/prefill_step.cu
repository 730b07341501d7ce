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
#include <algorithm>
#include <cfloat>
#include <cmath>

#include "common.cuh"
#include "decode.hpp"
#include "glue.cuh"
#include "prefill.hpp"
#include "prefill_quant.cuh"

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

// Sum of the `splits` partial outputs of a split-K GEMM at element i (split stride `stride`), in
// split order: the same value every consumer of the product forms.
__device__ __forceinline__ float split_sum(const float *p, int splits, int64_t stride, int64_t i) {
  float t[kMaxGemmSplits];  // every split's load issued before the first add
#pragma unroll
  for (int s = 0; s < kMaxGemmSplits; ++s) t[s] = s < splits ? p[s * stride + i] : 0.f;
  float v = t[0];
#pragma unroll
  for (int s = 1; s < kMaxGemmSplits; ++s)
    if (s < splits) v += t[s];
  return v;
}

// pf_rmsnorm fused with the quantisation of its output: x[t] += dx[t] (the sum of dx's splits),
// then token t = blockIdx.x's normed row goes straight into the packed GEMM operand (quants q_out,
// scales s_out) with prefill_quant's arithmetic, and into pre[t] (the trace) when given.  Same
// values as pf_rmsnorm then prefill_quant, bit for bit.
__global__ void __launch_bounds__(512) pf_norm_quant_kernel(float *__restrict__ x, const float *__restrict__ dx,
                                                            int dx_splits, int64_t dx_stride,
                                                            const float *__restrict__ w, int n, float eps,
                                                            uint8_t *__restrict__ q_out, float *__restrict__ s_out,
                                                            float *__restrict__ pre, uint32_t *status) {
  __shared__ float part[32];
  const int t = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float *xt = x + static_cast<int64_t>(t) * n;
  float ss = 0.f;
  for (int i = tid; i < n; i += blockDim.x) {
    float v = xt[i];
    if (dx) {
      v += split_sum(dx, dx_splits, dx_stride, static_cast<int64_t>(t) * n + i);
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
  const int nb = n / 32;
  bool bad = false;
  for (int b = warp; b < nb; b += blockDim.x >> 5) {
    const int i = b * 32 + lane;
    const float v = xt[i] * scale * w[i];
    if (pre) pre[static_cast<int64_t>(t) * n + i] = v;
    bad |= pf_quant_block(v, lane, t, b, nb, q_out, s_out);
  }
  if (bad && lane == 0) status_or(status, ST_NONFINITE_IN);
}

// SiLU(g) * u of the gate / up GEMM rows (summed over its splits) quantised per 32-block into the
// packed operand of the down GEMM; pre[t] (the trace) when given.  One warp per kSiluBlocks
// consecutive blocks of a token, every load issued before the first use.
constexpr int kSiluBlocks = 4;

__global__ void __launch_bounds__(256) pf_silu_quant_kernel(const float *__restrict__ gu, int64_t ld, int splits,
                                                            int64_t stride, int n, int n_ff,
                                                            uint8_t *__restrict__ q_out, float *__restrict__ s_out,
                                                            float *__restrict__ pre, uint32_t *status) {
  const int lane = threadIdx.x & 31, nb = n_ff / 32;
  const int per_token = (nb + kSiluBlocks - 1) / kSiluBlocks;
  const int64_t gw = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (gw >= static_cast<int64_t>(n) * per_token) return;  // warp-uniform
  const int b0 = static_cast<int>(gw % per_token) * kSiluBlocks;
  const int64_t t = gw / per_token;
  const float *row = gu + t * ld;
  float g[kSiluBlocks][kMaxGemmSplits], u[kSiluBlocks][kMaxGemmSplits];
#pragma unroll
  for (int k = 0; k < kSiluBlocks; ++k) {
    const int i = min(b0 + k, nb - 1) * 32 + lane;
#pragma unroll
    for (int sp = 0; sp < kMaxGemmSplits; ++sp) {
      g[k][sp] = sp < splits ? row[sp * stride + i] : 0.f;
      u[k][sp] = sp < splits ? row[sp * stride + n_ff + i] : 0.f;
    }
  }
  bool bad = false;
#pragma unroll
  for (int k = 0; k < kSiluBlocks; ++k) {
    if (b0 + k >= nb) break;  // warp-uniform
    float gv = g[k][0], uv = u[k][0];
#pragma unroll
    for (int sp = 1; sp < kMaxGemmSplits; ++sp)
      if (sp < splits) {
        gv += g[k][sp];
        uv += u[k][sp];
      }
    const float h = (gv / (1.0f + expf(-gv))) * uv;
    if (pre) pre[t * n_ff + (b0 + k) * 32 + lane] = h;
    bad |= pf_quant_block(h, lane, t, b0 + k, nb, q_out, s_out);
  }
  if (bad && lane == 0) status_or(status, ST_NONFINITE_IN);
}

// dst[r][i] = the sum of the splits of rows [row0, row0 + rows) of a split-K GEMM output [.][len].
__global__ void __launch_bounds__(256) pf_sum_splits_kernel(const float *__restrict__ src, int splits, int64_t stride,
                                                            int64_t row0, int64_t rows, int64_t len,
                                                            float *__restrict__ dst) {
  const int64_t total = rows * len;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    dst[i] = split_sum(src, splits, stride, row0 * len + i);
}

// Thread (token t = blockIdx.x, rotation pair or value element i): the query and key heads get
// their bias and rotation (rope_bias / prefill_rope, gpu_prefill.cu:73-81) from the Q/K/V GEMM rows
// (summed over its splits); the rotated query goes to q, the rotated key and the biased value into
// the cache at position pos0 + t (rounded to fp16 in an fp16 cache).
template <typename KV>
__global__ void __launch_bounds__(256) pf_rope_kv_kernel(PrefillAttn a) {
  const int t = blockIdx.x;
  const int pos = a.pos0 + t;
  const int qr = a.n_head * kHD, kr = a.n_kv * kHD;
  const int64_t row = static_cast<int64_t>(t) * a.ld;
  const float2 *rope = a.rope + static_cast<size_t>(pos) * (kHD / 2);
  const int pairs = (a.n_head + a.n_kv) * (kHD / 2);
  KV *kc = static_cast<KV *>(a.kcache), *vc = static_cast<KV *>(a.vcache);
  for (int i = threadIdx.x; i < pairs + kr; i += blockDim.x) {
    if (i < pairs) {
      const int h = i / (kHD / 2), j = i % (kHD / 2);
      const bool is_q = h < a.n_head;
      const int r0 = is_q ? h * kHD + j : qr + (h - a.n_head) * kHD + j;
      const float b0 = a.bias ? a.bias[r0] : 0.f, b1 = a.bias ? a.bias[r0 + kHD / 2] : 0.f;
      const float u = split_sum(a.qkv, a.splits, a.split_stride, row + r0) + b0;
      const float v = split_sum(a.qkv, a.splits, a.split_stride, row + r0 + kHD / 2) + b1;
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
      KvIO<KV>::store(vc + (static_cast<size_t>(kvh) * a.n_ctx + pos) * kHD + d,
                      split_sum(a.qkv, a.splits, a.split_stride, row + r) + (a.bias ? a.bias[r] : 0.f));
    }
  }
}

// ---- causal attention: partial items and their combine ------------------------------------
//
// Item (query tile of kAQ tokens = blockIdx.x, KV head = blockIdx.y, chunk group = blockIdx.z):
// the G query heads of the KV head for the tile's tokens (R = 16 G query rows, row g * 16 + token)
// against the cache positions of chunks [z * cpi, (z + 1) * cpi) (kAK positions each) that any of
// the tile's tokens sees.  Q, one chunk of K and of V sit in shared memory as fp32; thread
// (tr, tc) of 16 x 16 scores rows g * 16 + tr (g < G) against keys tc + 16 j (j < 4) and owns
// output dims 4 tc .. 4 tc + 3 and 64 + 4 tc .. 64 + 4 tc + 3 of its rows, so every shared load
// feeds several FMAs.  Per row the item keeps a running max m, sum l and output o over its chunks
// (rescaled by exp(m_old - m_new)) and writes them as one partial; the combine merges an item's
// partials with the log-sum-exp rule (flash-decoding's) and quantises the result.
constexpr int kAQ = 16;            // query tokens per item
constexpr int kAK = 64;            // cache positions per chunk
constexpr int kPadQ = kHD + 4;     // row pitch of Q and K in shared memory (float4 loads spread over banks)

__host__ __device__ constexpr size_t pf_attn_smem(int G) {
  return sizeof(float) * (static_cast<size_t>(16 * G) * kPadQ + kAK * kPadQ + kAK * kHD + 16 * G * (kAK + 1));
}

template <int G, typename KV>
__global__ void __launch_bounds__(256) pf_attn_partial_kernel(PrefillAttn a) {
  constexpr int R = 16 * G;
  extern __shared__ __align__(16) float sm[];
  float *qs = sm;                       // [R][kPadQ]
  float *ks = qs + R * kPadQ;           // [kAK][kPadQ]
  float *vs = ks + kAK * kPadQ;         // [kAK][kHD]
  float *ps = vs + kAK * kHD;           // [R][kAK + 1]
  const int tid = threadIdx.x, tr = tid >> 4, tc = tid & 15;
  const int t0 = blockIdx.x * kAQ, kvh = blockIdx.y;
  const int qr = a.n_head * kHD;
  const int last = a.pos0 + min(t0 + kAQ, a.n) - 1;  // the tile's last query position
  const int c_begin = blockIdx.z * a.cpi, c_end = min(c_begin + a.cpi, last / kAK + 1);
  if (c_begin >= c_end) return;  // no token of the tile sees these chunks
  const int my_pos = a.pos0 + min(t0 + tr, a.n - 1);  // padding rows act as the last token
  for (int i = tid; i < R * (kHD / 4); i += blockDim.x) {
    const int r = i / (kHD / 4), d = (i % (kHD / 4)) * 4, g = r / kAQ, tt = min(t0 + r % kAQ, a.n - 1);
    *reinterpret_cast<float4 *>(qs + r * kPadQ + d) =
        *reinterpret_cast<const float4 *>(a.q + static_cast<int64_t>(tt) * qr + (kvh * G + g) * kHD + d);
  }
  const KV *kc = static_cast<const KV *>(a.kcache) + static_cast<size_t>(kvh) * a.n_ctx * kHD;
  const KV *vc = static_cast<const KV *>(a.vcache) + static_cast<size_t>(kvh) * a.n_ctx * kHD;
  const float inv_sqrt = 1.0f / sqrtf(static_cast<float>(kHD));
  float m[G], l[G], o[G][8];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -FLT_MAX;
    l[g] = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) o[g][i] = 0.f;
  }
  for (int c = c_begin; c < c_end; ++c) {
    const int p0 = c * kAK;
    __syncthreads();  // the previous chunk's K, V and P are consumed (and Q is stored, the first time)
    for (int i = tid; i < kAK * (kHD / 4); i += blockDim.x) {
      const int pp = i / (kHD / 4), d = (i % (kHD / 4)) * 4;
      float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
      if (p0 + pp <= last) {  // positions past the tile's last are not written yet: zeros
        kv = KvIO<KV>::load4(kc + static_cast<size_t>(p0 + pp) * kHD + d);
        vv = KvIO<KV>::load4(vc + static_cast<size_t>(p0 + pp) * kHD + d);
      }
      *reinterpret_cast<float4 *>(ks + pp * kPadQ + d) = kv;
      *reinterpret_cast<float4 *>(vs + pp * kHD + d) = vv;
    }
    __syncthreads();
    float s[G][4];
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
      for (int j = 0; j < 4; ++j) s[g][j] = 0.f;
#pragma unroll 4
    for (int d = 0; d < kHD; d += 4) {
      float4 kf[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) kf[j] = *reinterpret_cast<const float4 *>(ks + (tc + 16 * j) * kPadQ + d);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float4 qf = *reinterpret_cast<const float4 *>(qs + (g * kAQ + tr) * kPadQ + d);
#pragma unroll
        for (int j = 0; j < 4; ++j) s[g][j] += qf.x * kf[j].x + qf.y * kf[j].y + qf.z * kf[j].z + qf.w * kf[j].w;
      }
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float cmax = -FLT_MAX;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const bool valid = p0 + tc + 16 * j <= my_pos;  // causal mask
        s[g][j] = valid ? s[g][j] * inv_sqrt : -FLT_MAX;
        cmax = fmaxf(cmax, s[g][j]);
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) cmax = fmaxf(cmax, __shfl_xor_sync(0xffffffffu, cmax, off));
      const float m_new = fmaxf(m[g], cmax);
      const float resc = m_new == -FLT_MAX ? 1.f : expf(m[g] - m_new);  // a row with nothing seen yet stays 0
      float csum = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float e = s[g][j] == -FLT_MAX ? 0.f : expf(s[g][j] - m_new);
        ps[(g * kAQ + tr) * (kAK + 1) + tc + 16 * j] = e;
        csum += e;
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) csum += __shfl_xor_sync(0xffffffffu, csum, off);
      l[g] = l[g] * resc + csum;
      m[g] = m_new;
#pragma unroll
      for (int i = 0; i < 8; ++i) o[g][i] *= resc;
    }
    __syncwarp();  // a row's probabilities are written and read by the same 16 lanes
    const int np = min(kAK, last + 1 - p0);
    for (int pp = 0; pp < np; ++pp) {
      const float4 v0 = *reinterpret_cast<const float4 *>(vs + pp * kHD + 4 * tc);
      const float4 v1 = *reinterpret_cast<const float4 *>(vs + pp * kHD + 64 + 4 * tc);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float pv = ps[(g * kAQ + tr) * (kAK + 1) + pp];
        o[g][0] += pv * v0.x;
        o[g][1] += pv * v0.y;
        o[g][2] += pv * v0.z;
        o[g][3] += pv * v0.w;
        o[g][4] += pv * v1.x;
        o[g][5] += pv * v1.y;
        o[g][6] += pv * v1.z;
        o[g][7] += pv * v1.w;
      }
    }
  }
  // partial of (tile, KV head, chunk group): m, l [R] and o [R][kHD]
  const int64_t item = (static_cast<int64_t>(blockIdx.x) * a.n_kv + kvh) * gridDim.z + blockIdx.z;
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const int r = g * kAQ + tr;
    if (tc == 0) {
      a.part_m[item * R + r] = m[g];
      a.part_l[item * R + r] = l[g];
    }
    float *po = a.part_o + (item * R + r) * kHD;
    *reinterpret_cast<float4 *>(po + 4 * tc) = make_float4(o[g][0], o[g][1], o[g][2], o[g][3]);
    *reinterpret_cast<float4 *>(po + 64 + 4 * tc) = make_float4(o[g][4], o[g][5], o[g][6], o[g][7]);
  }
}

// Token t = blockIdx.x, KV head blockIdx.y: merge the token's partials of the G query heads over
// the chunk groups holding positions <= pos0 + t (max, then exp(m_z - max) weights), write the
// output (trace) when asked and quantise it into the O GEMM's packed operand.  Warp w takes the
// 32-blocks w, w + 8, ... of the KV head's G * 128 outputs (block 4 g + j is dims 32 j .. of head
// kvh * G + g); the per-head weights are formed once, by warp g, into shared memory.
__global__ void __launch_bounds__(256) pf_attn_combine_kernel(PrefillAttn a, int groups) {
  constexpr int kMaxZ = 16;
  __shared__ float wz[8][kMaxZ];  // [head of the group][chunk group] weight exp(m_z - max) / L
  const int t = blockIdx.x, kvh = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = a.n_head / a.n_kv, R = 16 * G;
  const int pos = a.pos0 + t;
  const int nz = min(groups, (pos / kAK) / a.cpi + 1);  // chunk groups with positions <= pos
  const int64_t item0 = (static_cast<int64_t>(t / kAQ) * a.n_kv + kvh) * groups;
  if (warp < G) {
    const int r = warp * kAQ + t % kAQ;
    const float m = lane < nz ? a.part_m[(item0 + lane) * R + r] : -FLT_MAX;
    const float l = lane < nz ? a.part_l[(item0 + lane) * R + r] : 0.f;
    float mx = m;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const float e = lane < nz ? expf(m - mx) : 0.f;
    float L = e * l;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
    if (lane < kMaxZ) wz[warp][lane] = e / L;
  }
  __syncthreads();
  const int qr = a.n_head * kHD, nb = qr / 32;
  bool bad = false;
  for (int blk = warp; blk < 4 * G; blk += 8) {  // warp-uniform
    const int g = blk / 4, d = (blk % 4) * 32 + lane, h = kvh * G + g;
    const int64_t p0 = (item0 * R + g * kAQ + t % kAQ) * kHD + d;
    float ov[kMaxZ];
#pragma unroll
    for (int z = 0; z < kMaxZ; ++z) ov[z] = z < nz ? a.part_o[p0 + static_cast<int64_t>(z) * R * kHD] : 0.f;
    float v = 0.f;
#pragma unroll
    for (int z = 0; z < kMaxZ; ++z)
      if (z < nz) v += wz[g][z] * ov[z];
    if (a.out) a.out[static_cast<int64_t>(t) * qr + h * kHD + d] = v;
    bad |= pf_quant_block(v, lane, t, 4 * h + blk % 4, nb, a.q_out, a.s_out);
  }
  if (bad && lane == 0) status_or(a.status, ST_NONFINITE_IN);
}

}  // namespace

ugb_status launch_pf_embed(cudaStream_t s, const uint8_t *tok_embd, const int32_t *tokens, int n, int embd, int vocab,
                           float *x, uint32_t *status) {
  pf_embed_kernel<<<n, 256, 0, s>>>(tok_embd, tokens, embd, vocab, x, status);
  return cuda_status(cudaGetLastError());
}

ugb_status launch_pf_rope_kv(cudaStream_t s, const PrefillAttn &a) {
  if (a.kv16)
    pf_rope_kv_kernel<__half><<<a.n, 256, 0, s>>>(a);
  else
    pf_rope_kv_kernel<float><<<a.n, 256, 0, s>>>(a);
  return cuda_status(cudaGetLastError());
}

namespace {

template <int G, typename KV>
ugb_status set_attn_smem(ugb_ctx *ctx) {
  if (ctx->smem_optin < pf_attn_smem(G)) return UGB_EBACKEND;
  return cuda_status(cudaFuncSetAttribute(pf_attn_partial_kernel<G, KV>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          static_cast<int>(pf_attn_smem(G))));
}

template <int G>
ugb_status launch_partial(cudaStream_t s, const PrefillAttn &a, dim3 grid) {
  if (a.kv16)
    pf_attn_partial_kernel<G, __half><<<grid, 256, pf_attn_smem(G), s>>>(a);
  else
    pf_attn_partial_kernel<G, float><<<grid, 256, pf_attn_smem(G), s>>>(a);
  return cuda_status(cudaGetLastError());
}

}  // namespace

ugb_status init_prefill_step_kernels(ugb_ctx *ctx) {
  ugb_status st = UGB_OK;
#define UGB_ATTN_INIT(G)                                             \
  if (st == UGB_OK) st = set_attn_smem<G, float>(ctx);               \
  if (st == UGB_OK) st = set_attn_smem<G, __half>(ctx);
  UGB_ATTN_INIT(1) UGB_ATTN_INIT(2) UGB_ATTN_INIT(3) UGB_ATTN_INIT(4)
  UGB_ATTN_INIT(5) UGB_ATTN_INIT(6) UGB_ATTN_INIT(7) UGB_ATTN_INIT(8)
#undef UGB_ATTN_INIT
  return st;
}

int pf_attn_groups(int pos0, int n, int cpi) {
  const int chunks = (pos0 + n + kAK - 1) / kAK;
  return (chunks + cpi - 1) / cpi;
}

size_t pf_attn_partial_floats(int max_tokens, int n_head, int n_ctx, int max_groups) {
  const size_t tiles = (max_tokens + kAQ - 1) / kAQ;
  const int chunks = (n_ctx + kAK - 1) / kAK;
  const size_t groups = std::min(chunks, max_groups);
  return tiles * groups * 16 * static_cast<size_t>(n_head) * kHD;  // (n_kv x 16 G rows = 16 n_head) x 128
}

ugb_status launch_pf_attention(cudaStream_t s, const PrefillAttn &a) {
  const int G = a.n_head / a.n_kv;
  const int groups = pf_attn_groups(a.pos0, a.n, a.cpi);
  const dim3 grid((a.n + kAQ - 1) / kAQ, a.n_kv, groups);
  ugb_status st;
  switch (G) {
    case 1: st = launch_partial<1>(s, a, grid); break;
    case 2: st = launch_partial<2>(s, a, grid); break;
    case 3: st = launch_partial<3>(s, a, grid); break;
    case 4: st = launch_partial<4>(s, a, grid); break;
    case 5: st = launch_partial<5>(s, a, grid); break;
    case 6: st = launch_partial<6>(s, a, grid); break;
    case 7: st = launch_partial<7>(s, a, grid); break;
    case 8: st = launch_partial<8>(s, a, grid); break;
    default: return UGB_ESHAPE;
  }
  if (st != UGB_OK) return st;
  if (groups > 16) return UGB_ESHAPE;  // the combine weighs at most 16 chunk groups
  pf_attn_combine_kernel<<<dim3(a.n, a.n_kv), 256, 0, s>>>(a, groups);
  return cuda_status(cudaGetLastError());
}

ugb_status launch_pf_norm_quant(cudaStream_t s, float *x, const float *dx, int dx_splits, int64_t dx_stride,
                                const float *w, int n, int embd, float eps, uint8_t *packed, float *pre,
                                uint32_t *status) {
  const PackedLayout p = prefill_layout(n, embd);
  pf_norm_quant_kernel<<<n, 512, 0, s>>>(x, dx, dx_splits, dx_stride, w, embd, eps, packed,
                                         reinterpret_cast<float *>(packed + p.q_bytes), pre, status);
  return cuda_status(cudaGetLastError());
}

ugb_status launch_pf_silu_quant(cudaStream_t s, const float *gu, int64_t ld, int splits, int64_t stride, int n,
                                int n_ff, uint8_t *packed, float *pre, uint32_t *status) {
  const PackedLayout p = prefill_layout(n, n_ff);
  const int64_t warps = static_cast<int64_t>(n) * ((n_ff / 32 + kSiluBlocks - 1) / kSiluBlocks);
  pf_silu_quant_kernel<<<static_cast<unsigned>((warps + 7) / 8), 256, 0, s>>>(
      gu, ld, splits, stride, n, n_ff, packed, reinterpret_cast<float *>(packed + p.q_bytes), pre, status);
  return cuda_status(cudaGetLastError());
}

ugb_status launch_pf_sum_splits(cudaStream_t s, const float *src, int splits, int64_t stride, int64_t row0,
                                int64_t rows, int64_t len, float *dst) {
  const int64_t total = rows * len;
  const unsigned blocks = static_cast<unsigned>(std::min<int64_t>((total + 255) / 256, 4096));
  pf_sum_splits_kernel<<<blocks, 256, 0, s>>>(src, splits, stride, row0, rows, len, dst);
  return cuda_status(cudaGetLastError());
}

}  // namespace ugb
