// decode.hpp -- shared declarations of the decode-step glue kernels (decode.cu) and the
// decoder host object (decoder.cu).
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "internal.hpp"

namespace ugb {

constexpr int kAttnChunk = 64;  // context positions per flash-decoding chunk
constexpr int kHeadDim = 128;   // head dimension of every configuration served

struct AttnParams {
  const float *qkv;       // [n_head*HD (q) ; n_kv*HD (k) ; n_kv*HD (v)] of this layer
  const float *bias;      // same layout, or null
  const float2 *rope;     // [n_ctx][HD/2] (cos, sin)
  float *kcache;          // this layer: [n_kv][n_ctx][HD] (rotated keys)
  float *vcache;
  float *part_m, *part_l; // [n_kv][n_split][G]
  float *part_o;          // [n_kv][n_split][G][HD]
  const int32_t *state;   // [1] = position
  int n_head, n_kv, n_ctx, n_split;
  uint32_t *status;
};

size_t attn_partial_smem(int group);

ugb_status launch_embed(cudaStream_t s, bool pdl, const uint8_t *tok_embd, int embd, int vocab,
                        int n_ctx, int32_t *state, float *x, uint32_t *status);
ugb_status launch_rmsnorm_quant(cudaStream_t s, bool pdl, float *x, const float *dx, const float *w,
                                int n, float eps, uint8_t *xq, uint32_t *status);
ugb_status launch_silu_quant(cudaStream_t s, bool pdl, const float *gu, int n_ff, uint8_t *hq,
                             uint32_t *status);
ugb_status launch_attention(cudaStream_t s, bool pdl, const AttnParams &a, uint8_t *xq);
ugb_status launch_argmax(cudaStream_t s, bool pdl, const float *logits, int n, int32_t *state,
                         int sm_count);
ugb_status init_decode_kernels(ugb_ctx *ctx);

}  // namespace ugb
