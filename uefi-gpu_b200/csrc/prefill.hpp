// prefill.hpp -- tile geometry shared by the prefill kernels (prefill.cu) and the host code.
#pragma once
#include <cstdint>

#include "internal.hpp"

namespace ugb {

constexpr int kPrefillTile = 128;                     // rows (tokens or weight rows) per tile
constexpr int kPrefillTileBytes = kPrefillTile * 32;  // one tile x one 32-wide K-block of int8

ugb_status init_prefill_kernels(ugb_ctx *ctx);

// Packed operand of `rows` rows of length k: quants [tiles][nb][4096] then scales [tiles][nb][128].
struct PackedLayout {
  int64_t tiles = 0, nb = 0;
  size_t q_bytes = 0, bytes = 0;
};
PackedLayout prefill_layout(int64_t rows, int64_t k);

// Launchers without the entry points' checks (prefill.cu).  repack: n GGUF Q8_0 rows into
// quants q_out / scales s_out of tiles that start there (so matrices can be packed back to back
// as the row ranges of one operand, 128-row aligned).  quant: m fp32 rows of stride ldx.
ugb_status launch_prefill_repack(cudaStream_t stream, const uint8_t *w, int64_t n, int64_t k, uint8_t *q_out,
                                 float *s_out);
ugb_status launch_prefill_quant(ugb_ctx *ctx, cudaStream_t stream, const float *x, int64_t m, int64_t k, int64_t ldx,
                                uint8_t *packed);
ugb_status launch_prefill_gemm(ugb_ctx *ctx, cudaStream_t stream, const void *w_packed, const void *x_packed,
                               float *y, int64_t m, int64_t n, int64_t k, int64_t ldy);

// Glue of a prefill over n tokens at positions pos0 .. pos0 + n - 1 (prefill_step.cu).
struct PrefillAttn {
  const float *qkv;     // [n][q ; k ; v] GEMM output (row stride ld)
  int64_t ld;
  const float *bias;    // [q ; k ; v] of the layer, or null
  const float2 *rope;   // [n_ctx][64]
  float *q;             // [n][n_head * 128] rotated queries (out)
  void *kcache, *vcache;  // this layer of sequence 0: [n_kv][n_ctx][128], f32 or f16
  bool kv16;
  float *out;           // [n][n_head * 128] attention output
  int n, pos0, n_head, n_kv, n_ctx;
};
ugb_status init_prefill_step_kernels(ugb_ctx *ctx);
ugb_status launch_pf_embed(cudaStream_t s, const uint8_t *tok_embd, const int32_t *tokens, int n, int embd, int vocab,
                           float *x, uint32_t *status);
ugb_status launch_pf_rmsnorm(cudaStream_t s, float *x, const float *dx, const float *w, int n, int embd, float eps,
                             float *y, uint32_t *status);
ugb_status launch_pf_rope_kv(cudaStream_t s, const PrefillAttn &a);
ugb_status launch_pf_attention(cudaStream_t s, const PrefillAttn &a);
ugb_status launch_pf_silu(cudaStream_t s, const float *gu, int64_t ld, int n, int n_ff, float *h);

}  // namespace ugb
