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
// splits > 1: split K; split s writes its partial sums to y + s * m * ldy (the sum of the splits,
// in split order, is the product).
ugb_status launch_prefill_gemm(ugb_ctx *ctx, cudaStream_t stream, const void *w_packed, const void *x_packed,
                               float *y, int64_t m, int64_t n, int64_t k, int64_t ldy, int splits = 1);
constexpr int kMaxGemmSplits = 4;
// The split count that makes an m x n x k GEMM shortest on this device.
int prefill_gemm_splits(const ugb_ctx *ctx, int64_t m, int64_t n, int64_t k);

// Glue of a prefill over n tokens at positions pos0 .. pos0 + n - 1 (prefill_step.cu).
struct PrefillAttn {
  const float *qkv;     // [n][q ; k ; v] GEMM output (row stride ld)
  int64_t ld;
  const float *bias;    // [q ; k ; v] of the layer, or null
  const float2 *rope;   // [n_ctx][64]
  float *q;             // [n][n_head * 128] rotated queries (out)
  void *kcache, *vcache;  // this layer of sequence 0: [n_kv][n_ctx][128], f32 or f16
  bool kv16;
  int splits;           // qkv holds the GEMM's splits, split_stride floats apart (summed in order)
  int64_t split_stride;
  float *part_m, *part_l, *part_o;  // attention partials (pf_attn_partial_floats floats for part_o)
  int cpi;              // cache chunks (of 64 positions) per partial
  float *out;           // [n][n_head * 128] attention output (the trace), or null
  uint8_t *q_out;       // the output quantised into the O GEMM's packed operand
  float *s_out;         //   (quants, scales) for k = n_head * 128
  uint32_t *status;
  int n, pos0, n_head, n_kv, n_ctx;
};
ugb_status init_prefill_step_kernels(ugb_ctx *ctx);
ugb_status launch_pf_embed(cudaStream_t s, const uint8_t *tok_embd, const int32_t *tokens, int n, int embd, int vocab,
                           float *x, uint32_t *status);
ugb_status launch_pf_rope_kv(cudaStream_t s, const PrefillAttn &a);
// Causal attention of the prompt: partial items over chunk groups, then their combine quantised
// into a.q_out (and a.out when given).
ugb_status launch_pf_attention(cudaStream_t s, const PrefillAttn &a);
int pf_attn_groups(int pos0, int n, int cpi);
size_t pf_attn_partial_floats(int max_tokens, int n_head, int n_ctx, int max_groups);
// The glue fused with the quantisation of its output into a packed operand of n rows (pre: the
// values before quantisation, [n][len], or null).  dx / gu: a split-K GEMM's output, `splits`
// partial sums `stride` floats apart.
ugb_status launch_pf_norm_quant(cudaStream_t s, float *x, const float *dx, int dx_splits, int64_t dx_stride,
                                const float *w, int n, int embd, float eps, uint8_t *packed, float *pre,
                                uint32_t *status);
ugb_status launch_pf_silu_quant(cudaStream_t s, const float *gu, int64_t ld, int splits, int64_t stride, int n,
                                int n_ff, uint8_t *packed, float *pre, uint32_t *status);
// dst = the sum of the splits of rows [row0, row0 + rows) (each len floats) of a split-K output.
ugb_status launch_pf_sum_splits(cudaStream_t s, const float *src, int splits, int64_t stride, int64_t row0,
                                int64_t rows, int64_t len, float *dst);

}  // namespace ugb
