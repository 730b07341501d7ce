// decode.hpp -- shared declarations of the decode-step glue kernels (decode.cu), the MoE
// launchers (moe.cu) and the decoder host object (decoder.cu).
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "internal.hpp"

namespace ugb {

constexpr int kAttnChunk = 64;  // context positions per flash-decoding chunk
constexpr int kHeadDim = 128;   // head dimension of every configuration served
constexpr int kMaxSeq = 8;      // sequences one decoder steps together

// Token state of a decoder in device memory.  A step reads key[b] left by the previous step
// (0 = none): when set, sequence b's token becomes the key's id and the shared position
// advances, so replaying a captured step decodes autoregressively without the host.
struct DecodeState {
  int32_t token[kMaxSeq];
  int32_t pos;
  int32_t pad;
  unsigned long long key[kMaxSeq];  // greedy (value, complemented id) of the last head
};

// Trace of a decode step (ugb_decoder_set_trace): per layer one record of the fields of
// ugb.h's UGB_TRACE_* list, each [batch][len] at its own 256-byte aligned offset; record
// n_layer holds the residual, the output norm and the head's Q8_1 input.  Q8_1 fields use the
// ugb_q8act layout of their length and the decoder's batch.
struct TraceMap {
  uint8_t *base = nullptr;  // null: tracing off
  uint64_t rec = 0;         // bytes per record
  uint64_t off[UGB_TRACE_FIELDS] = {};
  uint64_t bytes[UGB_TRACE_FIELDS] = {};
  // Q8_1 sub-offsets (scales, sums) of the fields of length n_embd, n_head*HD and n_ff
  uint32_t d_e = 0, s_e = 0, d_q = 0, s_q = 0, d_f = 0, s_f = 0;
  __host__ __device__ uint8_t *at(int layer, int field) const {
    return base ? base + rec * static_cast<uint64_t>(layer) + off[field] : nullptr;
  }
  __host__ __device__ float *f32(int layer, int field) const { return reinterpret_cast<float *>(at(layer, field)); }
};

struct AttnParams {
  const float *qkv;       // [batch][n_head*HD (q) ; n_kv*HD (k) ; n_kv*HD (v)] of this layer
  const float *bias;      // [q ; k ; v] rows of this layer, or null
  const float2 *rope;     // [n_ctx][HD/2] (cos, sin)
  void *kcache;           // sequence 0, this layer: [n_kv][n_ctx][HD] (rotated keys), f32 or f16
  void *vcache;
  bool kv16;              // the cache holds fp16 (rounded to nearest even on write)
  int64_t cache_seq;      // elements between sequences' caches
  float *part_m, *part_l; // [batch][n_kv][n_split][G]
  float *part_o;          // [batch][n_kv][n_split][G][HD]
  const DecodeState *state;
  int n_head, n_kv, n_ctx, n_split;
  uint32_t *status;
};

size_t attn_partial_smem(int group, bool kv16);
size_t attn_partial_f32_smem(int group);  // the batch-1 form, the larger of the two

// `pre` (may be null): [batch][n] copy of the values before quantisation, for the trace.
ugb_status launch_embed(cudaStream_t s, bool pdl, const uint8_t *tok_embd, int embd, int vocab, int n_ctx,
                        int batch, DecodeState *state, float *x, uint32_t *status);
ugb_status launch_rmsnorm_quant(cudaStream_t s, bool pdl, float *x, const float *dx, const float *w, int n,
                                int batch, float eps, uint8_t *xq, DecodeState *clear_keys, uint32_t *status,
                                float *pre = nullptr);
ugb_status launch_silu_quant(cudaStream_t s, bool pdl, const float *gu, int n_ff, int batch, uint8_t *hq,
                             uint32_t *status, float *pre = nullptr);
ugb_status launch_attention(cudaStream_t s, bool pdl, const AttnParams &a, int batch, uint8_t *xq,
                            float *pre = nullptr);
ugb_status launch_argmax(cudaStream_t s, bool pdl, const float *logits, int n, int batch, int id0,
                         DecodeState *state, int sm_count);
ugb_status init_decode_kernels(ugb_ctx *ctx);

// The routed expert SwiGLU of one MoE layer (moe.cu), without the entry point's checks.
ugb_status launch_moe_experts(ugb_ctx *ctx, cudaStream_t stream, const ugb_moe_args &m);
ugb_status launch_moe_route(ugb_ctx *ctx, cudaStream_t stream, bool pdl, const float *logits, int n_expert,
                            int top_k, int batch, int32_t *ids, float *weights);

// ---- the persistent token kernel (token.cu) ----------------------------------------------------

constexpr uint32_t kTokItemMax = 64 * 1024;  // bytes of one streamed item (whole rows)

// One layer's tensors as the token kernel reads them (a device-side table, one entry per layer).
struct TokLayer {
  const uint8_t *wq, *wk, *wv, *wo, *wg, *wu, *wd;
  const float *attn_norm, *ffn_norm;
  const float *bias;  // [q; k; v] rows, or null
};

// Everything one launch of the token kernel needs (batch 1, dense FFN, one device).  The
// o_* fields and ring_bytes are the shared-memory layout, filled in by launch_token.
struct TokenStep {
  const TokLayer *layers;
  const uint8_t *tok_embd;    // Q8_0 [n_vocab][n_embd]
  const uint8_t *head;        // head_kind [n_vocab][n_embd]
  const float *out_norm;
  unsigned long long *tqkv;   // [q; k; v] of the current layer as tagged words (read by the
                              // attention units until every tag they need is current)
  unsigned long long *tdx;    // [2][n_embd] O then down projections as (tag << 32 | fp32 bits)
                              // words: the next phase's residual add reads them until every
                              // tag is the current layer's (no device-wide wait of its own)
  float *logits;              // [n_vocab]
  // Q8_1 vectors exchanged between CTAs as tagged words, kQ8TagWords per 32-block: eight of four
  // quants each, then the scale, then the sum (each word: tag << 32 | 32 data bits)
  unsigned long long *thq;    // SiLU(gate) * up, n_ff / 32 blocks
  unsigned long long *tatt;   // the attention output, n_head * HD / 32 blocks
  void *kcache, *vcache;      // [n_layer][n_kv][n_ctx][HD], f32 or (kv16) f16
  const float2 *rope;         // [n_ctx][HD/2]
  float *part_m, *part_l, *part_o;  // attention partials, [n_kv][n_split][G](.[HD])
  DecodeState *state;
  uint32_t *sync;             // token_sync_words() zeroed words: the step's counters
  uint32_t *status;
  int n_layer, n_embd, n_ff, n_head, n_kv, n_ctx, n_vocab, n_split;
  float eps;
  uint32_t rb_e, rb_q, rb_f, rb_h, rb_tok;  // row bytes at K = n_embd, n_head*HD, n_ff; head; embedding
  int gu_blocks;              // FFN blocks a CTA holds at most
  bool kv16;                  // fp16 KV cache
  uint32_t unreachable;       // test hook: extra arrivals the first attention wait needs (0 normally)
  uint64_t wait_ns;           // limit of every wait on other CTAs' progress
  TraceMap trace;             // per-layer trace of the step (tracing off: trace.base null)
  uint32_t o_xres, o_xq, o_xd, o_xs, o_scr, o_layers, o_gu, o_ring, ring_bytes;
};

constexpr int kQ8TagWords = 10;
constexpr size_t token_sync_words() { return 8 * 32 + 64; }  // counters, combine tickets, epoch

// Whether the token kernel serves this decoder on this device (kinds, shapes, row alignment,
// shared memory).
bool token_supported(const ugb_ctx *ctx, uint32_t kind, uint32_t head_kind, TokenStep p);
ugb_status launch_token(ugb_ctx *ctx, cudaStream_t stream, uint32_t kind, uint32_t head_kind, TokenStep p);

}  // namespace ugb
