// decoder.cu -- the decoder object behind ugb_decoder_*: device state, weight binding and
// the per-token launch sequence (captured once as a CUDA graph for ugb_decoder_token[s]).
//
// One token step for `batch` sequences (reference: gpu_graph.rs:139-162, llm.rs:339-388;
// MoE FFN: frontier_forward.rs:164-199):
//   embed -> per layer { rmsnorm+quant -> Q/K/V matvec (one launch over the three tensors)
//   -> attention (bias, RoPE, KV write, flash-decoding, combine + quant) -> O matvec ->
//   residual+rmsnorm+quant -> FFN } -> residual+rmsnorm+quant -> head matvec -> greedy.
//   Dense FFN: gate/up matvec (one launch) -> SiLU*up+quant -> down matvec.
//   MoE FFN: router matvec -> top-k routing -> routed expert gate/up -> SiLU*up+quant ->
//   routed down -> weighted combine [-> all-reduce over the expert-parallel devices].
//   A vocabulary-split head ends with an all-reduce (max) of the greedy keys.
// Every kernel after the first launches with programmatic dependent launch, so each matvec
// streams its first weight stages while the preceding kernel finishes.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <new>
#include <random>
#include <vector>

#include "common.cuh"
#include "decode.hpp"
#include "prefill.hpp"

struct ugb_decoder {
  ugb_ctx *ctx = nullptr;
  ugb_decoder_config cfg{};
  int batch = 1;
  int n_vocab_local = 0;   // head rows held
  int n_expert_local = 0;  // experts held (MoE)
  bool moe = false;
  // device state
  float *x = nullptr, *dx = nullptr, *qkv = nullptr, *gu = nullptr, *logits = nullptr;
  float *rlogits = nullptr, *rweights = nullptr;
  int32_t *rids = nullptr;
  uint8_t *xq = nullptr, *attq = nullptr, *hq = nullptr;
  void *kcache = nullptr, *vcache = nullptr;  // f32 or (kv16) f16
  bool kv16 = false;
  int64_t cache_seq = 0;   // elements of one sequence's cache (all layers)
  float2 *rope = nullptr;
  float *part_m = nullptr, *part_l = nullptr, *part_o = nullptr;
  void *moe_ws = nullptr;
  size_t moe_ws_bytes = 0;
  ugb::DecodeState *state = nullptr;
  ugb::DecodeState *state_host = nullptr;  // pinned mirror
  int n_split = 0;
  // weights
  ugb_model_weights w{};
  std::vector<ugb_layer_weights> layers;
  float *bias = nullptr;   // per layer [q;k;v] fused biases (bound when any bias is given)
  std::vector<void *> owned;
  // persistent token kernel (dense, batch 1): its own buffers and the per-layer tensor table
  unsigned long long *tok_tdx = nullptr;  // token kernel: tagged O / down outputs [2][n_embd]
  unsigned long long *tok_tqkv = nullptr; // token kernel: tagged Q/K/V rows
  unsigned long long *tok_thq = nullptr;  // token kernel: tagged Q8_1 of SiLU(gate) * up
  unsigned long long *tok_tatt = nullptr; // token kernel: tagged Q8_1 of the attention output
  uint32_t *tok_sync = nullptr;
  ugb::TokLayer *tok_layers = nullptr;
  int path = UGB_PATH_AUTO;
  ugb_comm *comm = nullptr;
  ugb::TraceMap trace;     // step trace (ugb_decoder_set_trace); base null: off
  uint64_t wait_ns = ugb::kWaitLimitNs;  // token kernel: limit of each wait on other CTAs
  uint32_t unreachable = 0;              // token kernel test hook (ugb_decoder_test_unreachable_wait)
  // whole-prompt prefill (ugb_decoder_prefill_prepare): packed Q8_0 operands of every layer and
  // the activations of up to pf_max tokens
  int pf_max = 0;
  bool pf_gu_fused = false;  // gate and up packed as one operand (n_ff a multiple of 128)
  uint8_t *pf_w = nullptr;   // all layers' packed weights
  std::vector<size_t> pf_off;  // per layer: qkv, o, gate(/up), up (unfused), down
  uint8_t *pf_ws = nullptr;  // workspace
  float *pf_x = nullptr, *pf_qkv = nullptr, *pf_q = nullptr, *pf_gu = nullptr, *pf_tmp = nullptr;
  float *pf_pm = nullptr, *pf_pl = nullptr, *pf_po = nullptr;  // attention partials
  float *pf_last = nullptr;  // the last token's summed down projection
  int pf_cpi = 1;            // attention chunks per partial
  uint8_t *pf_act = nullptr, *pf_xq = nullptr;
  int32_t *pf_tokens = nullptr;
  ugb::TraceMap ptrace;      // prefill trace, [pf_max] rows per field
  // replay
  cudaStream_t cap = nullptr;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
};

namespace ugb {
namespace {

template <typename T>
ugb_status dalloc(T **p, size_t count) {
  return cuda_status(cudaMalloc(reinterpret_cast<void **>(p), std::max<size_t>(count, 1) * sizeof(T)));
}

bool kind_ok(uint32_t k) { return k == UGB_Q8_0 || k == UGB_Q4_K || k == UGB_Q3_K; }

ugb_status check_config(const ugb_ctx *ctx, const ugb_decoder_config &c) {
  if (c.n_layer < 1 || c.n_embd < 32 || c.n_embd % 32 || c.n_head < 1 || c.n_head_kv < 1 ||
      c.n_head % c.n_head_kv || c.n_head / c.n_head_kv > 8 || c.head_dim != kHeadDim || c.n_vocab < 1 ||
      c.n_ctx < 1 || c.n_ctx > 32768 || !(c.norm_eps > 0.f) || !(c.rope_theta > 0.f) || c.batch < 1 ||
      c.batch > kMaxSeq)
    return UGB_ESHAPE;
  if (!kind_ok(c.kind) || !kind_ok(c.head_kind)) return UGB_EQUANT;
  if (c.kv_type != UGB_F32 && c.kv_type != UGB_F16) return UGB_EQUANT;
  if (ugb_row_bytes(c.kind, c.n_embd) < 0 || ugb_row_bytes(c.kind, static_cast<int64_t>(c.n_head) * c.head_dim) < 0 ||
      ugb_row_bytes(c.head_kind, c.n_embd) < 0)
    return UGB_ESHAPE;
  if (c.n_expert == 0) {
    if (c.n_ff < 32 || c.n_ff % 32 || ugb_row_bytes(c.kind, c.n_ff) < 0) return UGB_ESHAPE;
  } else {
    if (!matvec_kind(c.expert_kind)) return UGB_EQUANT;  // any matvec format for the experts
    const int local = c.n_expert_local ? c.n_expert_local : c.n_expert;
    if (c.n_expert < 1 || c.n_expert > 4096 || c.top_k < 1 || c.top_k > 32 || c.top_k > c.n_expert ||
        c.n_ff_expert < 32 || c.n_ff_expert % 32 || ugb_row_bytes(c.expert_kind, c.n_ff_expert) < 0 ||
        ugb_row_bytes(c.expert_kind, c.n_embd) < 0 || c.expert0 < 0 || local < 1 || c.expert0 + local > c.n_expert)
      return UGB_ESHAPE;
  }
  const int vl = c.n_vocab_local ? c.n_vocab_local : c.n_vocab;
  if (c.vocab0 < 0 || vl < 1 || c.vocab0 + vl > c.n_vocab) return UGB_ESHAPE;
  if (attn_partial_f32_smem(c.n_head / c.n_head_kv) > ctx->smem_optin) return UGB_ESHAPE;
  return UGB_OK;
}

void free_graph(ugb_decoder *d) {
  if (d->exec) cudaGraphExecDestroy(d->exec);
  if (d->graph) cudaGraphDestroy(d->graph);
  d->exec = nullptr;
  d->graph = nullptr;
}

void free_all(ugb_decoder *d) {
  void *bufs[] = {d->x, d->dx, d->qkv, d->gu, d->logits, d->rlogits, d->rweights, d->rids, d->xq, d->attq,
                  d->hq, d->kcache, d->vcache, d->rope, d->part_m, d->part_l, d->part_o, d->moe_ws, d->state,
                  d->bias, d->tok_tdx, d->tok_tqkv, d->tok_thq, d->tok_tatt, d->tok_sync, d->tok_layers, d->trace.base, d->pf_w, d->pf_ws,
                  d->ptrace.base};
  for (void *b : bufs)
    if (b) cudaFree(b);
  for (void *b : d->owned) cudaFree(b);
  if (d->state_host) cudaFreeHost(d->state_host);
  free_graph(d);
  if (d->cap) cudaStreamDestroy(d->cap);
}

// Field sizes and offsets of one trace record of `rows` rows per field (the decode step: the
// batch; a prefill: its token capacity).  The buffer itself is allocated by set_trace.
void plan_trace(const ugb_decoder *d, TraceMap &t, int64_t rows) {
  const ugb_decoder_config &c = d->cfg;
  const int64_t B = rows, E = c.n_embd, Q = static_cast<int64_t>(c.n_head) * c.head_dim;
  const int64_t brow = Q + 2 * static_cast<int64_t>(c.n_head_kv) * c.head_dim;
  const int64_t F = d->moe ? 0 : c.n_ff;
  const Q8Act xe = q8act_layout(E, B), xq = q8act_layout(Q, B);
  uint64_t *n = t.bytes;
  n[UGB_TRACE_X] = n[UGB_TRACE_ATTN_NORM] = n[UGB_TRACE_O] = n[UGB_TRACE_FFN_NORM] = n[UGB_TRACE_DOWN] = B * E * 4;
  n[UGB_TRACE_ATTN_XQ] = n[UGB_TRACE_FFN_XQ] = xe.bytes;
  n[UGB_TRACE_QKV] = B * brow * 4;
  n[UGB_TRACE_ATT] = B * Q * 4;
  n[UGB_TRACE_ATT_XQ] = xq.bytes;
  n[UGB_TRACE_GATE_UP] = B * 2 * F * 4;
  n[UGB_TRACE_H] = B * F * 4;
  n[UGB_TRACE_H_XQ] = F ? q8act_layout(F, B).bytes : 0;
  uint64_t o = 0;
  for (int f = 0; f < UGB_TRACE_FIELDS; ++f) {
    t.off[f] = o;
    o += round_up(n[f], 256);
  }
  t.rec = o;
  t.d_e = static_cast<uint32_t>(xe.d_off);
  t.s_e = static_cast<uint32_t>(xe.s_off);
  t.d_q = static_cast<uint32_t>(xq.d_off);
  t.s_q = static_cast<uint32_t>(xq.s_off);
  if (F) {
    const Q8Act xf = q8act_layout(F, B);
    t.d_f = static_cast<uint32_t>(xf.d_off);
    t.s_f = static_cast<uint32_t>(xf.s_off);
  }
}

}  // namespace
}  // namespace ugb

using namespace ugb;

extern "C" ugb_status ugb_decoder_create(ugb_ctx *ctx, const ugb_decoder_config *cfg, ugb_decoder **out) {
  if (!ctx || !cfg || !out) return UGB_ECONTEXT;
  *out = nullptr;
  ugb_status st = check_config(ctx, *cfg);
  if (st != UGB_OK) return st;
  if (cudaSetDevice(ctx->device) != cudaSuccess) return UGB_EBACKEND;
  ugb_decoder *d = new (std::nothrow) ugb_decoder();
  if (!d) return UGB_EBACKEND;
  d->ctx = ctx;
  d->cfg = *cfg;
  const ugb_decoder_config &c = *cfg;
  const int B = c.batch;
  d->batch = B;
  d->moe = c.n_expert > 0;
  d->n_vocab_local = c.n_vocab_local ? c.n_vocab_local : c.n_vocab;
  d->n_expert_local = d->moe ? (c.n_expert_local ? c.n_expert_local : c.n_expert) : 0;
  const int64_t qrows = static_cast<int64_t>(c.n_head) * c.head_dim;
  const int64_t kvrows = static_cast<int64_t>(c.n_head_kv) * c.head_dim;
  const int group = c.n_head / c.n_head_kv;
  d->n_split = (c.n_ctx + kAttnChunk - 1) / kAttnChunk;
  d->cache_seq = static_cast<int64_t>(c.n_layer) * kvrows * c.n_ctx;
  const size_t kv = static_cast<size_t>(B) * d->cache_seq;
  d->kv16 = c.kv_type == UGB_F16;
  const size_t kv_bytes = kv * (d->kv16 ? sizeof(__half) : sizeof(float));
  const size_t parts = static_cast<size_t>(B) * c.n_head_kv * d->n_split * group;
  bool ok = dalloc(&d->x, static_cast<size_t>(B) * c.n_embd) == UGB_OK &&
            dalloc(&d->dx, static_cast<size_t>(B) * c.n_embd) == UGB_OK &&
            dalloc(&d->qkv, static_cast<size_t>(B) * (qrows + 2 * kvrows)) == UGB_OK &&
            dalloc(&d->logits, static_cast<size_t>(B) * d->n_vocab_local) == UGB_OK &&
            dalloc(&d->xq, q8act_layout(c.n_embd, B).bytes) == UGB_OK &&
            dalloc(&d->attq, q8act_layout(qrows, B).bytes) == UGB_OK &&
            cudaMalloc(&d->kcache, kv_bytes) == cudaSuccess && cudaMalloc(&d->vcache, kv_bytes) == cudaSuccess &&
            dalloc(&d->rope, static_cast<size_t>(c.n_ctx) * (c.head_dim / 2)) == UGB_OK &&
            dalloc(&d->part_m, parts) == UGB_OK && dalloc(&d->part_l, parts) == UGB_OK &&
            dalloc(&d->part_o, parts * c.head_dim) == UGB_OK && dalloc(&d->state, 1) == UGB_OK &&
            cudaMallocHost(reinterpret_cast<void **>(&d->state_host), sizeof(DecodeState)) == cudaSuccess &&
            cudaStreamCreateWithFlags(&d->cap, cudaStreamNonBlocking) == cudaSuccess;
  if (ok && d->moe) {
    d->moe_ws_bytes = ugb_moe_workspace_bytes(c.n_embd, c.n_ff_expert, c.top_k, B);
    ok = dalloc(&d->rlogits, static_cast<size_t>(B) * c.n_expert) == UGB_OK &&
         dalloc(&d->rweights, static_cast<size_t>(B) * c.top_k) == UGB_OK &&
         dalloc(&d->rids, static_cast<size_t>(B) * c.top_k) == UGB_OK &&
         cudaMalloc(&d->moe_ws, d->moe_ws_bytes) == cudaSuccess;
  } else if (ok) {
    ok = dalloc(&d->gu, static_cast<size_t>(B) * 2 * c.n_ff) == UGB_OK &&
         dalloc(&d->hq, q8act_layout(c.n_ff, B).bytes) == UGB_OK;
    if (ok && B == 1)
      ok = dalloc(&d->tok_tdx, 2 * static_cast<size_t>(c.n_embd)) == UGB_OK &&
           cudaMemset(d->tok_tdx, 0, 2 * sizeof(unsigned long long) * c.n_embd) == cudaSuccess &&
           dalloc(&d->tok_tqkv, static_cast<size_t>(c.head_dim) * (c.n_head + 2 * c.n_head_kv)) == UGB_OK &&
           cudaMemset(d->tok_tqkv, 0, sizeof(unsigned long long) * c.head_dim * (c.n_head + 2 * c.n_head_kv)) ==
               cudaSuccess &&
           dalloc(&d->tok_thq, kQ8TagWords * static_cast<size_t>(c.n_ff / 32)) == UGB_OK &&
           cudaMemset(d->tok_thq, 0, 8 * kQ8TagWords * static_cast<size_t>(c.n_ff / 32)) == cudaSuccess &&
           dalloc(&d->tok_tatt, kQ8TagWords * static_cast<size_t>(c.n_head * c.head_dim / 32)) == UGB_OK &&
           cudaMemset(d->tok_tatt, 0, 8 * kQ8TagWords * static_cast<size_t>(c.n_head * c.head_dim / 32)) ==
               cudaSuccess &&
           dalloc(&d->tok_sync, token_sync_words()) == UGB_OK &&
           dalloc(&d->tok_layers, c.n_layer) == UGB_OK &&
           cudaMemset(d->tok_sync, 0, token_sync_words() * sizeof(uint32_t)) == cudaSuccess;
  }
  if (ok) {
    // RoPE table as the reference builds it (gpu_graph.rs:132, llm.rs:330): the angle is the
    // f32 product pos * powf(theta, -(2i)/head_dim); cos and sin of that f32 angle are taken in
    // double and rounded once.
    std::vector<float2> tab(static_cast<size_t>(c.n_ctx) * (c.head_dim / 2));
    for (int p = 0; p < c.n_ctx; ++p)
      for (int i = 0; i < c.head_dim / 2; ++i) {
        const float e = -static_cast<float>(2 * i) / static_cast<float>(c.head_dim);
        const float ang = static_cast<float>(p) * powf(c.rope_theta, e);
        tab[static_cast<size_t>(p) * (c.head_dim / 2) + i] =
            make_float2(static_cast<float>(std::cos(static_cast<double>(ang))),
                        static_cast<float>(std::sin(static_cast<double>(ang))));
      }
    ok = cudaMemcpy(d->rope, tab.data(), tab.size() * sizeof(float2), cudaMemcpyHostToDevice) == cudaSuccess &&
         cudaMemset(d->state, 0, sizeof(DecodeState)) == cudaSuccess &&
         cudaMemset(d->kcache, 0, kv_bytes) == cudaSuccess && cudaMemset(d->vcache, 0, kv_bytes) == cudaSuccess &&
         cudaMemset(d->dx, 0, static_cast<size_t>(B) * c.n_embd * sizeof(float)) == cudaSuccess;
  }
  if (!ok) {
    free_all(d);
    delete d;
    return UGB_EBACKEND;
  }
  plan_trace(d, d->trace, B);
  *out = d;
  return UGB_OK;
}

extern "C" ugb_status ugb_decoder_destroy(ugb_decoder *dec) {
  if (!dec) return UGB_ECONTEXT;
  cudaSetDevice(dec->ctx->device);
  cudaDeviceSynchronize();
  free_all(dec);
  delete dec;
  return UGB_OK;
}

extern "C" ugb_status ugb_decoder_set_comm(ugb_decoder *d, ugb_comm *comm) {
  if (!d) return UGB_ECONTEXT;
  d->comm = comm;
  free_graph(d);  // the captured step may or may not contain the collectives
  return UGB_OK;
}

namespace ugb {
namespace {

bool matrix_ok(uint32_t kind, const void *p) {
  return p && (reinterpret_cast<uintptr_t>(p) & 15) == 0 && kind != 0;
}

ugb_status copy_bias(float *dst, const void *src, int64_t n) {
  if (!src) return UGB_OK;
  return cuda_status(cudaMemcpy(dst, src, n * sizeof(float), cudaMemcpyDeviceToDevice));
}

// Host-generated f32 vector: center + amp * u, u uniform in [-1, 1).
ugb_status upload_vec(float **dst, int64_t n, float center, float amp, std::mt19937_64 &rng,
                      std::vector<void *> &owned) {
  std::vector<float> h(static_cast<size_t>(n));
  std::uniform_real_distribution<float> u(-1.f, 1.f);
  for (auto &v : h) v = center + amp * u(rng);
  if (cudaMalloc(reinterpret_cast<void **>(dst), n * sizeof(float)) != cudaSuccess) return UGB_EBACKEND;
  owned.push_back(*dst);
  return cuda_status(cudaMemcpy(*dst, h.data(), n * sizeof(float), cudaMemcpyHostToDevice));
}

// `count` matrices of m x k stacked back to back; matrix i filled from seed0 + i.
ugb_status synth_stack(ugb_ctx *ctx, const void **dst, uint32_t kind, int64_t k, int64_t m, int64_t count,
                       uint64_t seed0, std::vector<void *> &owned) {
  const int64_t rb = ugb_row_bytes(kind, k);
  void *p = nullptr;
  if (rb < 0 || cudaMalloc(&p, static_cast<size_t>(rb * m * count)) != cudaSuccess) return UGB_EBACKEND;
  owned.push_back(p);
  *dst = p;
  for (int64_t i = 0; i < count; ++i) {
    const ugb_status st = launch_fill_synthetic(ctx, nullptr, kind, static_cast<uint8_t *>(p) + i * rb * m, k, m,
                                                seed0 + static_cast<uint64_t>(i));
    if (st != UGB_OK) return st;
  }
  return UGB_OK;
}

}  // namespace
}  // namespace ugb

extern "C" ugb_status ugb_decoder_bind(ugb_decoder *d, const ugb_model_weights *w) {
  if (!d || !w || !w->layers) return UGB_ECONTEXT;
  const ugb_decoder_config &c = d->cfg;
  if (!matrix_ok(UGB_Q8_0, w->tok_embd) || !matrix_ok(c.head_kind, w->output) || !w->output_norm)
    return UGB_EALIGN;
  const int64_t qrows = static_cast<int64_t>(c.n_head) * c.head_dim;
  const int64_t kvrows = static_cast<int64_t>(c.n_head_kv) * c.head_dim;
  const int64_t brow = qrows + 2 * kvrows;
  bool any_bias = false;
  for (int l = 0; l < c.n_layer; ++l) {
    const ugb_layer_weights &L = w->layers[l];
    for (const void *m : {L.wq, L.wk, L.wv, L.wo})
      if (!matrix_ok(c.kind, m)) return UGB_EALIGN;
    if (d->moe) {
      if (!matrix_ok(c.kind, L.router)) return UGB_EALIGN;
      for (const void *m : {L.gate_exps, L.up_exps, L.down_exps})
        if (!matrix_ok(c.expert_kind, m)) return UGB_EALIGN;
    } else {
      for (const void *m : {L.w_gate, L.w_up, L.w_down})
        if (!matrix_ok(c.kind, m)) return UGB_EALIGN;
    }
    if (!L.attn_norm || !L.ffn_norm) return UGB_EALIGN;
    any_bias = any_bias || L.bq || L.bk || L.bv;
  }
  cudaSetDevice(d->ctx->device);
  if (d->bias) {
    cudaFree(d->bias);
    d->bias = nullptr;
  }
  if (any_bias) {
    if (dalloc(&d->bias, static_cast<size_t>(c.n_layer) * brow) != UGB_OK) return UGB_EBACKEND;
    if (cudaMemset(d->bias, 0, static_cast<size_t>(c.n_layer) * brow * sizeof(float)) != cudaSuccess) return UGB_EBACKEND;
    for (int l = 0; l < c.n_layer; ++l) {
      const ugb_layer_weights &L = w->layers[l];
      float *b = d->bias + static_cast<size_t>(l) * brow;
      if (copy_bias(b, L.bq, qrows) != UGB_OK || copy_bias(b + qrows, L.bk, kvrows) != UGB_OK ||
          copy_bias(b + qrows + kvrows, L.bv, kvrows) != UGB_OK)
        return UGB_EBACKEND;
    }
  }
  if (d->pf_w) {  // the packed prefill weights are of the old tensors: prepare again
    cudaDeviceSynchronize();
    cudaFree(d->pf_w);
    d->pf_w = nullptr;
  }
  d->w = *w;
  d->layers.assign(w->layers, w->layers + c.n_layer);
  d->w.layers = d->layers.data();
  free_graph(d);  // the captured step refers to the old weights
  if (d->tok_layers) {
    std::vector<TokLayer> tab(c.n_layer);
    for (int l = 0; l < c.n_layer; ++l) {
      const ugb_layer_weights &L = d->layers[l];
      tab[l] = TokLayer{static_cast<const uint8_t *>(L.wq),     static_cast<const uint8_t *>(L.wk),
                        static_cast<const uint8_t *>(L.wv),     static_cast<const uint8_t *>(L.wo),
                        static_cast<const uint8_t *>(L.w_gate), static_cast<const uint8_t *>(L.w_up),
                        static_cast<const uint8_t *>(L.w_down), static_cast<const float *>(L.attn_norm),
                        static_cast<const float *>(L.ffn_norm),
                        d->bias ? d->bias + static_cast<size_t>(l) * brow : nullptr};
    }
    if (cudaMemcpy(d->tok_layers, tab.data(), tab.size() * sizeof(TokLayer), cudaMemcpyHostToDevice) != cudaSuccess)
      return UGB_EBACKEND;
  }
  return UGB_OK;
}

extern "C" ugb_status ugb_decoder_synthetic(ugb_decoder *d, uint64_t seed) {
  if (!d) return UGB_ECONTEXT;
  const ugb_decoder_config &c = d->cfg;
  cudaSetDevice(d->ctx->device);
  const int64_t qrows = static_cast<int64_t>(c.n_head) * c.head_dim;
  const int64_t kvrows = static_cast<int64_t>(c.n_head_kv) * c.head_dim;
  std::vector<ugb_layer_weights> layers(c.n_layer);
  ugb_model_weights w{};
  // every tensor's seed depends on (seed, layer, tensor[, expert]) only, so the shards of an
  // expert-parallel or vocabulary-split model agree on the tensors they share
  const uint64_t base = seed * 1000003ull;
  auto tseed = [&](int layer, int slot) { return base + 64ull * (layer + 1) + slot; };
  ugb_status st = synth_stack(d->ctx, &w.tok_embd, UGB_Q8_0, c.n_embd, c.n_vocab, 1, base, d->owned);
  std::mt19937_64 rng0(seed);
  float *onorm = nullptr;
  if (st == UGB_OK) st = upload_vec(&onorm, c.n_embd, 1.f, 0.1f, rng0, d->owned);
  w.output_norm = onorm;
  if (st == UGB_OK) {
    if (c.head_kind == UGB_Q8_0) {  // tied embeddings: the held rows of token_embd
      w.output = static_cast<const uint8_t *>(w.tok_embd) + static_cast<int64_t>(c.vocab0) * ugb_row_bytes(UGB_Q8_0, c.n_embd);
    } else {
      st = synth_stack(d->ctx, &w.output, c.head_kind, c.n_embd, d->n_vocab_local, 1,
                       base + 7 + static_cast<uint64_t>(c.vocab0), d->owned);
    }
  }
  for (int l = 0; l < c.n_layer && st == UGB_OK; ++l) {
    ugb_layer_weights &L = layers[l];
    std::mt19937_64 rng(seed * 7919ull + l);
    float *an = nullptr, *fn = nullptr;
    st = upload_vec(&an, c.n_embd, 1.f, 0.1f, rng, d->owned);
    if (st == UGB_OK) st = upload_vec(&fn, c.n_embd, 1.f, 0.1f, rng, d->owned);
    L.attn_norm = an;
    L.ffn_norm = fn;
    if (!d->moe) {  // the dense (Qwen2) shapes carry Q/K/V biases
      float *bq = nullptr, *bk = nullptr, *bv = nullptr;
      if (st == UGB_OK) st = upload_vec(&bq, qrows, 0.f, 0.02f, rng, d->owned);
      if (st == UGB_OK) st = upload_vec(&bk, kvrows, 0.f, 0.02f, rng, d->owned);
      if (st == UGB_OK) st = upload_vec(&bv, kvrows, 0.f, 0.02f, rng, d->owned);
      L.bq = bq;
      L.bk = bk;
      L.bv = bv;
    }
    if (st == UGB_OK) st = synth_stack(d->ctx, &L.wq, c.kind, c.n_embd, qrows, 1, tseed(l, 0), d->owned);
    if (st == UGB_OK) st = synth_stack(d->ctx, &L.wk, c.kind, c.n_embd, kvrows, 1, tseed(l, 1), d->owned);
    if (st == UGB_OK) st = synth_stack(d->ctx, &L.wv, c.kind, c.n_embd, kvrows, 1, tseed(l, 2), d->owned);
    if (st == UGB_OK) st = synth_stack(d->ctx, &L.wo, c.kind, qrows, c.n_embd, 1, tseed(l, 3), d->owned);
    if (d->moe) {
      const uint64_t eb = base + (1ull << 32) + static_cast<uint64_t>(l) * 3 * c.n_expert;
      if (st == UGB_OK) st = synth_stack(d->ctx, &L.router, c.kind, c.n_embd, c.n_expert, 1, tseed(l, 4), d->owned);
      if (st == UGB_OK)
        st = synth_stack(d->ctx, &L.gate_exps, c.expert_kind, c.n_embd, c.n_ff_expert, d->n_expert_local,
                         eb + c.expert0, d->owned);
      if (st == UGB_OK)
        st = synth_stack(d->ctx, &L.up_exps, c.expert_kind, c.n_embd, c.n_ff_expert, d->n_expert_local,
                         eb + c.n_expert + c.expert0, d->owned);
      if (st == UGB_OK)
        st = synth_stack(d->ctx, &L.down_exps, c.expert_kind, c.n_ff_expert, c.n_embd, d->n_expert_local,
                         eb + 2 * c.n_expert + c.expert0, d->owned);
    } else {
      if (st == UGB_OK) st = synth_stack(d->ctx, &L.w_gate, c.kind, c.n_embd, c.n_ff, 1, tseed(l, 5), d->owned);
      if (st == UGB_OK) st = synth_stack(d->ctx, &L.w_up, c.kind, c.n_embd, c.n_ff, 1, tseed(l, 6), d->owned);
      if (st == UGB_OK) st = synth_stack(d->ctx, &L.w_down, c.kind, c.n_ff, c.n_embd, 1, tseed(l, 7), d->owned);
    }
  }
  if (st != UGB_OK) return st;
  if (cudaDeviceSynchronize() != cudaSuccess) return UGB_EBACKEND;
  w.layers = layers.data();
  return ugb_decoder_bind(d, &w);
}

namespace ugb {
namespace {

MatvecArgs mv_args(uint32_t kind, int64_t k, int64_t m, int batch, const uint8_t *xq, float *y) {
  MatvecArgs a;
  a.kind = kind;
  a.row_bytes = ugb_row_bytes(kind, k);
  a.k = k;
  a.m = m;
  a.xq = xq;
  a.xl = q8act_layout(k, batch);
  a.y = y;
  a.ldy = m;
  a.batch = batch;
  a.pdl = true;
  return a;
}

}  // namespace
}  // namespace ugb

namespace ugb {
namespace {

// The token kernel's launch description for this decoder; false when the decoder is not one it
// serves (MoE, batch > 1, a sharded head, kinds, shapes, alignment, shared memory).
bool token_step_of(const ugb_decoder *d, TokenStep &p) {
  const ugb_decoder_config &c = d->cfg;
  if (d->moe || d->batch != 1 || !d->tok_layers || !d->w.layers || d->n_vocab_local != c.n_vocab) return false;
  const int64_t qrows = static_cast<int64_t>(c.n_head) * c.head_dim;
  p = TokenStep{};
  p.layers = d->tok_layers;
  p.tok_embd = static_cast<const uint8_t *>(d->w.tok_embd);
  p.head = static_cast<const uint8_t *>(d->w.output);
  p.out_norm = static_cast<const float *>(d->w.output_norm);
  p.tqkv = d->tok_tqkv;
  p.tdx = d->tok_tdx;
  p.logits = d->logits;
  p.thq = d->tok_thq;
  p.tatt = d->tok_tatt;
  p.kcache = d->kcache;
  p.vcache = d->vcache;
  p.kv16 = d->kv16;
  p.trace = d->trace;
  p.wait_ns = d->wait_ns;
  p.unreachable = d->unreachable;
  p.rope = d->rope;
  p.part_m = d->part_m;
  p.part_l = d->part_l;
  p.part_o = d->part_o;
  p.state = d->state;
  p.sync = d->tok_sync;
  p.status = d->ctx->status;
  p.n_layer = c.n_layer;
  p.n_embd = c.n_embd;
  p.n_ff = c.n_ff;
  p.n_head = c.n_head;
  p.n_kv = c.n_head_kv;
  p.n_ctx = c.n_ctx;
  p.n_vocab = c.n_vocab;
  p.n_split = d->n_split;
  p.eps = c.norm_eps;
  p.rb_e = static_cast<uint32_t>(ugb_row_bytes(c.kind, c.n_embd));
  p.rb_q = static_cast<uint32_t>(ugb_row_bytes(c.kind, qrows));
  p.rb_f = static_cast<uint32_t>(ugb_row_bytes(c.kind, c.n_ff));
  p.rb_h = static_cast<uint32_t>(ugb_row_bytes(c.head_kind, c.n_embd));
  p.rb_tok = static_cast<uint32_t>(ugb_row_bytes(UGB_Q8_0, c.n_embd));
  for (int l = 0; l < c.n_layer; ++l) {
    const ugb_layer_weights &L = d->layers[l];
    for (const void *m : {L.wq, L.wk, L.wv, L.wo, L.w_gate, L.w_up, L.w_down})
      if (reinterpret_cast<uintptr_t>(m) & 15) return false;
  }
  if (reinterpret_cast<uintptr_t>(p.head) & 15) return false;
  return token_supported(d->ctx, c.kind, c.head_kind, p);
}

bool use_token(const ugb_decoder *d, TokenStep &p) {
  if (d->path == UGB_PATH_CHAIN || (d->comm && comm_world(d->comm) > 1)) return false;
  return token_step_of(d, p);
}

}  // namespace
}  // namespace ugb

extern "C" ugb_status ugb_decoder_set_path(ugb_decoder *d, int32_t path, int32_t *active) {
  if (!d) return UGB_ECONTEXT;
  if (path != UGB_PATH_AUTO && path != UGB_PATH_CHAIN && path != UGB_PATH_TOKEN) return UGB_ESHAPE;
  TokenStep p;
  const bool can = token_step_of(d, p) && !(d->comm && comm_world(d->comm) > 1);
  if (path == UGB_PATH_TOKEN && !can) return UGB_ESHAPE;
  if (d->path != path) free_graph(d);
  d->path = path;
  if (active) *active = (path != UGB_PATH_CHAIN && can) ? UGB_PATH_TOKEN : UGB_PATH_CHAIN;
  return UGB_OK;
}

extern "C" ugb_status ugb_decoder_step(ugb_decoder *d, ugb_stream stream) {
  if (!d || !d->w.layers) return UGB_ECONTEXT;
  {
    TokenStep tp;
    if (use_token(d, tp)) {
      cudaSetDevice(d->ctx->device);
      return launch_token(d->ctx, stream, d->cfg.kind, d->cfg.head_kind, tp);
    }
  }
  const ugb_decoder_config &c = d->cfg;
  ugb_ctx *ctx = d->ctx;
  uint32_t *status = ctx->status;
  const int B = d->batch;
  const int64_t qrows = static_cast<int64_t>(c.n_head) * c.head_dim;
  const int64_t kvrows = static_cast<int64_t>(c.n_head_kv) * c.head_dim;
  const int64_t brow = qrows + 2 * kvrows;
  const size_t kv_layer = static_cast<size_t>(kvrows) * c.n_ctx * (d->kv16 ? sizeof(__half) : sizeof(float));
  const TraceMap &T = d->trace;
  // Tracing: copy a device buffer into field f of record l after the kernel that wrote it.
  auto tcopy = [&](int l, int f, const void *src) {
    return T.base ? cuda_status(cudaMemcpyAsync(T.at(l, f), src, T.bytes[f], cudaMemcpyDeviceToDevice, stream))
                  : UGB_OK;
  };
  const bool ep_reduce = d->moe && d->comm && d->n_expert_local < c.n_expert;
  const bool vocab_reduce = d->comm && d->n_vocab_local < c.n_vocab;
  ugb_status st = launch_embed(stream, false, static_cast<const uint8_t *>(d->w.tok_embd), c.n_embd, c.n_vocab,
                               c.n_ctx, B, d->state, d->x, status);
  for (int l = 0; l < c.n_layer && st == UGB_OK; ++l) {
    const ugb_layer_weights &L = d->layers[l];
    st = launch_rmsnorm_quant(stream, true, d->x, l == 0 ? nullptr : d->dx, static_cast<const float *>(L.attn_norm),
                              c.n_embd, B, c.norm_eps, d->xq, l == 0 ? d->state : nullptr, status,
                              T.f32(l, UGB_TRACE_ATTN_NORM));
    if (st == UGB_OK) st = tcopy(l, UGB_TRACE_X, d->x);
    if (st == UGB_OK) st = tcopy(l, UGB_TRACE_ATTN_XQ, d->xq);
    if (st != UGB_OK) break;
    MatvecArgs a = mv_args(c.kind, c.n_embd, brow, B, d->xq, d->qkv);
    a.nseg = 3;
    a.ws[0] = static_cast<const uint8_t *>(L.wq);
    a.ws[1] = static_cast<const uint8_t *>(L.wk);
    a.ws[2] = static_cast<const uint8_t *>(L.wv);
    a.seg_rows[0] = qrows;
    a.seg_rows[1] = a.seg_rows[2] = kvrows;
    st = launch_matvec(ctx, stream, a);
    if (st == UGB_OK) st = tcopy(l, UGB_TRACE_QKV, d->qkv);
    if (st != UGB_OK) break;
    AttnParams ap{};
    ap.qkv = d->qkv;
    ap.bias = d->bias ? d->bias + static_cast<size_t>(l) * brow : nullptr;
    ap.rope = d->rope;
    ap.kcache = static_cast<uint8_t *>(d->kcache) + kv_layer * l;
    ap.vcache = static_cast<uint8_t *>(d->vcache) + kv_layer * l;
    ap.kv16 = d->kv16;
    ap.cache_seq = d->cache_seq;
    ap.part_m = d->part_m;
    ap.part_l = d->part_l;
    ap.part_o = d->part_o;
    ap.state = d->state;
    ap.n_head = c.n_head;
    ap.n_kv = c.n_head_kv;
    ap.n_ctx = c.n_ctx;
    ap.n_split = d->n_split;
    ap.status = status;
    st = launch_attention(stream, true, ap, B, d->attq, T.f32(l, UGB_TRACE_ATT));
    if (st == UGB_OK) st = tcopy(l, UGB_TRACE_ATT_XQ, d->attq);
    if (st != UGB_OK) break;
    a = mv_args(c.kind, qrows, c.n_embd, B, d->attq, d->dx);
    a.w = static_cast<const uint8_t *>(L.wo);
    st = launch_matvec(ctx, stream, a);
    if (st == UGB_OK) st = tcopy(l, UGB_TRACE_O, d->dx);
    if (st != UGB_OK) break;
    st = launch_rmsnorm_quant(stream, true, d->x, d->dx, static_cast<const float *>(L.ffn_norm), c.n_embd, B,
                              c.norm_eps, d->xq, nullptr, status, T.f32(l, UGB_TRACE_FFN_NORM));
    if (st == UGB_OK) st = tcopy(l, UGB_TRACE_FFN_XQ, d->xq);
    if (st != UGB_OK) break;
    if (d->moe) {
      a = mv_args(c.kind, c.n_embd, c.n_expert, B, d->xq, d->rlogits);
      a.w = static_cast<const uint8_t *>(L.router);
      st = launch_matvec(ctx, stream, a);
      if (st == UGB_OK)
        st = launch_moe_route(ctx, stream, true, d->rlogits, c.n_expert, c.top_k, B, d->rids, d->rweights);
      if (st != UGB_OK) break;
      ugb_moe_args m{};
      m.kind = c.expert_kind;
      m.accumulate = 0;
      m.hidden = c.n_embd;
      m.ffn = c.n_ff_expert;
      m.top_k = c.top_k;
      m.batch = B;
      m.n_expert = d->n_expert_local;
      m.expert0 = c.expert0;
      m.n_expert_total = c.n_expert;
      m.gate = L.gate_exps;
      m.up = L.up_exps;
      m.down = L.down_exps;
      m.xq = d->xq;
      m.ids = d->rids;
      m.weights = d->rweights;
      m.out = d->dx;
      m.workspace = d->moe_ws;
      m.workspace_bytes = d->moe_ws_bytes;
      st = launch_moe_experts(ctx, stream, m);
      if (st == UGB_OK && ep_reduce)
        st = comm_allreduce_sum_f32(d->comm, d->dx, static_cast<size_t>(B) * c.n_embd, stream);
      if (st == UGB_OK) st = tcopy(l, UGB_TRACE_DOWN, d->dx);
    } else {
      a = mv_args(c.kind, c.n_embd, 2 * static_cast<int64_t>(c.n_ff), B, d->xq, d->gu);
      a.nseg = 2;
      a.ws[0] = static_cast<const uint8_t *>(L.w_gate);
      a.ws[1] = static_cast<const uint8_t *>(L.w_up);
      a.seg_rows[0] = a.seg_rows[1] = c.n_ff;
      st = launch_matvec(ctx, stream, a);
      if (st == UGB_OK) st = tcopy(l, UGB_TRACE_GATE_UP, d->gu);
      if (st != UGB_OK) break;
      st = launch_silu_quant(stream, true, d->gu, c.n_ff, B, d->hq, status, T.f32(l, UGB_TRACE_H));
      if (st == UGB_OK) st = tcopy(l, UGB_TRACE_H_XQ, d->hq);
      if (st != UGB_OK) break;
      a = mv_args(c.kind, c.n_ff, c.n_embd, B, d->hq, d->dx);
      a.w = static_cast<const uint8_t *>(L.w_down);
      st = launch_matvec(ctx, stream, a);
      if (st == UGB_OK) st = tcopy(l, UGB_TRACE_DOWN, d->dx);
    }
  }
  if (st != UGB_OK) return st;
  st = launch_rmsnorm_quant(stream, true, d->x, d->dx, static_cast<const float *>(d->w.output_norm), c.n_embd, B,
                            c.norm_eps, d->xq, nullptr, status, T.f32(c.n_layer, UGB_TRACE_ATTN_NORM));
  if (st == UGB_OK) st = tcopy(c.n_layer, UGB_TRACE_X, d->x);
  if (st == UGB_OK) st = tcopy(c.n_layer, UGB_TRACE_ATTN_XQ, d->xq);
  if (st != UGB_OK) return st;
  MatvecArgs a = mv_args(c.head_kind, c.n_embd, d->n_vocab_local, B, d->xq, d->logits);
  a.w = static_cast<const uint8_t *>(d->w.output);
  st = launch_matvec(ctx, stream, a);
  if (st != UGB_OK) return st;
  st = launch_argmax(stream, true, d->logits, d->n_vocab_local, B, c.vocab0, d->state, ctx->sm_count);
  if (st == UGB_OK && vocab_reduce) st = comm_allreduce_max_u64(d->comm, d->state->key, B, stream);
  return st;
}

extern "C" ugb_status ugb_decoder_set_tokens(ugb_decoder *d, ugb_stream stream, const int32_t *tokens, int32_t pos) {
  if (!d || !tokens) return UGB_ECONTEXT;
  if (pos < 0 || pos >= d->cfg.n_ctx) return UGB_ESHAPE;
  for (int b = 0; b < d->batch; ++b)
    if (tokens[b] < 0 || tokens[b] >= d->cfg.n_vocab) return UGB_ESHAPE;
  cudaSetDevice(d->ctx->device);
  // Wait for any earlier copy out of the pinned mirror before overwriting it.
  if (cudaStreamSynchronize(stream) != cudaSuccess) return UGB_EBACKEND;
  std::memset(d->state_host, 0, sizeof(DecodeState));
  for (int b = 0; b < d->batch; ++b) d->state_host->token[b] = tokens[b];
  d->state_host->pos = pos;
  return cuda_status(cudaMemcpyAsync(d->state, d->state_host, sizeof(DecodeState), cudaMemcpyHostToDevice, stream));
}

extern "C" ugb_status ugb_decoder_set_state(ugb_decoder *d, ugb_stream stream, int32_t token, int32_t pos) {
  if (!d) return UGB_ECONTEXT;
  int32_t t[kMaxSeq];
  for (int b = 0; b < kMaxSeq; ++b) t[b] = token;
  return ugb_decoder_set_tokens(d, stream, t, pos);
}

namespace {

ugb_status fetch_state(ugb_decoder *d, cudaStream_t stream) {
  cudaSetDevice(d->ctx->device);
  if (cudaMemcpyAsync(d->state_host, d->state, sizeof(DecodeState), cudaMemcpyDeviceToHost, stream) != cudaSuccess ||
      cudaStreamSynchronize(stream) != cudaSuccess)
    return UGB_EBACKEND;
  return UGB_OK;
}

int32_t next_of(const DecodeState *s, int b) {
  return s->key[b] ? static_cast<int32_t>(~static_cast<uint32_t>(s->key[b])) : -1;
}

}  // namespace

extern "C" ugb_status ugb_decoder_get_tokens(ugb_decoder *d, ugb_stream stream, int32_t *tokens, int32_t *pos,
                                             int32_t *next_tokens) {
  if (!d) return UGB_ECONTEXT;
  const ugb_status st = fetch_state(d, stream);
  if (st != UGB_OK) return st;
  for (int b = 0; b < d->batch; ++b) {
    if (tokens) tokens[b] = d->state_host->token[b];
    if (next_tokens) next_tokens[b] = next_of(d->state_host, b);
  }
  if (pos) *pos = d->state_host->pos;
  return UGB_OK;
}

extern "C" ugb_status ugb_decoder_get_state(ugb_decoder *d, ugb_stream stream, int32_t *token, int32_t *pos,
                                            int32_t *next_token) {
  if (!d) return UGB_ECONTEXT;
  const ugb_status st = fetch_state(d, stream);
  if (st != UGB_OK) return st;
  if (token) *token = d->state_host->token[0];
  if (pos) *pos = d->state_host->pos;
  if (next_token) *next_token = next_of(d->state_host, 0);
  return UGB_OK;
}

extern "C" ugb_status ugb_decoder_logits(ugb_decoder *d, ugb_stream stream, float *logits_host) {
  if (!d || !logits_host) return UGB_ECONTEXT;
  cudaSetDevice(d->ctx->device);
  if (cudaMemcpyAsync(logits_host, d->logits, static_cast<size_t>(d->batch) * d->n_vocab_local * sizeof(float),
                      cudaMemcpyDeviceToHost, stream) != cudaSuccess)
    return UGB_EBACKEND;
  return cuda_status(cudaStreamSynchronize(stream));
}

namespace {

// Copy `count` cached positions from `pos` of one sequence and layer between the cache and host
// rows [n_kv][count][head_dim] of fp32 (converted to or from fp16 for an fp16 cache).
ugb_status kv_copy(ugb_decoder *d, cudaStream_t stream, int32_t seq, int32_t layer, int32_t pos, int32_t count,
                   float *k_out, float *v_out, const float *k_in, const float *v_in) {
  const ugb_decoder_config &c = d->cfg;
  if (seq < 0 || seq >= d->batch || layer < 0 || layer >= c.n_layer || pos < 0 || count < 1 || count > c.n_ctx - pos)
    return UGB_ESHAPE;
  cudaSetDevice(d->ctx->device);
  const size_t hd = static_cast<size_t>(c.head_dim);
  const size_t esz = d->kv16 ? sizeof(__half) : sizeof(float);
  const size_t off = static_cast<size_t>(seq) * d->cache_seq + static_cast<size_t>(layer) * c.n_head_kv * c.n_ctx * hd +
                     static_cast<size_t>(pos) * hd;
  const size_t n = static_cast<size_t>(c.n_head_kv) * count * hd;
  const size_t row = count * hd * esz, pitch = c.n_ctx * hd * esz;
  const bool out = k_out != nullptr;
  std::vector<__half> stage(d->kv16 ? n : 0);
  for (int which = 0; which < 2; ++which) {
    uint8_t *dev = static_cast<uint8_t *>(which ? d->vcache : d->kcache) + off * esz;
    float *host_out = which ? v_out : k_out;
    const float *host_in = which ? v_in : k_in;
    void *host = d->kv16 ? static_cast<void *>(stage.data()) : (out ? static_cast<void *>(host_out) : const_cast<float *>(host_in));
    if (!out && d->kv16)
      for (size_t i = 0; i < n; ++i) stage[i] = __float2half_rn(host_in[i]);
    // one row per KV head: [n_kv][n_ctx][hd] (pitch n_ctx*hd) <-> [n_kv][count][hd]
    const cudaError_t e = out ? cudaMemcpy2DAsync(host, row, dev, pitch, row, c.n_head_kv, cudaMemcpyDeviceToHost, stream)
                              : cudaMemcpy2DAsync(dev, pitch, host, row, row, c.n_head_kv, cudaMemcpyHostToDevice, stream);
    if (e != cudaSuccess || cudaStreamSynchronize(stream) != cudaSuccess) return UGB_EBACKEND;
    if (out && d->kv16)
      for (size_t i = 0; i < n; ++i) host_out[i] = __half2float(stage[i]);
  }
  return UGB_OK;
}

}  // namespace

extern "C" ugb_status ugb_decoder_read_kv(ugb_decoder *d, ugb_stream stream, int32_t seq, int32_t layer, int32_t pos,
                                          int32_t count, float *k_host, float *v_host) {
  if (!d || !k_host || !v_host) return UGB_ECONTEXT;
  return kv_copy(d, stream, seq, layer, pos, count, k_host, v_host, nullptr, nullptr);
}

extern "C" ugb_status ugb_decoder_write_kv(ugb_decoder *d, ugb_stream stream, int32_t seq, int32_t layer, int32_t pos,
                                           int32_t count, const float *k_host, const float *v_host) {
  if (!d || !k_host || !v_host) return UGB_ECONTEXT;
  return kv_copy(d, stream, seq, layer, pos, count, nullptr, nullptr, k_host, v_host);
}

namespace ugb {
namespace {
ugb_status sync_prefill_trace(ugb_decoder *d);
}  // namespace
}  // namespace ugb

extern "C" ugb_status ugb_decoder_set_trace(ugb_decoder *d, int32_t enable) {
  if (!d) return UGB_ECONTEXT;
  cudaSetDevice(d->ctx->device);
  const size_t bytes = d->trace.rec * (static_cast<size_t>(d->cfg.n_layer) + 1);
  if (enable && !d->trace.base) {
    void *p = nullptr;
    if (cudaMalloc(&p, bytes) != cudaSuccess) return UGB_EBACKEND;
    if (cudaMemset(p, 0, bytes) != cudaSuccess) {
      cudaFree(p);
      return UGB_EBACKEND;
    }
    d->trace.base = static_cast<uint8_t *>(p);
    free_graph(d);  // the captured step has no trace stores
  } else if (!enable && d->trace.base) {
    if (cudaDeviceSynchronize() != cudaSuccess) return UGB_EBACKEND;
    cudaFree(d->trace.base);
    d->trace.base = nullptr;
    free_graph(d);
  }
  return sync_prefill_trace(d);
}

extern "C" ugb_status ugb_decoder_set_wait_limit(ugb_decoder *d, uint64_t ns) {
  if (!d) return UGB_ECONTEXT;
  if (ns < 1000 || ns > 60ull * 1000000000ull) return UGB_ESHAPE;
  d->wait_ns = ns;
  free_graph(d);  // the captured step holds the old limit
  return UGB_OK;
}

extern "C" ugb_status ugb_decoder_test_unreachable_wait(ugb_decoder *d, int32_t enable) {
  if (!d) return UGB_ECONTEXT;
  d->unreachable = enable ? 1u : 0u;
  free_graph(d);
  return UGB_OK;
}

extern "C" size_t ugb_decoder_trace_bytes(const ugb_decoder *d, int32_t field) {
  if (!d || field < 0 || field >= UGB_TRACE_FIELDS) return 0;
  return d->trace.bytes[field];
}

extern "C" ugb_status ugb_decoder_read_trace(ugb_decoder *d, ugb_stream stream, int32_t layer, int32_t field,
                                             void *host, size_t bytes) {
  if (!d || !host) return UGB_ECONTEXT;
  if (!d->trace.base) return UGB_ECONTEXT;
  if (field < 0 || field >= UGB_TRACE_FIELDS || layer < 0 || layer > d->cfg.n_layer) return UGB_ESHAPE;
  if (layer == d->cfg.n_layer && field != UGB_TRACE_X && field != UGB_TRACE_ATTN_NORM && field != UGB_TRACE_ATTN_XQ)
    return UGB_ESHAPE;
  if (bytes != d->trace.bytes[field] || bytes == 0) return UGB_ESHAPE;
  cudaSetDevice(d->ctx->device);
  if (cudaMemcpyAsync(host, d->trace.at(layer, field), bytes, cudaMemcpyDeviceToHost, stream) != cudaSuccess)
    return UGB_EBACKEND;
  return cuda_status(cudaStreamSynchronize(stream));
}

extern "C" ugb_status ugb_decoder_tokens(ugb_decoder *d, ugb_stream stream, const int32_t *tokens, int32_t pos,
                                         int32_t *next_tokens) {
  if (!d || !tokens || !next_tokens) return UGB_ECONTEXT;
  cudaSetDevice(d->ctx->device);
  if (!d->exec) {
    if (cudaStreamBeginCapture(d->cap, cudaStreamCaptureModeThreadLocal) != cudaSuccess) return UGB_EBACKEND;
    const ugb_status st = ugb_decoder_step(d, d->cap);
    cudaGraph_t g = nullptr;
    const cudaError_t e = cudaStreamEndCapture(d->cap, &g);
    if (st != UGB_OK || e != cudaSuccess) {
      if (g) cudaGraphDestroy(g);
      return st != UGB_OK ? st : UGB_EBACKEND;
    }
    if (cudaGraphInstantiate(&d->exec, g, 0) != cudaSuccess) {
      cudaGraphDestroy(g);
      return UGB_EBACKEND;
    }
    d->graph = g;
  }
  ugb_status st = ugb_decoder_set_tokens(d, stream, tokens, pos);
  if (st != UGB_OK) return st;
  if (cudaGraphLaunch(d->exec, stream) != cudaSuccess) return UGB_EBACKEND;
  if (cudaMemcpyAsync(d->state_host, d->state, sizeof(DecodeState), cudaMemcpyDeviceToHost, stream) != cudaSuccess)
    return UGB_EBACKEND;
  uint32_t bits = 0;
  st = ugb_status_read(d->ctx, stream, &bits);  // synchronises the stream
  if (st != UGB_OK) return st;
  for (int b = 0; b < d->batch; ++b) {
    next_tokens[b] = next_of(d->state_host, b);
    if (next_tokens[b] < 0) return UGB_ENONFINITE;  // every logit of a sequence was non-finite
  }
  return UGB_OK;
}

extern "C" ugb_status ugb_decoder_token(ugb_decoder *d, ugb_stream stream, int32_t token, int32_t pos,
                                        int32_t *next_token) {
  if (!d || !next_token) return UGB_ECONTEXT;
  int32_t t[kMaxSeq], n[kMaxSeq];
  for (int b = 0; b < kMaxSeq; ++b) t[b] = token;
  const ugb_status st = ugb_decoder_tokens(d, stream, t, pos, n);
  *next_token = n[0];
  return st;
}

// ---- whole-prompt prefill ------------------------------------------------------------------

namespace ugb {
namespace {

// (Re)allocate the prefill trace when tracing is on and a prefill is prepared.
ugb_status sync_prefill_trace(ugb_decoder *d) {
  const bool want = d->trace.base && d->pf_max > 0;
  if (d->ptrace.base && (!want || d->ptrace.rec == 0)) {
    cudaDeviceSynchronize();
    cudaFree(d->ptrace.base);
    d->ptrace.base = nullptr;
  }
  if (!want || d->ptrace.base) return UGB_OK;
  plan_trace(d, d->ptrace, d->pf_max);
  const size_t bytes = d->ptrace.rec * (static_cast<size_t>(d->cfg.n_layer) + 1);
  void *p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return UGB_EBACKEND;
  if (cudaMemset(p, 0, bytes) != cudaSuccess) {
    cudaFree(p);
    return UGB_EBACKEND;
  }
  d->ptrace.base = static_cast<uint8_t *>(p);
  return UGB_OK;
}

// Sequence 0's state after a prefill of n tokens from pos0: the last prompt token at position
// pos0 + n - 1, greedy key cleared for the head's argmax.
__global__ void prefill_state_kernel(const int32_t *__restrict__ tokens, int n, int pos0, DecodeState *state) {
  state->token[0] = tokens[n - 1];
  state->pos = pos0 + n - 1;
  state->key[0] = 0;
}

// Every kernel of one prefill, enqueued on `s` (graph-capturable).  Per layer: RMSNorm +
// quantisation into the packed operand, the Q/K/V GEMM, bias + RoPE + KV write, attention
// (partials + combine + quantisation), the O GEMM, RMSNorm + quantisation, the gate/up GEMM,
// SiLU * up + quantisation, the down GEMM.  A GEMM may be split over K; its consumer sums the
// splits in order.
ugb_status prefill_enqueue(ugb_decoder *d, cudaStream_t s, const int32_t *tokens, int n, int pos0) {
  const ugb_decoder_config &c = d->cfg;
  ugb_ctx *ctx = d->ctx;
  uint32_t *status = ctx->status;
  const int E = c.n_embd, Q = c.n_head * c.head_dim, KV = c.n_head_kv * c.head_dim, F = c.n_ff;
  const int brow = Q + 2 * KV;
  const size_t kv_layer = static_cast<size_t>(KV) * c.n_ctx * (d->kv16 ? sizeof(__half) : sizeof(float));
  const TraceMap &T = d->ptrace;
  const int s_qkv = prefill_gemm_splits(ctx, n, brow, E), s_o = prefill_gemm_splits(ctx, n, E, Q),
            s_gu = d->pf_gu_fused ? prefill_gemm_splits(ctx, n, 2 * F, E) : 1, s_dn = prefill_gemm_splits(ctx, n, E, F);
  // the split-K outputs: [splits][n][len] (partial sums of the first n rows, split stride n * len)
  const int64_t st_qkv = static_cast<int64_t>(n) * brow, st_e = static_cast<int64_t>(n) * E,
                st_gu = static_cast<int64_t>(n) * 2 * F;
  // trace: the sum of a split-K output, or a plain buffer, into field f of record l
  auto tsum = [&](int l, int f, const float *src, int splits, int64_t len) {
    return T.base ? launch_pf_sum_splits(s, src, splits, n * len, 0, n, len, T.f32(l, f)) : UGB_OK;
  };
  auto gemm = [&](size_t w_off, int64_t k, float *y, int64_t rows, int splits) {
    return launch_prefill_gemm(ctx, s, d->pf_w + w_off, d->pf_act, y, n, rows, k, rows, splits);
  };
  ugb_status st = launch_pf_embed(s, static_cast<const uint8_t *>(d->w.tok_embd), tokens, n, E, c.n_vocab, d->pf_x,
                                  status);
  for (int l = 0; l < c.n_layer && st == UGB_OK; ++l) {
    const ugb_layer_weights &L = d->layers[l];
    const size_t *off = d->pf_off.data() + 5 * l;
    // the residual entering the layer: x += the previous layer's down projection (its splits)
    st = launch_pf_norm_quant(s, d->pf_x, l ? d->pf_tmp : nullptr, s_dn, st_e, static_cast<const float *>(L.attn_norm),
                              n, E, c.norm_eps, d->pf_act, T.f32(l, UGB_TRACE_ATTN_NORM), status);
    if (st == UGB_OK && T.base)
      st = cuda_status(cudaMemcpyAsync(T.at(l, UGB_TRACE_X), d->pf_x, static_cast<size_t>(n) * E * 4,
                                       cudaMemcpyDeviceToDevice, s));
    if (st == UGB_OK && l) st = tsum(l - 1, UGB_TRACE_DOWN, d->pf_tmp, s_dn, E);
    if (st == UGB_OK) st = gemm(off[0], E, d->pf_qkv, brow, s_qkv);
    if (st == UGB_OK) st = tsum(l, UGB_TRACE_QKV, d->pf_qkv, s_qkv, brow);
    PrefillAttn a{};
    a.qkv = d->pf_qkv;
    a.ld = brow;
    a.splits = s_qkv;
    a.split_stride = st_qkv;
    a.bias = d->bias ? d->bias + static_cast<size_t>(l) * brow : nullptr;
    a.rope = d->rope;
    a.q = d->pf_q;
    a.kcache = static_cast<uint8_t *>(d->kcache) + kv_layer * l;
    a.vcache = static_cast<uint8_t *>(d->vcache) + kv_layer * l;
    a.kv16 = d->kv16;
    a.part_m = d->pf_pm;
    a.part_l = d->pf_pl;
    a.part_o = d->pf_po;
    a.cpi = d->pf_cpi;
    a.out = T.f32(l, UGB_TRACE_ATT);
    a.q_out = d->pf_act;
    a.s_out = reinterpret_cast<float *>(d->pf_act + prefill_layout(n, Q).q_bytes);
    a.status = status;
    a.n = n;
    a.pos0 = pos0;
    a.n_head = c.n_head;
    a.n_kv = c.n_head_kv;
    a.n_ctx = c.n_ctx;
    if (st == UGB_OK) st = launch_pf_rope_kv(s, a);
    if (st == UGB_OK) st = launch_pf_attention(s, a);
    if (st == UGB_OK) st = gemm(off[1], Q, d->pf_tmp, E, s_o);
    if (st == UGB_OK)
      st = launch_pf_norm_quant(s, d->pf_x, d->pf_tmp, s_o, st_e, static_cast<const float *>(L.ffn_norm), n, E,
                                c.norm_eps, d->pf_act, T.f32(l, UGB_TRACE_FFN_NORM), status);
    if (st == UGB_OK) st = tsum(l, UGB_TRACE_O, d->pf_tmp, s_o, E);
    if (d->pf_gu_fused) {
      if (st == UGB_OK) st = gemm(off[2], E, d->pf_gu, 2 * F, s_gu);
    } else {
      if (st == UGB_OK) st = launch_prefill_gemm(ctx, s, d->pf_w + off[2], d->pf_act, d->pf_gu, n, F, E, 2 * F, 1);
      if (st == UGB_OK) st = launch_prefill_gemm(ctx, s, d->pf_w + off[3], d->pf_act, d->pf_gu + F, n, F, E, 2 * F, 1);
    }
    if (st == UGB_OK) st = tsum(l, UGB_TRACE_GATE_UP, d->pf_gu, s_gu, 2 * F);
    if (st == UGB_OK)
      st = launch_pf_silu_quant(s, d->pf_gu, 2 * F, s_gu, st_gu, n, F, d->pf_act, T.f32(l, UGB_TRACE_H), status);
    if (st == UGB_OK) st = gemm(off[4], F, d->pf_tmp, E, s_dn);
  }
  if (st != UGB_OK) return st;
  st = tsum(c.n_layer - 1, UGB_TRACE_DOWN, d->pf_tmp, s_dn, E);
  // Only the last prompt token goes through the head (gpu_prefill.rs:138-148): its residual plus
  // the last down projection (summed over its splits), the output norm and Q8_1, the head matvec
  // and greedy selection.
  float *x_last = d->pf_x + static_cast<size_t>(n - 1) * E;
  if (st == UGB_OK) st = launch_pf_sum_splits(s, d->pf_tmp, s_dn, st_e, n - 1, 1, E, d->pf_last);
  if (st == UGB_OK)
    st = launch_rmsnorm_quant(s, false, x_last, d->pf_last, static_cast<const float *>(d->w.output_norm), E, 1,
                              c.norm_eps, d->pf_xq, nullptr, status, T.f32(c.n_layer, UGB_TRACE_ATTN_NORM));
  if (st == UGB_OK && T.base)
    st = cuda_status(cudaMemcpyAsync(T.at(c.n_layer, UGB_TRACE_X), x_last, E * 4, cudaMemcpyDeviceToDevice, s));
  if (st == UGB_OK && T.base)
    st = cuda_status(cudaMemcpyAsync(T.at(c.n_layer, UGB_TRACE_ATTN_XQ), d->pf_xq, q8act_layout(E, 1).bytes,
                                     cudaMemcpyDeviceToDevice, s));
  if (st != UGB_OK) return st;
  MatvecArgs a = mv_args(c.head_kind, E, c.n_vocab, 1, d->pf_xq, d->logits);
  a.w = static_cast<const uint8_t *>(d->w.output);
  a.pdl = false;
  st = launch_matvec(ctx, s, a);
  if (st != UGB_OK) return st;
  prefill_state_kernel<<<1, 1, 0, s>>>(tokens, n, pos0, d->state);
  st = cuda_status(cudaGetLastError());
  if (st == UGB_OK) st = launch_argmax(s, false, d->logits, c.n_vocab, 1, 0, d->state, ctx->sm_count);
  return st;
}

}  // namespace
}  // namespace ugb

extern "C" ugb_status ugb_decoder_prefill_prepare(ugb_decoder *d, ugb_stream stream, int32_t max_tokens) {
  if (!d || !d->w.layers) return UGB_ECONTEXT;
  const ugb_decoder_config &c = d->cfg;
  if (d->moe || d->batch != 1 || c.kind != UGB_Q8_0 || d->n_vocab_local != c.n_vocab) return UGB_ESHAPE;
  if (max_tokens < 1 || max_tokens > c.n_ctx) return UGB_ESHAPE;
  cudaSetDevice(d->ctx->device);
  if (cudaStreamSynchronize(stream) != cudaSuccess) return UGB_EBACKEND;
  if (d->pf_w) cudaFree(d->pf_w);
  if (d->pf_ws) cudaFree(d->pf_ws);
  d->pf_w = d->pf_ws = nullptr;
  d->pf_max = 0;
  const int64_t E = c.n_embd, Q = static_cast<int64_t>(c.n_head) * c.head_dim,
                KV = static_cast<int64_t>(c.n_head_kv) * c.head_dim, F = c.n_ff, brow = Q + 2 * KV;
  d->pf_gu_fused = F % kPrefillTile == 0;
  // packed weights: per layer qkv (one operand, the three matrices' 128-row tiles back to back),
  // o, gate (with up when fused), up (unfused), down
  d->pf_off.assign(5 * static_cast<size_t>(c.n_layer), 0);
  size_t total = 0;
  auto take = [&](size_t bytes) {
    const size_t o = total;
    total += round_up(bytes, 256);
    return o;
  };
  for (int l = 0; l < c.n_layer; ++l) {
    size_t *off = d->pf_off.data() + 5 * l;
    off[0] = take(prefill_layout(brow, E).bytes);
    off[1] = take(prefill_layout(E, Q).bytes);
    off[2] = take(prefill_layout(d->pf_gu_fused ? 2 * F : F, E).bytes);
    off[3] = d->pf_gu_fused ? 0 : take(prefill_layout(F, E).bytes);
    off[4] = take(prefill_layout(E, F).bytes);
  }
  const int64_t M = max_tokens, W = std::max({E, Q, F});
  size_t ws = 0;
  auto wtake = [&](size_t bytes) {
    const size_t o = ws;
    ws += round_up(bytes, 256);
    return o;
  };
  // attention partials: at most kMaxAttnGroups chunk groups per (16-token tile, KV head)
  constexpr int kMaxAttnGroups = 16;
  const int chunks = (c.n_ctx + 63) / 64;
  d->pf_cpi = (chunks + kMaxAttnGroups - 1) / kMaxAttnGroups;
  const size_t part_o = pf_attn_partial_floats(max_tokens, c.n_head, c.n_ctx, kMaxAttnGroups);
  const int64_t S = kMaxGemmSplits;
  const size_t o_x = wtake(M * E * 4), o_qkv = wtake(S * M * brow * 4), o_q = wtake(M * Q * 4),
               o_gu = wtake(S * M * 2 * F * 4), o_tmp = wtake(S * M * E * 4), o_act = wtake(prefill_layout(M, W).bytes),
               o_xq = wtake(q8act_layout(E, 1).bytes), o_tok = wtake(M * 4), o_pm = wtake(part_o / kHeadDim * 4),
               o_pl = wtake(part_o / kHeadDim * 4), o_po = wtake(part_o * 4), o_last = wtake(E * 4);
  if (cudaMalloc(&d->pf_w, total) != cudaSuccess) return UGB_EBACKEND;
  if (cudaMalloc(&d->pf_ws, ws) != cudaSuccess) {
    cudaFree(d->pf_w);
    d->pf_w = nullptr;
    return UGB_EBACKEND;
  }
  d->pf_x = reinterpret_cast<float *>(d->pf_ws + o_x);
  d->pf_pm = reinterpret_cast<float *>(d->pf_ws + o_pm);
  d->pf_pl = reinterpret_cast<float *>(d->pf_ws + o_pl);
  d->pf_po = reinterpret_cast<float *>(d->pf_ws + o_po);
  d->pf_last = reinterpret_cast<float *>(d->pf_ws + o_last);
  d->pf_qkv = reinterpret_cast<float *>(d->pf_ws + o_qkv);
  d->pf_q = reinterpret_cast<float *>(d->pf_ws + o_q);
  d->pf_gu = reinterpret_cast<float *>(d->pf_ws + o_gu);
  d->pf_tmp = reinterpret_cast<float *>(d->pf_ws + o_tmp);
  d->pf_act = d->pf_ws + o_act;
  d->pf_xq = d->pf_ws + o_xq;
  d->pf_tokens = reinterpret_cast<int32_t *>(d->pf_ws + o_tok);
  // repack: matrix `w` of `rows` rows at 128-row tile `tile0` of the operand at `off` of `all_rows`
  ugb_status st = UGB_OK;
  auto pack = [&](size_t off, int64_t all_rows, int64_t k, const void *w, int64_t rows, int64_t tile0) {
    if (st != UGB_OK) return;
    const PackedLayout p = prefill_layout(all_rows, k);
    uint8_t *q = d->pf_w + off + static_cast<size_t>(tile0) * p.nb * kPrefillTileBytes;
    float *sc = reinterpret_cast<float *>(d->pf_w + off + p.q_bytes) + static_cast<size_t>(tile0) * p.nb * kPrefillTile;
    st = launch_prefill_repack(stream, static_cast<const uint8_t *>(w), rows, k, q, sc);
  };
  for (int l = 0; l < c.n_layer; ++l) {
    const ugb_layer_weights &L = d->layers[l];
    const size_t *off = d->pf_off.data() + 5 * l;
    pack(off[0], brow, E, L.wq, Q, 0);
    pack(off[0], brow, E, L.wk, KV, Q / kPrefillTile);
    pack(off[0], brow, E, L.wv, KV, (Q + KV) / kPrefillTile);
    pack(off[1], E, Q, L.wo, E, 0);
    if (d->pf_gu_fused) {
      pack(off[2], 2 * F, E, L.w_gate, F, 0);
      pack(off[2], 2 * F, E, L.w_up, F, F / kPrefillTile);
    } else {
      pack(off[2], F, E, L.w_gate, F, 0);
      pack(off[3], F, E, L.w_up, F, 0);
    }
    pack(off[4], E, F, L.w_down, E, 0);
  }
  if (st == UGB_OK) st = cuda_status(cudaStreamSynchronize(stream));
  if (st != UGB_OK) return st;
  d->pf_max = max_tokens;
  return sync_prefill_trace(d);
}

extern "C" ugb_status ugb_decoder_prefill_async(ugb_decoder *d, ugb_stream stream, const int32_t *tokens_dev, int32_t n,
                                                int32_t pos0) {
  if (!d || !d->pf_w || !tokens_dev) return UGB_ECONTEXT;
  if (n < 1 || n > d->pf_max || pos0 < 0 || pos0 + n > d->cfg.n_ctx) return UGB_ESHAPE;
  cudaSetDevice(d->ctx->device);
  return prefill_enqueue(d, stream, tokens_dev, n, pos0);
}

extern "C" ugb_status ugb_decoder_prefill(ugb_decoder *d, ugb_stream stream, const int32_t *tokens_host, int32_t n,
                                          int32_t pos0, int32_t *next_token) {
  if (!d || !d->pf_w || !tokens_host || !next_token) return UGB_ECONTEXT;
  if (n < 1 || n > d->pf_max || pos0 < 0 || pos0 + n > d->cfg.n_ctx) return UGB_ESHAPE;
  for (int i = 0; i < n; ++i)
    if (tokens_host[i] < 0 || tokens_host[i] >= d->cfg.n_vocab) return UGB_ESHAPE;
  cudaSetDevice(d->ctx->device);
  if (cudaMemcpyAsync(d->pf_tokens, tokens_host, static_cast<size_t>(n) * 4, cudaMemcpyHostToDevice, stream) !=
      cudaSuccess)
    return UGB_EBACKEND;
  ugb_status st = prefill_enqueue(d, stream, d->pf_tokens, n, pos0);
  if (st != UGB_OK) return st;
  if (cudaMemcpyAsync(d->state_host, d->state, sizeof(DecodeState), cudaMemcpyDeviceToHost, stream) != cudaSuccess)
    return UGB_EBACKEND;
  st = ugb_status_read(d->ctx, stream, nullptr);  // synchronises the stream
  if (st != UGB_OK) return st;
  *next_token = next_of(d->state_host, 0);
  return *next_token < 0 ? UGB_ENONFINITE : UGB_OK;
}

extern "C" size_t ugb_decoder_prefill_trace_bytes(const ugb_decoder *d, int32_t field) {
  if (!d || field < 0 || field >= UGB_TRACE_FIELDS || !d->ptrace.base) return 0;
  return d->ptrace.bytes[field];
}

extern "C" ugb_status ugb_decoder_read_prefill_trace(ugb_decoder *d, ugb_stream stream, int32_t layer, int32_t field,
                                                     void *host, size_t bytes) {
  if (!d || !host || !d->ptrace.base) return UGB_ECONTEXT;
  if (field < 0 || field >= UGB_TRACE_FIELDS || layer < 0 || layer > d->cfg.n_layer) return UGB_ESHAPE;
  if (bytes == 0 || bytes > d->ptrace.bytes[field]) return UGB_ESHAPE;
  cudaSetDevice(d->ctx->device);
  if (cudaMemcpyAsync(host, d->ptrace.at(layer, field), bytes, cudaMemcpyDeviceToHost, stream) != cudaSuccess)
    return UGB_EBACKEND;
  return cuda_status(cudaStreamSynchronize(stream));
}
