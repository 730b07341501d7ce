/*
 * ugb.h -- C ABI of libugb, the B200 (sm_100a) quantized linear-layer hot path of the
 * nodnarbrox/uefi-gpu GGUF runtime.
 *
 * Drop-in boundary.  The reference drives its kernels from Rust through QMD/GPFIFO
 * submission (gpu_graph.rs:24-80, gpu_prefill.rs:10-30, frontier_gpu.rs:6-34,
 * frontier_batch.rs:19-72) and exposes them to the model code as Gpu::matvec / Gpu::batch
 * (llm.rs:226-273) and trait Weights::{linear,batch} (frontier_forward.rs:14-22).  Each
 * entry point below names the reference interface it replaces.  A Rust host binds them with
 * `extern "C"` declarations of the same names and #[repr(C)] structs of the same field order;
 * the CUDA stream argument replaces the GPFIFO channel.
 *
 * Conventions
 *  - Plain pointers and sizes only.  Pointers named `*_dev` or documented as device memory
 *    are CUDA device pointers; `*_host` pointers are host memory.
 *  - Buffers are caller-owned and must stay live until the work on `stream` completes
 *    (the reference holds its leases until the fence, frontier_backend.rs:211-213).
 *  - Calls are asynchronous on `stream` unless the name ends in a host-buffer form
 *    (ugb_linear / ugb_linear_batch), which synchronise and check results like the
 *    reference's Gpu::matvec (llm.rs:246-273).
 *  - Errors: ugb_status.  Shape / alignment / kind problems are caught on the host before
 *    anything is launched.  Device-side conditions (non-finite values, a timed-out wait)
 *    set bits in the context's status word, read with ugb_status_read().
 *  - One ugb_ctx per device; a context may be used from one host thread at a time.
 *  - `ugb_stream` is a CUstream / cudaStream_t (NULL = the legacy default stream).
 */
#ifndef UGB_H
#define UGB_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *ugb_stream;
typedef struct ugb_ctx ugb_ctx;

/* Status codes.  Mirrors the reference's Error{Backend,Shape,NonFinite,Context}
 * (frontier_forward.rs:10) plus alignment / quant-kind / timeout detail. */
typedef enum ugb_status {
  UGB_OK = 0,
  UGB_ESHAPE = 1,     /* a size or count is out of range (Error::Shape) */
  UGB_ENONFINITE = 2, /* non-finite input or output (Error::NonFinite) */
  UGB_ETIMEOUT = 3,   /* a bounded device-side wait gave up (the reference's poll timeout) */
  UGB_EBACKEND = 4,   /* a CUDA call failed (Error::Backend) */
  UGB_EALIGN = 5,     /* a pointer or stride breaks the documented alignment */
  UGB_EQUANT = 6,     /* unsupported quant kind (frontier_core::Error::QuantType) */
  UGB_ECONTEXT = 7    /* bad or missing context / not initialised (Error::Context) */
} ugb_status;

/* GGML type ids, the same numbers the reference uses for `kind` (frontier_core.rs:54-57).
 * Q8_0, Q4_K and Q3_K are the configurations' formats; Q6_K, IQ3_XXS, IQ4_NL and IQ4_XS are the
 * reference's other block formats (frontier_core.rs:85-103), accepted by the matvec entry points
 * (ugb_matvec, ugb_matvec_f32, ugb_matvec_jobs, ugb_linear, ugb_block_dots) and as the MoE expert
 * kind. */
enum {
  UGB_F32 = 0,
  UGB_F16 = 1,
  UGB_Q8_0 = 8,
  UGB_Q3_K = 11,
  UGB_Q4_K = 12,
  UGB_Q6_K = 14,
  UGB_IQ3_XXS = 18,
  UGB_IQ4_NL = 20,
  UGB_IQ4_XS = 23
};

/* Device status-word bits reported by ugb_status_read(). */
enum {
  UGB_STATUS_NONFINITE_IN = 1u << 0,
  UGB_STATUS_NONFINITE_OUT = 1u << 1,
  UGB_STATUS_TIMEOUT = 1u << 2,
  UGB_STATUS_BADARG = 1u << 3
};

/* Largest number of activation vectors one matvec launch multiplies (decode batch). */
#define UGB_MAX_BATCH 8
/* Largest row length K accepted.  The reference caps n at 16384 because of its 64 KiB input
 * window (frontier_backend.rs:245); the 7B-shaped configs need K = 18944, so this is larger. */
#define UGB_MAX_K 65536

/* ---- context --------------------------------------------------------------------------- */

/* Create a context on CUDA device `device`: queries the SM count, allocates the 4-byte
 * device status word and prepares every kernel's launch attributes.  Replaces the
 * reference's channel / compute-object setup (m4.rs:6-105). */
ugb_status ugb_init(int device, ugb_ctx **out);
ugb_status ugb_destroy(ugb_ctx *ctx);
const char *ugb_status_string(ugb_status s);

/* Synchronise `stream`, return the device status bits accumulated since the last read in
 * *bits, and clear them.  Returns UGB_ENONFINITE / UGB_ETIMEOUT when the corresponding bits
 * are set (TIMEOUT wins), UGB_OK otherwise. */
ugb_status ugb_status_read(ugb_ctx *ctx, ugb_stream stream, uint32_t *bits);

/* ---- formats ----------------------------------------------------------------------------- */

/* Bytes of one row of n elements of GGML type `kind`, or a negative value: -1 unknown kind,
 * -2 n not a positive multiple of the block.  frontier_core.rs:54-57 row_bytes(), with
 * the same table (F32, BF16, Q8_0, Q6_K, IQ3_XXS, IQ4_NL, IQ4_XS) plus Q4_K and Q3_K. */
int64_t ugb_row_bytes(uint32_t kind, int64_t n);

/* Q8_1 activation buffer ("xq"): `batch` vectors of k elements (k a multiple of 32), laid
 * out as int8 quants [batch][k] at offset 0, f32 block scales [batch][nbp] at
 * ugb_q8act_scale_offset, int32 block sums [batch][nbp] at ugb_q8act_sum_offset, where
 * nbp = k/32 rounded up to a multiple of 4.  The reference's activation block is
 * {f32 d; i8 q[32]} (gpu_dp4a.cu:23-31); this is the same data split into 16-byte aligned
 * arrays plus the block sum that Q4_K's min term needs. */
size_t ugb_q8act_bytes(int64_t k, int64_t batch);
size_t ugb_q8act_scale_offset(int64_t k, int64_t batch);
size_t ugb_q8act_sum_offset(int64_t k, int64_t batch);

/* ---- kernels ----------------------------------------------------------------------------- */

/* Quantise `batch` fp32 vectors x_dev [batch][k] into the Q8_1 buffer xq_dev.
 * Per 32-block: a = max|x|, d = a/127, q = clamp(rint(x*(127/a)), -127, 127), s = sum q.
 * Replaces quant_act (gpu_dp4a.cu:23-31, host hook graph_quant gpu_graph.rs:70-73) and
 * prefill_quant's arithmetic (gpu_prefill.cu:111-123).  Non-finite inputs quantise to 0 and
 * set UGB_STATUS_NONFINITE_IN. */
ugb_status ugb_quant_q8_1(ugb_ctx *ctx, ugb_stream stream, const float *x_dev, void *xq_dev,
                          int64_t k, int64_t batch);

/* y_dev[v][r] = sum over 32-blocks b of row r of the scaled int32 block dot with activation
 * vector v, for r < m, v < batch (<= UGB_MAX_BATCH).  w_dev holds m rows of `row_bytes`
 * bytes in the unchanged GGUF block layout of `kind` (Q8_0, Q4_K or Q3_K), 16-byte aligned.
 * Per block: Q8_0 isum*(d_w*d_x); Q4_K d_x*((d*sc)*isum - (dmin*m)*s); Q3_K isum*(d*d_x).
 * Replaces linear_dp4a (gpu_dp4a.cu:40-52; hook graph_linear gpu_graph.rs:74-80) and
 * frontier_matvec (frontier_quant.cu:58-66) with Q8_1 activations.  Weights are streamed
 * once with bulk copies into shared memory; y rows are written once. */
ugb_status ugb_matvec(ugb_ctx *ctx, ugb_stream stream, uint32_t kind, const void *w_dev,
                      int64_t row_bytes, const void *xq_dev, float *y_dev, int64_t k, int64_t m,
                      int64_t batch);

/* ugb_quant_q8_1 then ugb_matvec as one call: y_dev = W x for fp32 activations x_dev
 * [batch][k] (the quant_act + linear pair of graph_quant / graph_linear, gpu_graph.rs:70-80).
 * The quants, scales and sums are ugb_quant_q8_1's bit for bit, so y_dev equals the two-call
 * result exactly.  xq_scratch is a Q8_1 buffer of ugb_q8act_bytes(k, batch) bytes: a batch-1
 * matrix small enough to be staged whole (one CTA per SM) is quantised inside the matvec
 * itself and the scratch is not touched; other shapes quantise into it first.  Same
 * arguments, limits and status bits as the two calls. */
ugb_status ugb_matvec_f32(ugb_ctx *ctx, ugb_stream stream, uint32_t kind, const void *w_dev,
                          int64_t row_bytes, const float *x_dev, void *xq_scratch, float *y_dev,
                          int64_t k, int64_t m, int64_t batch);

/* Several matrices of the same kind and row length that share one activation, in one
 * launch: y_dev[v] = [W_0 x_v ; W_1 x_v ; ...] (rows concatenated in order), count <= 4.
 * w_devs (host array) holds the count device pointers, rows the count row counts.
 * Replaces qkv_dp4a / gateup_dp4a (gpu_dp4a.cu:53-64, the fused Q/K/V and gate/up launches
 * over separate GGUF tensors) and Gpu::batch (llm.rs:226-245, up to 3 tensors sharing one
 * input).  Results are bit-identical to one ugb_matvec per matrix, except Q4_K / Q8_0 with
 * 5..8 vectors: that form splits K by the launch's total rows, so the fp32 sums may associate
 * differently from the single launches' (same block dots, each within fp32 rounding). */
ugb_status ugb_matvec_multi(ugb_ctx *ctx, ugb_stream stream, uint32_t kind,
                            const void *const *w_devs, const int64_t *rows, int count,
                            int64_t row_bytes, const void *xq_dev, float *y_dev, int64_t k,
                            int64_t batch);

/* Debug / parity view of the same kernel: out_dev[r][b] = the int32 block dot of row r and
 * 32-block b with activation vector 0, no scaling (the integer the reference's CPU check
 * forms, gpu_prefill.rs:111-115).  Used to prove the integer parts bit-exact. */
ugb_status ugb_block_dots(ugb_ctx *ctx, ugb_stream stream, uint32_t kind, const void *w_dev,
                          int64_t row_bytes, const void *xq_dev, int32_t *out_dev, int64_t k,
                          int64_t m);

/* Fill a weight matrix of m rows x k elements of `kind` with seeded synthetic blocks
 * (quants uniform over the whole code range, fp16 scales |N(0,1)|*0.002 from a fixed
 * 256-entry quantile table).  Stand-in for GGUF weights when benchmarking. */
ugb_status ugb_fill_synthetic(ugb_ctx *ctx, ugb_stream stream, uint32_t kind, void *w_dev,
                              int64_t k, int64_t m, uint64_t seed);

/* ---- streams and graphs ------------------------------------------------------------------ */

/* Launch this context's kernels with programmatic dependent launch (enable != 0): each
 * kernel starts streaming its weights while the previous kernel in the stream drains, and
 * waits for that kernel's results before reading its activation.  Only valid when the kernel
 * immediately before a matvec does not write that matvec's weights (true for a decode graph,
 * whose weights are static).  Off by default. */
ugb_status ugb_set_pdl(ugb_ctx *ctx, int enable);

/* CUDA-graph capture of a sequence of ugb_* calls on `stream`, replacing the reference's
 * prebuilt per-token command list submitted as one GPFIFO entry (gpu_graph.rs:24-69,
 * forward_gpu gpu_graph.rs:170-197).  begin/end bracket the calls (cudaStreamBeginCapture /
 * cudaStreamEndCapture + instantiate); launch replays the graph on any stream. */
typedef struct ugb_graph ugb_graph;
ugb_status ugb_graph_begin(ugb_ctx *ctx, ugb_stream stream);
ugb_status ugb_graph_end(ugb_ctx *ctx, ugb_stream stream, ugb_graph **out);
ugb_status ugb_graph_launch(ugb_graph *graph, ugb_stream stream);
ugb_status ugb_graph_destroy(ugb_graph *graph);
/* Kernel launches one replay of the graph performs (its kernel nodes; collectives captured in
 * it contribute their own kernels). */
ugb_status ugb_graph_kernels(const ugb_graph *graph, int64_t *count);

/* ---- MoE expert path ----------------------------------------------------------------------- */

/* One independent matvec job: the 48-byte little-endian layout of the reference's
 * FrontierJob / Dispatch descriptor (frontier_quant.cu:71-78, frontier_dispatch.rs:9-31).
 * Here `input` is a Q8_1 activation (ugb_q8act layout for k = n and the call's batch) instead
 * of fp32, and `output` receives [batch][m] fp32.  first_row / padding are ignored: the
 * library assigns CTAs to jobs itself. */
typedef struct ugb_job {
  uint64_t weights, input, output; /* device pointers */
  uint32_t kind, n, m, row_bytes;
  uint32_t first_row, padding;
} ugb_job;
#define UGB_MAX_JOBS 32

/* Up to UGB_MAX_JOBS matvecs in as few launches as possible (one per (kind, n) group); each
 * job streams its own matrix against its own activation (frontier_multi_matvec,
 * frontier_quant.cu:79-93).  As the reference's packer, rejects empty or oversized jobs,
 * inconsistent row_bytes and overlapping outputs (UGB_ESHAPE).  jobs is a host array. */
ugb_status ugb_matvec_jobs(ugb_ctx *ctx, ugb_stream stream, const ugb_job *jobs, int count,
                           int64_t batch);

/* Router: per token, softmax over n_expert logits (frontier_forward.rs:47-51), the top_k
 * experts by descending probability with ties to the lower id (:167), and weights
 * p / (sum of the top_k p in rank order) (:168, :193).  logits [batch][n_expert] fp32 ->
 * ids [batch][top_k] int32, weights [batch][top_k] fp32, all device memory.  A token with a
 * non-finite logit gets ids -1 and sets the non-finite status bit.  n_expert <= 4096,
 * top_k <= 32. */
ugb_status ugb_moe_route(ugb_ctx *ctx, ugb_stream stream, const float *logits_dev, int64_t n_expert,
                         int64_t top_k, int64_t batch, int32_t *ids_dev, float *weights_dev);

/* out[t] (= or, with accumulate, +=) sum over ranks r of weights[t][r] * values[t][r] in rank
 * order with a separate fp32 multiply and add (frontier_forward.rs:193-195,
 * frontier_cpu_axpy.rs:13-21).  Ranks whose id is outside [expert0, expert0 + n_local) are
 * left out (expert parallelism: another device adds them). */
ugb_status ugb_moe_combine(ugb_ctx *ctx, ugb_stream stream, const float *values_dev,
                           const float *weights_dev, const int32_t *ids_dev, int64_t top_k,
                           int64_t d, int64_t batch, int64_t expert0, int64_t n_local,
                           int accumulate, float *out_dev);

/* The routed expert SwiGLU of one MoE layer, device-resident (Forward::ffn's expert part,
 * frontier_forward.rs:169-195): for every (token, rank) slot whose expert this device holds,
 * h = silu(gate_e x) * up_e x, value = down_e h, and out[t] (+)= sum of weight * value.
 * gate / up / down are the stacked GGUF expert tensors ([n_expert][rows][row_bytes]: gate and
 * up ffn rows of length hidden, down hidden rows of length ffn) of global experts
 * [expert0, expert0 + n_expert).  xq: Q8_1 of the batch tokens (length hidden). */
typedef struct ugb_moe_args {
  uint32_t kind;                 /* expert quant kind (UGB_Q3_K in config 5) */
  int32_t accumulate;            /* 0: out = sum; 1: out += sum */
  int64_t hidden, ffn, top_k, batch;
  int64_t n_expert, expert0, n_expert_total;
  const void *gate, *up, *down;  /* device, 16-byte aligned */
  const void *xq;                /* device Q8_1 [batch] */
  const int32_t *ids;            /* device [batch][top_k] global expert ids (ugb_moe_route) */
  const float *weights;          /* device [batch][top_k] */
  float *out;                    /* device [batch][hidden] */
  void *workspace;               /* device, 256-byte aligned, >= ugb_moe_workspace_bytes() */
  size_t workspace_bytes;
} ugb_moe_args;
/* Workspace of ugb_moe_experts, slots = batch * top_k, regions in this order, each starting
 * 256-byte aligned: gate/up outputs f32 [slots][2 * ffn]; the SiLU outputs as Q8_1 (ugb_q8act
 * layout for k = ffn, batch = slots); the expert outputs f32 [slots][hidden].  Slots routed to
 * another device's experts are left unwritten. */
size_t ugb_moe_workspace_bytes(int64_t hidden, int64_t ffn, int64_t top_k, int64_t batch);
ugb_status ugb_moe_experts(ugb_ctx *ctx, ugb_stream stream, const ugb_moe_args *args);

/* ---- Q8 prefill (INT8 tensor-core GEMM) ------------------------------------------------- */

/* Bytes of a packed prefill operand of `rows` rows (weight rows or tokens) of length k:
 * ceil(rows/128) tiles x k/32 blocks x (4096 B of int8 quants in the tcgen05 canonical
 * K-major layout + 512 B of f32 scales).  -1 if k is not a positive multiple of 32. */
int64_t ugb_prefill_packed_bytes(int64_t rows, int64_t k);

/* One-time lossless repack of an n x k Q8_0 matrix (GGUF rows) into the packed prefill
 * layout: the same quants and exactly converted fp16 scales, re-laid out in 128-row tiles
 * (prefill_repack / init_swizzle, gpu_prefill.cu:39-46, gpu_prefill.rs:58-94, which pack
 * 16-row mma.sync fragments instead).  packed_dev: ugb_prefill_packed_bytes(n, k) bytes,
 * 16-byte aligned. */
ugb_status ugb_prefill_repack_q8_0(ugb_ctx *ctx, ugb_stream stream, const void *w_dev, int64_t n,
                                   int64_t k, void *packed_dev);

/* Token-batched block-32 activation quantisation of x_dev [m][k] (fp32, row-major) into the
 * packed prefill layout (prefill_quant, gpu_prefill.cu:47-59; the arithmetic of quant_act).
 * Non-finite inputs are quantised as 0 and reported in the status word. */
ugb_status ugb_prefill_quant(ugb_ctx *ctx, ugb_stream stream, const float *x_dev, int64_t m,
                             int64_t k, void *packed_dev);

/* y_dev[t][r] (row stride ldy) = sum over 32-blocks b of (float)I_b * (dw[r][b] * dx[t][b]),
 * I_b the exact int32 block dot, for t < m tokens and r < n weight rows
 * (prefill_gemm, gpu_prefill.cu:10-36; p_gemm, gpu_prefill.rs:25-30).  tcgen05 INT8 MMA:
 * each block's int32 tile lands in tensor memory and is rescaled into fp32 accumulators. */
ugb_status ugb_prefill_gemm_q8_0(ugb_ctx *ctx, ugb_stream stream, const void *w_packed,
                                 const void *x_packed, float *y_dev, int64_t m, int64_t n,
                                 int64_t k, int64_t ldy);

/* Test path of the same GEMM: also writes every int32 block dot, dots_dev[b][t][r]
 * (k/32 x m x n int32), and y_dev with ldy = n.  Proves the tensor-core integer parts
 * bit-exact. */
ugb_status ugb_prefill_block_dots(ugb_ctx *ctx, ugb_stream stream, const void *w_packed,
                                  const void *x_packed, int32_t *dots_dev, float *y_dev, int64_t m,
                                  int64_t n, int64_t k);

/* ---- collectives (NCCL over NVLink) for sharded decoding -------------------------------- */

/* A communicator over the devices of one sharded decoder (one process or thread per GPU, at
 * most 8, all able to map each other's memory: one NVLink / NVSwitch node).  NCCL is loaded at
 * run time to create it; without NCCL these return UGB_EBACKEND.  Rank 0 makes the id with
 * ugb_comm_unique_id and the caller hands it to every rank (e.g. over its own process group);
 * ugb_comm_init is collective: every rank calls it at the same time.  It allocates each rank's
 * receive area and maps every peer's (CUDA IPC), so the collectives below are the library's own
 * kernels over peer memory (replacing the reference's single-GPU expert loop and vocabulary
 * projection, frontier_forward.rs:164-199, gpu_greedy.cu:13-27, when they are sharded).
 * ugb_comm_destroy is collective too. */
typedef struct ugb_comm ugb_comm;
#define UGB_COMM_ID_BYTES 128
#define UGB_COMM_MAX_WORDS 32768
ugb_status ugb_comm_unique_id(uint8_t *id_out /* UGB_COMM_ID_BYTES */);
ugb_status ugb_comm_init(ugb_ctx *ctx, int rank, int world, const uint8_t *id, ugb_comm **out);
ugb_status ugb_comm_destroy(ugb_comm *comm);

/* In-place all-reduce of n values of a device buffer (aligned to its element) over the communicator's
 * ranks, asynchronous on `stream` and capturable: every rank pushes its data into every rank's
 * receive area with peer stores, raises a flag there, waits (bounded by the wait limit; on
 * expiry the context's status word gets UGB_STATUS_TIMEOUT and the result is not valid) for
 * every rank's flag, and reduces the ranks' data in rank order, so all ranks hold the same bits.
 * f32: sum, n <= UGB_COMM_MAX_WORDS.  u64: maximum, n <= UGB_COMM_MAX_WORDS / 2.  Every rank must
 * make the same sequence of calls. */
ugb_status ugb_comm_allreduce_f32(ugb_comm *comm, ugb_stream stream, float *buf_dev, int64_t n);
ugb_status ugb_comm_allreduce_max_u64(ugb_comm *comm, ugb_stream stream, uint64_t *buf_dev, int64_t n);

/* ---- decoder (the per-token graph around the matvecs) ------------------------------------ */

/* Shape of a Qwen2/Qwen3-MoE-style decoder.  The reference hard-codes the 1.5B shape
 * (llm.rs:314-321: DIM 1536, HIDDEN 8960, KV 256, HEAD 128, LAYERS 28) and decodes one
 * sequence; here `batch` sequences (1..8) step together at a shared position, each with its
 * own tokens and KV cache.
 *  - n_expert = 0: dense SwiGLU FFN of n_ff (configs 2-4).  n_expert > 0: MoE FFN (config 5):
 *    router matvec (kind) over n_expert experts, top_k routing, SwiGLU experts of
 *    n_ff_expert in expert_kind (Forward::ffn, frontier_forward.rs:164-199).
 *  - Expert parallelism: this device holds global experts [expert0, expert0 + n_expert_local)
 *    (n_expert_local = 0: all).  With a communicator the layer outputs are summed over devices.
 *  - Vocabulary split: this device holds head rows [vocab0, vocab0 + n_vocab_local)
 *    (n_vocab_local = 0: all).  With a communicator the greedy keys are reduced over devices.
 *  - kv_type: element type of the KV cache, UGB_F32 (0, the reference's own cache,
 *    gpu_attention.cu:1) or UGB_F16 (1: keys and values rounded to nearest even as they are
 *    written; attention reads them back as fp16, the current position included). */
typedef struct ugb_decoder_config {
  int32_t n_layer, n_embd, n_ff, n_head, n_head_kv, head_dim, n_vocab, n_ctx;
  float rope_theta, norm_eps;
  uint32_t kind;      /* quant kind of the attention (and dense FFN / router) matrices */
  uint32_t head_kind; /* quant kind of the output head */
  int32_t batch;
  int32_t n_expert, top_k, n_ff_expert;
  uint32_t expert_kind;
  int32_t expert0, n_expert_local;
  int32_t vocab0, n_vocab_local;
  uint32_t kv_type;
} ugb_decoder_config;

/* Device pointers of one layer's GGUF tensors (blk.N.*): matrices in their GGUF block layout
 * with row length n_embd (w_down: n_ff; wo: n_head*head_dim), norms f32, biases f32 or NULL.
 * MoE layers use router (ffn_gate_inp, [n_expert][n_embd]) and the stacked expert tensors of
 * the held experts (ffn_{gate,up,down}_exps: [n_expert_local][rows][row_bytes]) instead of
 * w_gate / w_up / w_down. */
typedef struct ugb_layer_weights {
  const void *attn_norm, *wq, *wk, *wv, *bq, *bk, *bv, *wo;
  const void *ffn_norm, *w_gate, *w_up, *w_down;
  const void *router, *gate_exps, *up_exps, *down_exps;
} ugb_layer_weights;

typedef struct ugb_model_weights {
  const void *tok_embd;            /* Q8_0 [n_vocab][n_embd] (token_embd.weight) */
  const void *output_norm;         /* f32 [n_embd] */
  const void *output;              /* head_kind: the held rows [vocab0, +n_vocab_local) of the head */
  const ugb_layer_weights *layers; /* host array of n_layer entries */
} ugb_model_weights;

typedef struct ugb_decoder ugb_decoder;

/* Allocate the decoder's device state: KV cache of kv_type (batch x n_layer x n_head_kv x n_ctx
 * x head_dim, for K and V; the reference keeps its cache in fp32, gpu_attention.cu:1),
 * activations, RoPE table (f32 angle pos * powf(theta, -2i/head_dim), gpu_graph.rs:132),
 * attention partials, MoE workspace and the token state.  Replaces the reference's VRAM arenas
 * and graph build (gpu_graph.rs:81-169).  head_dim must be 128; n_head a multiple of
 * n_head_kv with at most 8 query heads per KV head. */
ugb_status ugb_decoder_create(ugb_ctx *ctx, const ugb_decoder_config *cfg, ugb_decoder **out);
ugb_status ugb_decoder_destroy(ugb_decoder *dec);

/* Use the given weights (device memory, caller-owned, must outlive the decoder). */
ugb_status ugb_decoder_bind(ugb_decoder *dec, const ugb_model_weights *w);

/* Allocate and bind seeded synthetic weights owned by the decoder (see ugb_fill_synthetic;
 * norms 1 +- 0.1, biases N(0, 0.02^2) approximately for dense models; tied head when
 * head_kind is Q8_0).  Expert e's tensors depend only on (seed, layer, e), so expert-parallel
 * shards of one seed form one model. */
ugb_status ugb_decoder_synthetic(ugb_decoder *dec, uint64_t seed);

/* Collectives for a sharded decoder (expert parallel and / or vocabulary split); NULL: none
 * (a shard then computes its partial results only). */
ugb_status ugb_decoder_set_comm(ugb_decoder *dec, ugb_comm *comm);

/* How a step runs.
 *   UGB_PATH_CHAIN -- the launch chain: about nine kernels per layer (matvecs, norms,
 *     attention, SiLU), each waiting for the previous one, as the reference's per-token
 *     command list (gpu_graph.rs:139-162).  Serves every configuration.
 *   UGB_PATH_TOKEN -- one persistent cooperative kernel per token, one CTA per SM: weights
 *     stream continuously through shared memory while device-wide counters order the phases.
 *     Dense decoders at batch 1 on one device only, with Q8_0 or Q4_K layers, a Q8_0 head,
 *     and 16-byte aligned tensors and rows.
 *   UGB_PATH_AUTO (default) -- TOKEN where it applies, else CHAIN.
 * Both paths compute the same step with the same arithmetic, except for fp32 summation order.
 * `active` (may be NULL) receives the path the next steps take.  Asking for TOKEN where it does
 * not apply returns UGB_ESHAPE and changes nothing.  No counterpart in the reference. */
#define UGB_PATH_AUTO 0
#define UGB_PATH_CHAIN 1
#define UGB_PATH_TOKEN 2
ugb_status ugb_decoder_set_path(ugb_decoder *dec, int32_t path, int32_t *active);

/* Enqueue one token step on `stream`: embedding of the current tokens, every layer, the head
 * and greedy selection.  A sequence's token comes from the previous step's greedy choice when
 * there is one (the position then advances), else from ugb_decoder_set_tokens, so replaying a
 * captured step decodes autoregressively on the device. */
ugb_status ugb_decoder_step(ugb_decoder *dec, ugb_stream stream);

/* Set the tokens ([batch]) and the shared position the next step starts from (asynchronous
 * host-to-device copy).  ugb_decoder_set_state sets every sequence to `token`. */
ugb_status ugb_decoder_set_tokens(ugb_decoder *dec, ugb_stream stream, const int32_t *tokens, int32_t pos);
ugb_status ugb_decoder_set_state(ugb_decoder *dec, ugb_stream stream, int32_t token, int32_t pos);

/* Synchronous: the tokens, position and greedy choices ([batch], -1 if none) of the last step.
 * ugb_decoder_get_state reports sequence 0. */
ugb_status ugb_decoder_get_tokens(ugb_decoder *dec, ugb_stream stream, int32_t *tokens, int32_t *pos,
                                  int32_t *next_tokens);
ugb_status ugb_decoder_get_state(ugb_decoder *dec, ugb_stream stream, int32_t *token,
                                 int32_t *pos, int32_t *next_token);

/* Synchronous copy of the last step's logits of the held head rows ([batch][n_vocab_local or
 * n_vocab] floats) to host memory. */
ugb_status ugb_decoder_logits(ugb_decoder *dec, ugb_stream stream, float *logits_host);

/* Synchronous copy of `count` cached positions starting at `pos` of sequence `seq`'s rotated
 * keys and values in one layer to host memory, each laid out [n_head_kv][count][head_dim].
 * No counterpart in the reference, whose host reads its KV cache at fixed device addresses
 * (llm.rs:319-320); here it serves inspection and checkpointing of a sequence. */
ugb_status ugb_decoder_read_kv(ugb_decoder *dec, ugb_stream stream, int32_t seq, int32_t layer, int32_t pos,
                               int32_t count, float *k_host, float *v_host);

/* The inverse of ugb_decoder_read_kv: host keys (already rotated) and values, each
 * [n_head_kv][count][head_dim], into `count` cached positions from `pos` of sequence `seq` in
 * one layer (an fp16 cache rounds them to nearest even).  Synchronous.  Restores a checkpointed
 * sequence, or seeds a history to decode from.  No counterpart in the reference (its host
 * writes the cache at fixed device addresses, llm.rs:319-320). */
ugb_status ugb_decoder_write_kv(ugb_decoder *dec, ugb_stream stream, int32_t seq, int32_t layer, int32_t pos,
                                int32_t count, const float *k_host, const float *v_host);

/* Step trace, for checking a step stage by stage against a CPU restatement: with tracing on,
 * every step also records, per layer l < n_layer, the fields below for every sequence
 * ([batch][len], fp32 unless Q8_1; a Q8_1 field is a ugb_q8act buffer of its length and the
 * decoder's batch):
 *   X         residual stream entering the layer (the embedding at l = 0)   [n_embd]
 *   ATTN_NORM RMSNorm output before quantisation                             [n_embd]
 *   ATTN_XQ   its Q8_1 quantisation, the Q/K/V matvec input                  Q8_1 n_embd
 *   QKV       the Q/K/V matvec output (before biases)                        [q ; k ; v rows]
 *   ATT       the attention output before quantisation                       [n_head * head_dim]
 *   ATT_XQ    its Q8_1, the O matvec input                                   Q8_1 n_head*head_dim
 *   O         the O matvec output                                            [n_embd]
 *   FFN_NORM  the second RMSNorm output before quantisation                  [n_embd]
 *   FFN_XQ    its Q8_1, the FFN input                                        Q8_1 n_embd
 *   GATE_UP   gate rows then up rows (dense FFN)                             [2 n_ff]
 *   H         SiLU(gate) * up before quantisation (dense FFN)                [n_ff]
 *   H_XQ      its Q8_1, the down matvec input (dense FFN)                    Q8_1 n_ff
 *   DOWN      the FFN output (down matvec, or the combined MoE experts)      [n_embd]
 * and in record l = n_layer: X (the final residual), ATTN_NORM (the output norm) and ATTN_XQ
 * (the head's input).  Tracing costs time and memory and is meant for tests; it is off by
 * default.  ugb_decoder_trace_bytes gives a field's size (0: no such field);
 * ugb_decoder_read_trace copies one field of the last step to host memory (synchronous).
 * No counterpart in the reference. */
/* Time limit of each wait of the persistent token kernel on other CTAs' progress (device-wide
 * phase counters, ring hand-offs), in ns: 1e3 .. 6e10, default 2e9.  When a wait runs out the
 * kernel records UGB_STATUS_TIMEOUT, every CTA leaves at its next wait, the counters are reset
 * for the next launch and the step's results are not valid: ugb_decoder_token / tokens and
 * ugb_status_read return UGB_ETIMEOUT, and the next step starts afresh.  The reference bounds its
 * own waits the same way (frontier_gpu.rs:30-33, llm.rs:267-269). */
ugb_status ugb_decoder_set_wait_limit(ugb_decoder *dec, uint64_t ns);

/* Test hook for that path: with enable != 0 the first attention wait of every token-kernel step
 * asks for one arrival more than there are CTAs, so it can end only by its time limit.  Lets a
 * test see a bounded wait run out without any fault.  The launch chain has no such wait and is
 * unaffected.  No counterpart in the reference. */
ugb_status ugb_decoder_test_unreachable_wait(ugb_decoder *dec, int32_t enable);

enum {
  UGB_TRACE_X = 0, UGB_TRACE_ATTN_NORM, UGB_TRACE_ATTN_XQ, UGB_TRACE_QKV, UGB_TRACE_ATT, UGB_TRACE_ATT_XQ,
  UGB_TRACE_O, UGB_TRACE_FFN_NORM, UGB_TRACE_FFN_XQ, UGB_TRACE_GATE_UP, UGB_TRACE_H, UGB_TRACE_H_XQ,
  UGB_TRACE_DOWN, UGB_TRACE_FIELDS
};
ugb_status ugb_decoder_set_trace(ugb_decoder *dec, int32_t enable);
size_t ugb_decoder_trace_bytes(const ugb_decoder *dec, int32_t field);
ugb_status ugb_decoder_read_trace(ugb_decoder *dec, ugb_stream stream, int32_t layer, int32_t field, void *host,
                                  size_t bytes);

/* One token end to end, as the reference's forward() (llm.rs:339-388 / forward_gpu
 * gpu_graph.rs:170-197): host tokens and position in, greedy next tokens out.  Replays a CUDA
 * graph of the step (captured on first use) and checks the status word.  ugb_decoder_token is
 * the single-sequence form (every sequence gets `token`; returns sequence 0's choice). */
ugb_status ugb_decoder_tokens(ugb_decoder *dec, ugb_stream stream, const int32_t *tokens, int32_t pos,
                              int32_t *next_tokens);
ugb_status ugb_decoder_token(ugb_decoder *dec, ugb_stream stream, int32_t token, int32_t pos,
                             int32_t *next_token);

/* ---- whole-prompt prefill ------------------------------------------------------------------ */

/* One-time preparation of ugb_decoder_prefill for the bound weights: repacks every layer's Q8_0
 * matrices into the tensor-core operand layout (the reference's init_swizzle / prefill_repack,
 * gpu_prefill.rs:58-94; Q/K/V and, when n_ff is a multiple of 128, gate/up become one operand
 * each; about 1.06x the layer weights in device memory) and allocates the activations of up to
 * max_tokens tokens (<= n_ctx).  Dense decoders with batch 1, Q8_0 layers and the whole head.
 * Synchronous.  Binding other weights drops the preparation: prepare again after
 * ugb_decoder_bind. */
ugb_status ugb_decoder_prefill_prepare(ugb_decoder *dec, ugb_stream stream, int32_t max_tokens);

/* Prefill n prompt tokens at positions pos0 .. pos0 + n - 1 in one pass (the reference's prefill
 * graph, gpu_prefill.rs:122-150, kernels gpu_prefill.cu:10-101): per layer the RMSNorm, block-32
 * quantisation of all n tokens, the Q/K/V, O, gate/up and down INT8 tensor-core GEMMs, bias +
 * RoPE with the KV-cache write, causal attention over positions [0, pos0 + t] for token t, and
 * SiLU * up; then only the last token through the final norm, the head and greedy selection
 * (gpu_prefill.rs:138-148).  Afterwards the decoder's state is that of a decode step of the last
 * prompt token at pos0 + n - 1 with its greedy choice, so ugb_decoder_step continues the
 * sequence at pos0 + n, and ugb_decoder_logits returns the last token's logits.
 * ugb_decoder_prefill: host tokens in, the greedy next token out (synchronous, status checked).
 * ugb_decoder_prefill_async: tokens in device memory (caller-owned, live until the work is
 * done), asynchronous on `stream` and capturable in a CUDA graph. */
ugb_status ugb_decoder_prefill(ugb_decoder *dec, ugb_stream stream, const int32_t *tokens_host, int32_t n,
                               int32_t pos0, int32_t *next_token);
ugb_status ugb_decoder_prefill_async(ugb_decoder *dec, ugb_stream stream, const int32_t *tokens_dev, int32_t n,
                                     int32_t pos0);

/* Trace of the last prefill while tracing is on (ugb_decoder_set_trace): the fields of the step
 * trace, each with max_tokens rows (the first n filled) instead of the batch: X, ATTN_NORM, QKV,
 * ATT, O, FFN_NORM, GATE_UP, H, DOWN per layer (the packed Q8_1 operands are not recorded), and in
 * record n_layer the last token's X, ATTN_NORM (row 0) and its head input ATTN_XQ (a ugb_q8act
 * buffer of batch 1 at the field's start).  bytes may be less than the field's size. */
size_t ugb_decoder_prefill_trace_bytes(const ugb_decoder *dec, int32_t field);
ugb_status ugb_decoder_read_prefill_trace(ugb_decoder *dec, ugb_stream stream, int32_t layer, int32_t field,
                                          void *host, size_t bytes);

/* ---- GGUF ingestion ------------------------------------------------------------------------ */

/* A parsed GGUF v3 directory (one file, or one shard of a split model): metadata and tensor
 * table, bounded and checked as the reference's Shard::parse (frontier_gguf.rs:145-200).  Tensor
 * bodies are not read: the directory gives each tensor's absolute file range, and the caller
 * copies the bytes it needs to the device.  The object copies what it keeps, so the prefix may be
 * freed after parsing.  Host code only; no CUDA call. */
typedef struct ugb_gguf ugb_gguf;

/* Results of the ugb_gguf_* calls: 0 or the reference's frontier_gguf::Error variant
 * (frontier_gguf.rs:7-8), in its order. */
enum {
  UGB_GGUF_OK = 0, UGB_GGUF_TRUNCATED, UGB_GGUF_MAGIC, UGB_GGUF_VERSION, UGB_GGUF_LIMIT, UGB_GGUF_TYPE,
  UGB_GGUF_UTF8, UGB_GGUF_ALIGNMENT, UGB_GGUF_SHAPE, UGB_GGUF_OVERFLOW, UGB_GGUF_TENSOR_BOUNDS,
  UGB_GGUF_OVERLAP, UGB_GGUF_DUPLICATE, UGB_GGUF_MISSING, UGB_GGUF_SPLIT
};

/* One tensor of the directory (Tensor, frontier_gguf.rs:84-88): dims[0] is the row length;
 * offset is absolute in the file (data section start + the tensor's own offset); bytes =
 * row_bytes x dims[1] x ... ; name is owned by the ugb_gguf. */
typedef struct ugb_gguf_tensor {
  const char *name;
  uint64_t dims[4];
  uint32_t rank, kind;
  uint64_t offset, bytes, row_bytes;
} ugb_gguf_tensor;

/* Parse the header prefix of a file of logical_bytes bytes (the prefix must hold the whole
 * directory, at most 16 MiB).  Limits: version 3, <= 4096 tensors, <= 1024 keys, keys and names
 * <= 256 bytes, strings <= 16 MiB, arrays <= 1e6 elements and not nested, alignment a power of
 * two <= 4096 (default 32), split.no < split.count <= 64, tensors rank 1..4 with non-zero dims,
 * aligned offsets, row lengths whole blocks of their kind, every tensor inside the file, no two
 * overlapping.  Kinds: those of ugb_row_bytes plus F16. */
int32_t ugb_gguf_parse(const uint8_t *prefix, size_t prefix_len, uint64_t logical_bytes, ugb_gguf **out);
void ugb_gguf_free(ugb_gguf *g);
/* data_offset: start of the data section; split_no / split_count / total_tensors of the split
 * set (0 / 1 / this file's count for an unsplit file). */
int32_t ugb_gguf_info(const ugb_gguf *g, uint64_t *data_offset, uint64_t *split_no, uint64_t *split_count,
                      uint64_t *total_tensors, int64_t *n_tensors);
int32_t ugb_gguf_tensor_at(const ugb_gguf *g, int64_t index, ugb_gguf_tensor *out);
int32_t ugb_gguf_find_tensor(const ugb_gguf *g, const char *name, ugb_gguf_tensor *out);
/* Absolute file range of rows [start, start + count) (Tensor::rows), and of expert `id` of a
 * rank-3 stacked expert tensor (Tensor::expert, frontier_gguf.rs:89-104). */
int32_t ugb_gguf_tensor_rows(const ugb_gguf_tensor *t, uint64_t start, uint64_t count, uint64_t *offset,
                             uint64_t *bytes);
int32_t ugb_gguf_tensor_expert(const ugb_gguf_tensor *t, uint32_t id, uint64_t *offset, uint64_t *bytes);

/* Metadata (Value, frontier_gguf.rs:42-72).  kind: the GGUF value type (0 u8 .. 12 f64).
 * unsigned: u8 / u16 / u32 / u64 values; float: f32; string: copies at most cap bytes and gives
 * the full length; array: element kind and count, and element `index` of an unsigned or string
 * array.  UGB_GGUF_MISSING for an absent key, UGB_GGUF_TYPE for another kind. */
int32_t ugb_gguf_meta_kind(const ugb_gguf *g, const char *key, uint32_t *kind);
int32_t ugb_gguf_meta_unsigned(const ugb_gguf *g, const char *key, uint64_t *value);
int32_t ugb_gguf_meta_float(const ugb_gguf *g, const char *key, float *value);
int32_t ugb_gguf_meta_string(const ugb_gguf *g, const char *key, char *buf, size_t cap, size_t *len);
int32_t ugb_gguf_meta_array(const ugb_gguf *g, const char *key, uint32_t *elem_kind, uint64_t *count);
int32_t ugb_gguf_meta_array_unsigned(const ugb_gguf *g, const char *key, uint64_t index, uint64_t *value);
int32_t ugb_gguf_meta_array_string(const ugb_gguf *g, const char *key, uint64_t index, char *buf, size_t cap,
                                   size_t *len);

/* A split model's shards as one directory (ModelIndex::new, frontier_gguf.rs:113-125): shard i
 * must be split i of `count`, all with the same total tensor count, no name twice, and every
 * tensor present (UGB_GGUF_SPLIT / UGB_GGUF_DUPLICATE otherwise).  inventory: on-disk bytes of
 * ordinary tensors, of per_layer_token_embd.weight and of *_exps.weight tensors
 * (ModelIndex::inventory). */
int32_t ugb_gguf_check_index(ugb_gguf *const *shards, int32_t count);
int32_t ugb_gguf_inventory(ugb_gguf *const *shards, int32_t count, uint64_t *counts /* [3] */);

/* A Qwen2 / Qwen3-MoE decoder from a model's directory (shards as ugb_gguf_check_index accepts):
 * ugb_gguf_decoder_config fills the shape from the architecture's metadata (<arch>.block_count,
 * embedding_length, feed_forward_length, attention.head_count(_kv), context_length,
 * rope.freq_base, attention.layer_norm_rms_epsilon, expert_count, expert_used_count,
 * expert_feed_forward_length) and the kinds from the tensors; batch 1, all experts and head rows,
 * fp32 KV.  ugb_gguf_model_weights points every tensor of cfg's layers into device copies of the
 * shards' bytes: dev_bases[i] holds shard i's file bytes from file offset base_offsets[i]
 * (normally its data_offset), dev_sizes[i] bytes of them; a tied model (no output.weight) reuses
 * token_embd.weight.  layers: n_layer entries.  UGB_GGUF_MISSING names no tensor, and
 * UGB_GGUF_SHAPE / UGB_GGUF_TYPE a tensor whose dims or kind do not fit cfg. */
int32_t ugb_gguf_decoder_config(ugb_gguf *const *shards, int32_t count, ugb_decoder_config *cfg);
int32_t ugb_gguf_model_weights(ugb_gguf *const *shards, int32_t count, const void *const *dev_bases,
                               const uint64_t *base_offsets, const uint64_t *dev_sizes,
                               const ugb_decoder_config *cfg, ugb_model_weights *weights,
                               ugb_layer_weights *layers);

/* ---- host-buffer entry points (synchronous) --------------------------------------------- */

/* y_host[m] = W x_host[k], synchronously: copy x to the device, quantise, matvec, copy y
 * back, then check the status word.  Returns UGB_ENONFINITE for a non-finite x or y, as the
 * reference's Gpu::matvec (llm.rs:246-273) and Weights::linear (frontier_backend.rs:243-275)
 * fail on non-finite data.  Uses a per-context device workspace grown on demand. */
ugb_status ugb_linear(ugb_ctx *ctx, ugb_stream stream, uint32_t kind, const void *w_dev,
                      int64_t row_bytes, const float *x_host, float *y_host, int64_t k,
                      int64_t m);

/* ugb_linear without any allocation: the same x -> quantise -> matvec -> y round trip, with
 * its device scratch in a fixed 2,183,168-byte array compiled into the library.  No
 * counterpart in the reference (whose firmware host owns fixed VRAM arenas); it is for
 * callers that must not let a library allocate on their behalf -- hosts that plan device
 * memory up front, or loops that cannot take the implicit synchronisation or late
 * out-of-memory failure of a first-use cudaMalloc.
 *   - k <= UGB_LINEAR_STATIC_MAX_K and m <= UGB_LINEAR_STATIC_MAX_M, else UGB_ESHAPE (the
 *     reference's own Weights::linear caps, frontier_backend.rs:245-248).
 *   - Every call makes ctx's device current, as every entry point does.  The first call on a
 *     device looks up the array's address (cudaGetSymbolAddress with that device current) and
 *     caches it for the process; make that first call before any stream capture begins.  The
 *     cache assumes the device's primary context lives as long as the process (not across a
 *     cudaDeviceReset).
 *   - Nothing needs to start at zero: every scratch byte a call reads it wrote first.
 *   - One array per device, shared by all contexts and streams: calls on the same device
 *     that overlap in time race on it.  The call is synchronous, so back-to-back calls from
 *     one thread are safe. */
#define UGB_LINEAR_STATIC_MAX_K 16384
#define UGB_LINEAR_STATIC_MAX_M 524288
ugb_status ugb_linear_static(ugb_ctx *ctx, ugb_stream stream, uint32_t kind, const void *w_dev,
                             int64_t row_bytes, const float *x_host, float *y_host, int64_t k,
                             int64_t m);

#ifdef __cplusplus
}
#endif
#endif /* UGB_H */
