// token.cu -- one batch-1 decode step of a dense decoder as a single persistent kernel.
//
// The launch chain of decoder.cu runs about nine dependent kernels per layer.  At batch 1
// each of them is latency-bound, and HBM idles while every matvec ramps up and drains.
// Here one CTA per SM lives for the whole token:
//  * a producer warp streams the CTA's share of every weight matrix of the step (all layers,
//    then the head) into a byte ring in shared memory with cp.async.bulk, in the order the
//    consumers use it.  Weights do not depend on activations, so the stream waits only for
//    ring space, never for a layer boundary, and HBM stays busy across the glue phases;
//  * sixteen consumer warps run the step's phases.  A phase that needs other CTAs' outputs
//    reads them as tagged 64-bit words -- 32 data bits and a launch/layer tag in one store: the
//    Q/K/V rows, the O and down outputs, and the Q8_1 attention and SiLU outputs -- until every
//    tag it needs is current.  There is no device-wide barrier between phases: each waits only
//    for the words it reads.  Every wait is bounded, and an abort flag ends all of them at once.
// Phases of layer l:
//   A  x += dx_down (x = the token's embedding row at l = 0); RMSNorm; Q8_1 into shared
//      memory (every CTA keeps its own copy of the residual stream and of the activation);
//      the CTA's Q/K/V rows -> qkv
//   B  attention partials of (KV head, 64-position chunk) units: bias, RoPE, KV-cache write,
//      scores, chunk softmax, P.V (the launch chain's attn_partial_kernel, per CTA)
//      and the last unit of each (KV head, query subgroup) combines that subgroup's chunks and
//      writes its heads' quantised attention output (a ticket per subgroup picks the last unit)
//   C  every CTA loads the quantised attention output; the CTA's O rows -> dx_o
//   D  x += dx_o; RMSNorm; Q8_1; the CTA's gate and up rows of whole 32-row blocks, so the
//      CTA forms SiLU(gate) * up of those blocks and their Q8_1 blocks itself -> hq
//   E  hq into shared memory; the CTA's down rows -> dx_down
// and after the last layer: x += dx_down, the output norm, the CTA's head rows (logits), and
// a per-CTA greedy key folded into the token state with one atomicMax.
// The arithmetic of every step is the launch chain's (reference: gpu_graph.rs:139-162,
// llm.rs:339-388); only fp32 summation orders differ.
#include <algorithm>
#include <cfloat>
#include <cmath>

#include "decode.hpp"
#include "formats.cuh"
#include "glue.cuh"

namespace ugb {
namespace {

constexpr int kCW = 16;                  // consumer warps
constexpr int kCT = kCW * 32;            // consumer threads
constexpr int kTT = kCT + 32;            // + the producer warp
constexpr int kNS = 16;                  // ring items in flight at most (mbarrier pairs)
constexpr uint32_t kMiscBytes = 1024;    // TokMisc, after the mbarriers
constexpr int kSyncStride = 32;          // u32 words per counter: one 128-byte line each
constexpr uint32_t kRingSlack = 16;      // readable bytes after the ring
constexpr int kPV = kCT / kHeadDim;      // threads per output dimension in the P.V step
static_assert(kCT % kHeadDim == 0 && kAttnChunk % kPV == 0, "P.V thread layout");

// Device-wide counters of a step (TokenStep::sync), zero between launches: the last CTA to
// leave zeroes them for the next launch.  (Words kCntA..kCntE are kept in the layout, unused:
// the phases now hand over through tagged words.)
enum : int { kStart, kCntA, kCntB, kCntC, kCntD, kCntE, kAbort, kExit, kNumSync };
// After the counters: one ticket per (KV head, query subgroup), counting the attention units of
// the subgroup that have written their partials (the last one combines them); zero between uses.
constexpr int kTicket0 = kNumSync * kSyncStride;
constexpr int kMaxTickets = 32;
// Then the launch epoch: the tags of the exchanged O / down outputs are epoch * 256 + layer + 1,
// so a word left from an earlier layer or launch (or the zeroed start) never matches the current
// one.  The last CTA out advances it.
constexpr int kEpochWord = kTicket0 + kMaxTickets;
static_assert(kEpochWord < static_cast<int>(token_sync_words()), "counter block too small");
__host__ __device__ constexpr uint32_t dx_tag(uint32_t epoch, int layer) {
  return epoch * 256u + static_cast<uint32_t>(layer) + 1u;
}

// Matrices of a layer, in the order the producer streams them.
enum : int { kSlotQKV, kSlotO, kSlotGate, kSlotUp, kSlotDown, kSlotHead };

__device__ __forceinline__ void cbar() {
  asm volatile("bar.sync 1, %0;" ::"n"(kCT) : "memory");
}

// AND of a predicate over the consumer threads (also a consumer barrier).
__device__ __forceinline__ bool cbar_and(bool v) {
  uint32_t all;
  asm volatile(
      "{\n\t.reg .pred pi, po;\n\tsetp.ne.u32 pi, %1, 0;\n\t"
      "bar.red.and.pred po, 1, %2, pi;\n\tselp.u32 %0, 1, 0, po;\n\t}"
      : "=r"(all)
      : "r"(v ? 1u : 0u), "n"(kCT)
      : "memory");
  return all != 0;
}

__device__ __forceinline__ uint32_t ld_relaxed(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint32_t *sync_word(const TokenStep &p, int which) {
  return p.sync + which * kSyncStride;
}

__device__ __forceinline__ bool aborted(const TokenStep &p) { return ld_relaxed(sync_word(p, kAbort)) != 0; }

__device__ __forceinline__ void abort_all(const TokenStep &p) {
  atomicExch(sync_word(p, kAbort), 1u);
  status_or(p.status, ST_TIMEOUT);
}


__device__ __forceinline__ unsigned long long ld_relaxed64(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// One exchanged output: value and tag in one 64-bit store, so a reader sees both or neither.
__device__ __forceinline__ void st_tagged_bits(unsigned long long *p, uint32_t bits, uint32_t tag) {
  const unsigned long long w = (static_cast<unsigned long long>(tag) << 32) | bits;
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ void st_tagged(unsigned long long *p, float v, uint32_t tag) {
  st_tagged_bits(p, __float_as_uint(v), tag);
}

// One warp, one element per lane: the block-32 quantisation of quant_block, stored as the
// block's kQ8TagWords tagged words at w (lanes 4j store quants 4j..4j+3, lane 0 the scale and the
// sum).  Returns whether any element was non-finite.
__device__ __forceinline__ bool quant_block_tagged(float v, int lane, unsigned long long *w, uint32_t tag) {
  int qi, sum;
  float d;
  const bool bad = quant_block_values(v, qi, d, sum);
  const uint32_t b = static_cast<uint32_t>(qi) & 0xffu;
  const uint32_t word = b | (__shfl_down_sync(0xffffffffu, b, 1) << 8) | (__shfl_down_sync(0xffffffffu, b, 2) << 16) |
                        (__shfl_down_sync(0xffffffffu, b, 3) << 24);
  if ((lane & 3) == 0) st_tagged_bits(w + (lane >> 2), word, tag);
  if (lane == 0) {
    st_tagged_bits(w + 8, __float_as_uint(d), tag);
    st_tagged_bits(w + 9, static_cast<uint32_t>(sum), tag);
  }
  return bad;
}
static_assert(kQ8TagWords == 10, "tagged Q8_1 block: 8 quant words, scale, sum");

// A tagged word written by another CTA in this phase: read until its tag is `tag` (false when the
// step was aborted or the wait limit passed, then the value is 0).
__device__ __forceinline__ float poll_tagged(const TokenStep &p, const unsigned long long *w, uint32_t tag, bool &ok) {
  unsigned long long v = ld_relaxed64(w);
  if (static_cast<uint32_t>(v >> 32) == tag) return __uint_as_float(static_cast<uint32_t>(v));
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    v = ld_relaxed64(w);
    if (static_cast<uint32_t>(v >> 32) == tag) return __uint_as_float(static_cast<uint32_t>(v));
    if ((it & 15) == 0) {
      if (aborted(p)) break;
      if (globaltimer_ns() - t0 > p.wait_ns) {
        abort_all(p);
        break;
      }
    }
  }
  ok = false;
  return 0.f;
}

__device__ __forceinline__ uint32_t ld_acquire(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// One thread: wait until counter `which` reaches `target` (acquire: the counted CTAs' writes
// are visible to this thread, and through the consumer barrier that follows to the whole CTA).
// False when another CTA aborted the step or the limit passed (this thread then aborts it).
__device__ bool spin_until(const TokenStep &p, int which, uint32_t target) {
  const uint32_t *c = sync_word(p, which);
  if (ld_acquire(c) >= target) return true;
  // Poll with relaxed loads (one L2 round trip each); the abort flag and the clock are looked
  // at every 16th poll only, and the acquire fence is taken once the count is reached.
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t n = 1;; ++n) {
    if (ld_relaxed(c) >= target) {
      asm volatile("fence.acq_rel.gpu;" ::: "memory");
      return true;
    }
    if ((n & 15) == 0) {
      if (aborted(p)) return false;
      if (globaltimer_ns() - t0 > p.wait_ns) {
        abort_all(p);
        return false;
      }
    }
  }
}

// Bounded wait on an mbarrier phase that also ends when the step is aborted.
__device__ bool mbar_wait_step(const TokenStep &p, uint32_t bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
    if (mbar_try_wait(bar, parity)) return true;
    if (aborted(p)) return false;
    if (globaltimer_ns() - t0 > p.wait_ns) {
      abort_all(p);
      return false;
    }
  }
}

// ---- the schedule: which rows of which matrix each CTA streams, in which order -------------

constexpr int kJ = 3;                // (row, unit) slots a lane holds, activation units in registers
constexpr int kMaxTokLayers = 256;   // layer tables staged in shared memory at most

// Rows [r0, r1) of m, CTA c of P (balanced contiguous split).
__device__ __forceinline__ void share(int m, int c, int P, int &r0, int &r1) {
  r0 = static_cast<int>(static_cast<int64_t>(m) * c / P);
  r1 = static_cast<int>(static_cast<int64_t>(m) * (c + 1) / P);
}

// One span of a CTA's schedule: rows [first, first + n) of one matrix, streamed as ni items of
// per + 1 (the first rem items) or per rows, each at most kTokItemMax bytes; out0 is the output
// row of the span's first row.  The spans are the same in every layer, so each CTA computes
// them once per launch (integer divisions stay off the per-item path).
struct Span {
  int first, n, ni, per, rem, out0;
};
enum : int { kSpanQ, kSpanK, kSpanV, kSpanO, kSpanGate, kSpanUp, kSpanDown, kSpanHead, kNumSpans };

struct TokPlan {
  Span sp[kNumSpans];
  int gb0, gb1;  // the CTA's FFN blocks (of 32 rows of gate and of up)
};

__device__ void make_span(Span &s, int first, int n, uint32_t rb, int out0) {
  const int maxr = max(1, static_cast<int>(kTokItemMax / rb));
  s.first = first;
  s.n = max(n, 0);
  s.out0 = out0;
  s.ni = (s.n + maxr - 1) / maxr;
  s.per = s.ni ? s.n / s.ni : 0;
  s.rem = s.ni ? s.n % s.ni : 0;
}

// The CTA's spans (one thread).  Output rows: Q/K/V -> row of the concatenated [q; k; v];
// gate / up -> row of the FFN; O, down -> row of the hidden state; head -> vocabulary id.
__device__ void make_plan(const TokenStep &p, TokPlan &pl) {
  const int c = blockIdx.x, P = gridDim.x;
  const int qr = p.n_head * kHeadDim, kr = p.n_kv * kHeadDim;
  int r0, r1;
  share(qr + 2 * kr, c, P, r0, r1);
  const int s0[4] = {0, qr, qr + kr, qr + 2 * kr};
  for (int s = 0; s < 3; ++s) {
    const int a = max(r0, s0[s]), b = min(r1, s0[s + 1]);
    make_span(pl.sp[kSpanQ + s], a - s0[s], b - a, p.rb_e, a);
  }
  share(p.n_embd, c, P, r0, r1);
  make_span(pl.sp[kSpanO], r0, r1 - r0, p.rb_q, r0);
  make_span(pl.sp[kSpanDown], r0, r1 - r0, p.rb_f, r0);
  share(p.n_ff / 32, c, P, pl.gb0, pl.gb1);
  make_span(pl.sp[kSpanGate], 32 * pl.gb0, 32 * (pl.gb1 - pl.gb0), p.rb_e, 32 * pl.gb0);
  make_span(pl.sp[kSpanUp], 32 * pl.gb0, 32 * (pl.gb1 - pl.gb0), p.rb_e, 32 * pl.gb0);
  share(p.n_vocab, c, P, r0, r1);
  make_span(pl.sp[kSpanHead], r0, r1 - r0, p.rb_h, r0);
}

// Spans [s0, s1] of matrix `slot`, and the matrix and row bytes of span `sp`.
__device__ __forceinline__ void slot_spans(int slot, int &s0, int &s1) {
  s0 = slot == kSlotQKV ? kSpanQ : slot + (kSpanO - kSlotO);
  s1 = slot == kSlotQKV ? kSpanV : s0;
}
__device__ __forceinline__ const uint8_t *span_matrix(const TokenStep &p, const TokLayer &L, int sp) {
  switch (sp) {
    case kSpanQ: return L.wq;
    case kSpanK: return L.wk;
    case kSpanV: return L.wv;
    case kSpanO: return L.wo;
    case kSpanGate: return L.wg;
    case kSpanUp: return L.wu;
    case kSpanDown: return L.wd;
    default: return p.head;
  }
}
__device__ __forceinline__ uint32_t span_rb(const TokenStep &p, int sp) {
  return sp == kSpanO ? p.rb_q : sp == kSpanDown ? p.rb_f : sp == kSpanHead ? p.rb_h : p.rb_e;
}

// The items of matrix `slot` (of layer L) that this CTA streams, in stream order:
// f(src, bytes, first output row, rows).  f has a single call site, so a caller's item body is
// inlined once (the consumers' row-dot loops are the bulk of the kernel's code, and the code
// a layer runs has to stay small enough for the instruction caches).
template <class F>
__device__ void visit(const TokenStep &p, const TokPlan &pl, const TokLayer &L, int slot, F &&f) {
  int s0, s1;
  slot_spans(slot, s0, s1);
  for (int sp = s0; sp <= s1; ++sp) {
    const Span &s = pl.sp[sp];
    const uint8_t *w = span_matrix(p, L, sp);
    const uint32_t rb = span_rb(p, sp);
    int a = 0;
    for (int i = 0; i < s.ni; ++i) {
      const int nr = s.per + (i < s.rem ? 1 : 0);
      f(w + static_cast<uint64_t>(s.first + a) * rb, static_cast<uint32_t>(nr) * rb, s.out0 + a, nr);
      a += nr;
    }
  }
}

// Placement of items in the byte ring, computed identically by the producer and the
// consumers: each item right after the previous one, or at 0 when it would run past the end.
struct Cursor {
  uint32_t t = 0, end = 0;
  __device__ __forceinline__ uint32_t place(uint32_t len, uint32_t ring_bytes) {
    const uint32_t off = end + len > ring_bytes ? 0u : end;
    end = off + len;
    ++t;
    return off;
  }
};

__device__ __forceinline__ bool overlaps(uint32_t a0, uint32_t alen, uint32_t b0, uint32_t blen) {
  return a0 < b0 + blen && b0 < a0 + alen;
}

// Per-CTA scratch at the start of shared memory, after the mbarriers.
struct TokMisc {
  int ok;            // result of the last phase wait, broadcast to the consumer warps
  int last;          // this CTA's attention unit was its subgroup's last (it combines)
  int tok, pos;
  uint32_t issued;   // items the producer issued
  uint32_t epoch;    // the launch epoch (tags of the exchanged outputs)
  uint32_t pad[2];
  float red[32];
  unsigned long long key[32];
  TokPlan plan;
};
static_assert(sizeof(TokMisc) <= kMiscBytes, "TokMisc outgrew its slot");

// ---- producer -------------------------------------------------------------------------------

// Lane 0 of the producer warp: stream every item of the step into the ring.  Before item t
// lands at [off, off + len), the items still in flight that overlap it -- and the one that last
// used its mbarrier pair -- must have been released by the consumers (in order, oldest first).
// Returns the number of items issued (all of them unless the step was aborted).
__device__ uint32_t produce(const TokenStep &p, uint32_t base, const TokPlan &pl, const TokLayer *layers) {
  const uint32_t full = base, empty = base + 8 * kNS, ring = base + p.o_ring;
  const uint64_t pol = policy_evict_first();  // every weight byte is read once per token
  Cursor cur;
  uint32_t qoff[kNS], qlen[kNS];
  uint32_t done = 0;  // items known to be released
  bool ok = true;
  auto issue = [&](const uint8_t *src, uint32_t bytes, int, int) {
    if (!ok) return;
    const uint32_t off = cur.place(bytes, p.ring_bytes);
    const uint32_t t = cur.t - 1;
    for (;;) {
      bool need = done + kNS <= t;
      for (uint32_t j = done; !need && j < t; ++j) need = overlaps(qoff[j % kNS], qlen[j % kNS], off, bytes);
      if (!need) break;
      if (!mbar_wait_step(p, empty + 8 * (done % kNS), (done / kNS) & 1)) {
        ok = false;
        cur.t = t;  // this item was not issued
        return;
      }
      ++done;
    }
    qoff[t % kNS] = off;
    qlen[t % kNS] = bytes;
    mbar_arrive_expect_tx(full + 8 * (t % kNS), bytes);
    bulk_g2s(ring + off, src, bytes, full + 8 * (t % kNS), pol);
  };
  for (int l = 0; l < p.n_layer && ok; ++l) {
    for (int slot = kSlotQKV; slot <= kSlotDown && ok; ++slot) visit(p, pl, layers[l], slot, issue);
  }
  if (ok) visit(p, pl, layers[0], kSlotHead, issue);
  return cur.t;
}

// ---- consumers: matvec over the items of one matrix -----------------------------------------

// How the consumer warps cover a matrix of U units per row, fixed for a phase:
//  * rows of at most 32 kJ units: warp w takes RW rows at a time (RW = 4, 2 or 1, the most
//    that fit kJ slots); lane slot j is flat index lane + 32 j of that RW x U (row, unit)
//    space, its activation unit staying in registers, and the RW totals come out of one
//    transposed shuffle tree (reduce_rows) per group -- the launch chain's mv_rows_kernel
//    layout;
//  * longer rows: one row per warp, lane l taking units l, l + 32, ... with the activation
//    read from shared memory.
// Either way an item's row groups are dealt round-robin over the warps, continuing from the
// previous items of the matrix, so consecutive items are worked on by different warps at once.
struct Slots {
  int U, rw, rwl;  // units per row, rows per group and its log2
  bool longrows;
  uint32_t off[kJ];  // byte offset of the slot's row inside a group
  int row[kJ];       // row of the slot inside a group (kNoRow: slot unused)
  int unit[kJ];
  XUnit x[kJ];
};
constexpr int kNoRow = 1 << 20;

__device__ __forceinline__ void make_slots(const TokenStep &p, uint32_t base, int k, uint32_t rb, Slots &s) {
  const int lane = threadIdx.x & 31;
  s.U = k / 32;
  s.longrows = s.U > 32 * kJ;
  s.rw = s.U <= 8 * kJ ? 4 : (s.U <= 16 * kJ ? 2 : 1);
  s.rwl = s.rw == 4 ? 2 : s.rw == 2 ? 1 : 0;
  const int total = s.longrows ? 0 : s.rw * s.U;
#pragma unroll
  for (int j = 0; j < kJ; ++j) {
    const int f = lane + 32 * j;
    const bool valid = f < total;
    const int r = valid ? f / s.U : 0;
    const int u = valid ? f - r * s.U : 0;
    s.row[j] = valid ? r : kNoRow;
    s.unit[j] = u;
    s.off[j] = static_cast<uint32_t>(r) * rb;
    load_xunit(base + p.o_xq + 32 * u, base + p.o_xd + 4 * u, base + p.o_xs + 4 * u, true, s.x[j]);
  }
}

// Short rows: groups of RW rows starting at row `first` * RW, every kCW-th group.
template <int KIND, int RW, class Out>
__device__ __forceinline__ void warp_rows(uint32_t item, int nrows, uint32_t rb, const Slots &s, int row0,
                                          int first, Out &out) {
  const int lane = threadIdx.x & 31;
  for (int g = first * RW; g < nrows; g += kCW * RW) {
    const uint32_t gbase = item + static_cast<uint32_t>(g) * rb;
    // Branch-free over the slots (a branch per slot would serialise their loads): a slot past
    // the item's last row reads unit 0 of the group's first row instead and adds nothing.
    float acc[kJ];
#pragma unroll
    for (int j = 0; j < kJ; ++j) {
      const bool live = g + s.row[j] < nrows;
      WUnit w;
      load_wunit<KIND>(gbase + (live ? s.off[j] : 0u), live ? s.unit[j] : 0, w);
      const float t = unit_term<KIND>(w, s.x[j], unit_isum<KIND>(w, s.x[j]));
      acc[j] = live ? t : 0.f;
    }
    float rs[RW];
#pragma unroll
    for (int r = 0; r < RW; ++r) {
      rs[r] = 0.f;
#pragma unroll
      for (int j = 0; j < kJ; ++j) rs[r] += s.row[j] == r ? acc[j] : 0.f;
    }
    float tot;
    if (reduce_rows<RW>(rs, lane, tot)) {
      const int rr = g + lane / (32 / RW);
      if (rr < nrows) out(row0 + rr, tot);
    }
  }
}

// Long rows: row `first`, first + kCW, ... of the item, one per warp.
template <int KIND, class Out>
__device__ __forceinline__ void warp_rows_long(const TokenStep &p, uint32_t base, uint32_t item, int nrows,
                                               uint32_t rb, int U, int row0, int first, Out &out) {
  const int lane = threadIdx.x & 31;
  for (int g = first; g < nrows; g += kCW) {
    const uint32_t row = item + static_cast<uint32_t>(g) * rb;
    float acc = 0.f;
#pragma unroll 4
    for (int u = lane; u < U; u += 32) {
      WUnit w;
      XUnit x;
      load_wunit<KIND>(row, u, w);
      load_xunit(base + p.o_xq + 32 * u, base + p.o_xd + 4 * u, base + p.o_xs + 4 * u, Fmt<KIND>::kNeedsSum, x);
      acc += unit_term<KIND>(w, x, unit_isum<KIND>(w, x));
    }
    acc = warp_sum(acc);
    if (lane == 0) out(row0 + g, acc);
  }
}

// Consumer warps: take this CTA's items of matrix `slot` from the ring in stream order;
// out(row, value) runs once per row, in the lane that holds the row's total.  Returns false
// when the step was aborted.
template <int KIND, class Out>
__device__ bool consume(const TokenStep &p, uint32_t base, Cursor &cur, const TokPlan &pl, const TokLayer &L,
                        int slot, uint32_t rb, const Slots &s, Out &&out) {
  const uint32_t full = base, empty = base + 8 * kNS, ring = base + p.o_ring;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  bool ok = true;
  int groups = 0;  // row groups of the matrix's earlier items
  visit(p, pl, L, slot, [&](const uint8_t *, uint32_t bytes, int row0, int nrows) {
    if (!ok) return;
    const uint32_t off = cur.place(bytes, p.ring_bytes);
    const uint32_t t = cur.t - 1;
    const uint32_t item = ring + off;
    const int group0 = groups;
    const int ng = (nrows + s.rw - 1) >> s.rwl;  // row groups of the item
    groups += ng;
    const int first = (warp - group0) & (kCW - 1);  // this warp's first group in the item
    // A warp with no group of the item neither waits for it nor releases it: the warp holding
    // the item's group 0 releases it for them as well.  Every release follows a wait on the
    // item, so none can overtake the previous use of the barrier slot (the producer reuses a
    // slot only after seeing its previous item released).
    if (first >= ng) return;
    ok = __all_sync(0xffffffffu, mbar_wait_step(p, full + 8 * (t % kNS), (t / kNS) & 1));
    if (!ok) return;
    if (s.longrows) {
      warp_rows_long<KIND>(p, base, item, nrows, rb, s.U, row0, first, out);
    } else if (s.rw == 4) {
      warp_rows<KIND, 4>(item, nrows, rb, s, row0, first, out);
    } else if (s.rw == 2) {
      warp_rows<KIND, 2>(item, nrows, rb, s, row0, first, out);
    } else {
      warp_rows<KIND, 1>(item, nrows, rb, s, row0, first, out);
    }
    __syncwarp();
    if (lane == 0)
      mbar_arrive_relaxed_n(empty + 8 * (t % kNS), first == 0 ? static_cast<uint32_t>(kCW - min(ng, kCW) + 1) : 1u);
  });
  return ok;
}

// ---- consumers: glue -------------------------------------------------------------------------
//
// Every glue step is a short chain of dependent reads of data other SMs just wrote (L2 round
// trips of ~0.5 us each on the critical path of the token), so each step issues all of its
// global loads before it uses any of them.

constexpr int kMaxEmbdPer = 16;  // n_embd <= 4096 = 16 * 256

// x (shared) += dx (global, written by other CTAs) when dx is given; then the RMSNorm of x times
// w, Q8_1-quantised into the shared activation (fused_resnorm + quant_act, gpu_fused.cu:28-35,
// gpu_dp4a.cu:23-31).  Sum of squares in a fixed order.
// Tracing (CTA 0 only, else rec < 0): the residual, the norm output and its Q8_1 go to fields X,
// ATTN_NORM / FFN_NORM (fn) and the Q8_1 field after it of trace record `rec`.
// dx (tagged words, or null at the first layer): each thread reads its elements until every tag
// is `tag` -- the other CTAs' outputs of the previous phase, all written -- with the step's wait
// limit; false (on every consumer thread) when the step was aborted or the limit passed.
template <bool TRACE>
__device__ bool norm_quant(const TokenStep &p, uint8_t *smem, TokMisc *ms, const unsigned long long *dx,
                           uint32_t tag, const float *w, int rec, int fn) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n = p.n_embd;
  float *x = reinterpret_cast<float *>(smem + p.o_xres);
  constexpr int kPer = kMaxEmbdPer / (kCW / 8);  // elements (and blocks) of x per thread (warp)
  float d[kPer], wv[kPer];
  uint32_t pend = 0;  // elements whose tag is not yet the current one
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int i = tid + k * kCT, b = warp + k * kCW;
    d[k] = 0.f;
    if (dx && i < n) {
      const unsigned long long v = ld_relaxed64(dx + i);
      if (static_cast<uint32_t>(v >> 32) == tag) {
        d[k] = __uint_as_float(static_cast<uint32_t>(v));
      } else {
        pend |= 1u << k;
      }
    }
    wv[k] = b < n / 32 ? w[b * 32 + lane] : 0.f;
  }
  bool ok = true;
  if (pend) {
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 1; pend; ++it) {
#pragma unroll
      for (int k = 0; k < kPer; ++k)
        if (pend & (1u << k)) {
          const unsigned long long v = ld_relaxed64(dx + tid + k * kCT);
          if (static_cast<uint32_t>(v >> 32) == tag) {
            d[k] = __uint_as_float(static_cast<uint32_t>(v));
            pend &= ~(1u << k);
          }
        }
      if (pend && (it & 15) == 0) {
        if (aborted(p)) {
          ok = false;
          break;
        }
        if (globaltimer_ns() - t0 > p.wait_ns) {
          abort_all(p);
          ok = false;
          break;
        }
      }
    }
  }
  // X is the residual entering a layer (or the head): the attention-side norm's input only
  float *tx = TRACE && rec >= 0 && fn == UGB_TRACE_ATTN_NORM ? p.trace.f32(rec, UGB_TRACE_X) : nullptr;
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int i = tid + k * kCT;
    if (i < n) {
      const float v = x[i] + d[k];
      x[i] = v;
      if (TRACE && tx) tx[i] = v;
      ss += v * v;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (lane == 0) ms->red[warp] = ss;
  if (!cbar_and(ok)) return false;
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < kCW; ++i) tot += ms->red[i];
  const float scale = 1.0f / sqrtf(tot / static_cast<float>(n) + p.eps);
  int8_t *q = reinterpret_cast<int8_t *>(smem + p.o_xq);
  float *qd = reinterpret_cast<float *>(smem + p.o_xd);
  int32_t *qs = reinterpret_cast<int32_t *>(smem + p.o_xs);
  bool bad = false;
  constexpr int kQ = 4;  // blocks quantised together
#pragma unroll
  for (int k0 = 0; k0 < kPer; k0 += kQ) {
    if (warp + k0 * kCW < n / 32) {  // warp-uniform
      float v[kQ];
      int b[kQ];
      bool live[kQ];
#pragma unroll
      for (int k = 0; k < kQ; ++k) {
        b[k] = warp + (k0 + k) * kCW;
        live[k] = b[k] < n / 32;
        v[k] = live[k] ? x[b[k] * 32 + lane] * scale * wv[k0 + k] : 0.f;
      }
      bad |= quant_blocks<kQ>(v, b, live, lane, q, qd, qs);
      if (TRACE && rec >= 0) {  // the same arithmetic again, into the trace
        float *tn = p.trace.f32(rec, fn);
        uint8_t *tq = p.trace.at(rec, fn + 1);
#pragma unroll
        for (int k = 0; k < kQ; ++k)
          if (live[k]) tn[b[k] * 32 + lane] = v[k];
        quant_blocks<kQ>(v, b, live, lane, reinterpret_cast<int8_t *>(tq), reinterpret_cast<float *>(tq + p.trace.d_e),
                         reinterpret_cast<int32_t *>(tq + p.trace.s_e));
      }
    }
  }
  if (bad && lane == 0) status_or(p.status, ST_NONFINITE_IN);
  cbar();  // the activation is complete, and ms->red may be reused
  return true;
}

// Ask L2 for the cached keys and values an attention unit of layer l will read (positions before
// pos of its chunk), so phase B finds them there instead of in HBM.  One thread.
template <typename KV>
__device__ __forceinline__ void prefetch_unit(const TokenStep &p, int l, int kvh, int c, int pos) {
  constexpr int HD = kHeadDim;
  const int t0 = c * kAttnChunk;
  const int n_old = min(kAttnChunk, pos - t0);  // the row at pos is written in phase B
  if (n_old <= 0) return;
  const size_t row0 = ((static_cast<size_t>(l) * p.n_kv + kvh) * p.n_ctx + t0) * HD;
  const uint32_t bytes = static_cast<uint32_t>(n_old) * HD * sizeof(KV);
  const KV *k = static_cast<const KV *>(p.kcache) + row0, *v = static_cast<const KV *>(p.vcache) + row0;
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(k), "r"(bytes) : "memory");
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(v), "r"(bytes) : "memory");
}

// One attention unit: KV head kvh, context chunk c (positions [64 c, 64 c + nt)) and query
// subgroup sg (heads [g0, g0 + gn) of the KV head's G, at most kMaxGroup) of layer l -- the
// launch chain's attn_partial_kernel arithmetic (rope_bias, gpu_ops.cu:9-20; fused_attention,
// gpu_attention.cu:2-26) on the consumer threads: the subgroup's query heads biased and
// rotated; the chunk holding `pos` also biases and rotates the new key (subgroup 0 stores it and
// the value in the cache); scores q.k / sqrt(HD); the chunk's max, sum of exp and exp-weighted
// V into the partial buffers.  Splitting the group doubles the CTAs that share the attention
// work.  The subgroup is padded to kMaxGroup heads (zero queries, zero probabilities) so that no
// loop below branches on its size.
constexpr int kMaxGroup = 4;

__host__ __device__ constexpr int attn_subgroups(int G) { return (G + kMaxGroup - 1) / kMaxGroup; }

template <typename KV>
__device__ bool attn_unit(const TokenStep &p, uint8_t *smem, const float *bias, int l, int kvh, int c, int sg,
                          int pos, uint32_t tag) {
  constexpr int HD = kHeadDim, C = kAttnChunk, GM = kMaxGroup;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = p.n_head / p.n_kv, nsg = attn_subgroups(G);
  const int g0 = G * sg / nsg, gn = G * (sg + 1) / nsg - g0;
  const int qr = p.n_head * HD, kr = p.n_kv * HD;
  float *qs = reinterpret_cast<float *>(smem + p.o_scr);  // [GM][HD]
  float *kn = qs + GM * HD;                               // [2][HD] new key, value
  float *ps = kn + 2 * HD;                                // [GM][C]
  float *ored = ps + GM * C;                              // [kPV - 1][GM][HD]
  const int t0 = c * C, nt = min(C, pos + 1 - t0);
  const bool has_new = pos < t0 + C;
  const float2 *rope = p.rope + static_cast<size_t>(pos) * (HD / 2);
  const size_t cache_head = (static_cast<size_t>(l) * p.n_kv + kvh) * p.n_ctx * HD;
  KV *kcache = static_cast<KV *>(p.kcache) + cache_head, *vcache = static_cast<KV *>(p.vcache) + cache_head;
  // Threads [0, GM*64) take rotation pair (g, j) = (tid / 64, tid % 64) of the padded
  // subgroup; in the chunk holding pos, threads [GM*64, GM*64 + 64) take key pair j and the next
  // HD threads one value element each.  Every load is issued before any is used.
  static_assert(GM * HD / 2 + HD / 2 + HD <= kCT, "attention load layout");
  // The chunk's cached keys (scores: 8 lanes per position, lane j of a group takes float4
  // columns j, j+8, j+16, j+24, 4 positions per warp) and values (P.V: thread (dd, sl) takes
  // positions tl = sl, sl + kPV, ... of output dimension dd), requested first: they do not
  // depend on this step's Q/K/V rows, so both round trips overlap.  The row at pos is not in the
  // cache yet; the new key replaces it below and P.V takes the new value.
  const float inv_sqrt = 1.0f / sqrtf(static_cast<float>(HD));
  const int sub = lane & 7, grp = lane >> 3;
  constexpr int kPass = C / (kCW * 4);
  static_assert(kPass * kCW * 4 == C, "score passes");
  const int dd = tid & (HD - 1), sl = tid / HD;
  float4 k4[kPass][4];
#pragma unroll
  for (int ps_i = 0; ps_i < kPass; ++ps_i) {
    const int tl = (ps_i * kCW + warp) * 4 + grp, t = t0 + min(tl, nt - 1);
    const KV *row = kcache + static_cast<size_t>(t) * HD;
#pragma unroll
    for (int i = 0; i < 4; ++i) k4[ps_i][i] = KvIO<KV>::load4(row + 4 * (sub + 8 * i));
  }
  float vv[C / kPV];
#pragma unroll
  for (int m = 0; m < C / kPV; ++m) {
    const int tl = min(sl + kPV * m, nt - 1), t = t0 + tl;
    vv[m] = KvIO<KV>::load(vcache + static_cast<size_t>(t) * HD + dd);
  }
  bool ok = true;  // the Q/K/V rows arrive as tagged words, read until current (bounded)
  if (tid < GM * HD / 2) {
    const int g = tid / (HD / 2), j = tid % (HD / 2);
    const int qrow = (kvh * G + g0 + min(g, gn - 1)) * HD + j;
    const float b0 = bias ? bias[qrow] : 0.f, b1 = bias ? bias[qrow + HD / 2] : 0.f;
    const float q0 = poll_tagged(p, p.tqkv + qrow, tag, ok) + b0, q1 = poll_tagged(p, p.tqkv + qrow + HD / 2, tag, ok) + b1;
    const float2 cs = rope[j];
    const bool live = g < gn;
    qs[g * HD + j] = live ? q0 * cs.x - q1 * cs.y : 0.f;
    qs[g * HD + j + HD / 2] = live ? q0 * cs.y + q1 * cs.x : 0.f;
  } else if (has_new && tid < GM * HD / 2 + HD / 2) {
    const int j = tid - GM * HD / 2, krow = qr + kvh * HD + j;
    const float b0 = bias ? bias[krow] : 0.f, b1 = bias ? bias[krow + HD / 2] : 0.f;
    const float k0 = poll_tagged(p, p.tqkv + krow, tag, ok) + b0, k1 = poll_tagged(p, p.tqkv + krow + HD / 2, tag, ok) + b1;
    const float2 cs = rope[j];
    // the new row takes part as the cache holds it (rounded to fp16 in an fp16 cache)
    const float a = KvIO<KV>::round(k0 * cs.x - k1 * cs.y), b = KvIO<KV>::round(k0 * cs.y + k1 * cs.x);
    kn[j] = a;
    kn[j + HD / 2] = b;
    if (sg == 0) {
      KvIO<KV>::store(kcache + static_cast<size_t>(pos) * HD + j, a);
      KvIO<KV>::store(kcache + static_cast<size_t>(pos) * HD + j + HD / 2, b);
    }
  } else if (has_new && tid < GM * HD / 2 + HD / 2 + HD) {
    const int dd = tid - GM * HD / 2 - HD / 2, vrow = qr + kr + kvh * HD + dd;
    const float v = KvIO<KV>::round(poll_tagged(p, p.tqkv + vrow, tag, ok) + (bias ? bias[vrow] : 0.f));
    kn[HD + dd] = v;
    if (sg == 0) KvIO<KV>::store(vcache + static_cast<size_t>(pos) * HD + dd, v);
  }
  if (!cbar_and(ok)) return false;
  // Scores of all padded heads (zero queries score 0 and are not stored).
#pragma unroll
  for (int ps_i = 0; ps_i < kPass; ++ps_i) {  // the row at pos: the new key (all rows of kn now written)
    const int tl = (ps_i * kCW + warp) * 4 + grp, t = t0 + min(tl, nt - 1);
    if (t == pos) {
      const float4 *own = reinterpret_cast<const float4 *>(kn);
#pragma unroll
      for (int i = 0; i < 4; ++i) k4[ps_i][i] = own[sub + 8 * i];
    }
  }
#pragma unroll
  for (int ps_i = 0; ps_i < kPass; ++ps_i) {
    const int tl = (ps_i * kCW + warp) * 4 + grp;
#pragma unroll
    for (int g = 0; g < GM; ++g) {
      const float4 *q4 = reinterpret_cast<const float4 *>(qs + g * HD);
      float dot = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float4 a = q4[sub + 8 * i];
        dot += a.x * k4[ps_i][i].x + a.y * k4[ps_i][i].y + a.z * k4[ps_i][i].z + a.w * k4[ps_i][i].w;
      }
      dot += __shfl_xor_sync(0xffffffffu, dot, 1);
      dot += __shfl_xor_sync(0xffffffffu, dot, 2);
      dot += __shfl_xor_sync(0xffffffffu, dot, 4);
      if (sub == 0) ps[g * C + tl] = tl < nt && g < gn ? dot * inv_sqrt : 0.f;
    }
  }
  cbar();
  const size_t part = static_cast<size_t>(kvh) * p.n_split + c;
  if (warp < gn) {
    float mx = -FLT_MAX;
    for (int t = lane; t < nt; t += 32) mx = fmaxf(mx, ps[warp * C + t]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.f;
    for (int t = lane; t < nt; t += 32) {
      const float e = expf(ps[warp * C + t] - mx);
      ps[warp * C + t] = e;
      sum += e;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) {
      p.part_m[part * G + g0 + warp] = mx;
      p.part_l[part * G + g0 + warp] = sum;
    }
  }
  cbar();
  float acc[GM];
#pragma unroll
  for (int g = 0; g < GM; ++g) acc[g] = 0.f;
  const float vnew = kn[HD + dd];
#pragma unroll
  for (int m = 0; m < C / kPV; ++m) {
    const int tl = sl + kPV * m;
    const bool live = tl < nt;
    const float v = live ? (t0 + tl == pos ? vnew : vv[m]) : 0.f;
#pragma unroll
    for (int g = 0; g < GM; ++g) acc[g] += ps[g * C + min(tl, C - 1)] * v;
  }
  if (sl > 0)
#pragma unroll
    for (int g = 0; g < GM; ++g) ored[((sl - 1) * GM + g) * HD + dd] = acc[g];
  cbar();
  if (sl == 0)
#pragma unroll
    for (int g = 0; g < GM; ++g) {
      float o = acc[g];
#pragma unroll
      for (int q = 1; q < kPV; ++q) o += ored[((q - 1) * GM + g) * HD + dd];
      if (g < gn) p.part_o[(part * G + g0 + g) * HD + dd] = o;
    }
  cbar();  // the scratch is free for the next unit
  return true;
}

// The attention unit just finished (KV head kvh, subgroup sg, one of nch chunks) takes its
// subgroup's ticket; the last of the nch units to do so combines the subgroup's chunk partials
// (log-sum-exp: weights exp(m_c - max), the launch chain's attn_combine_quant_kernel arithmetic
// and order) and writes the gn heads' attention output, quantised per 32-block, as tagged
// words into p.tatt.  Phase C of every CTA then reads that vector (by its tags) instead of
// combining all heads itself.  Tracing (rec >= 0): the unit writes its heads' slice of fields ATT and ATT_XQ.
template <bool TRACE>
__device__ void attn_finish(const TokenStep &p, uint8_t *smem, TokMisc *ms, int kvh, int sg, int nch, uint32_t tag,
                            int rec) {
  constexpr int HD = kHeadDim, GM = kMaxGroup;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = p.n_head / p.n_kv, nsg = attn_subgroups(G);
  const int g0 = G * sg / nsg, gn = G * (sg + 1) / nsg - g0;
  if (tid == 0) {
    uint32_t *ticket = p.sync + kTicket0 + kvh * nsg + sg;
    uint32_t t;
    // acq_rel: this CTA's partials (ordered before by the unit's last consumer barrier) are
    // published with the ticket, and the last unit sees every other unit's
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(t) : "l"(ticket) : "memory");
    ms->last = t + 1 == static_cast<uint32_t>(nch) ? 1 : 0;
    if (ms->last) atomicExch(ticket, 0u);  // ready for the next layer's units
  }
  cbar();
  if (!ms->last) return;
  const int ns = nch;
  float *cw = reinterpret_cast<float *>(smem + p.o_scr);  // [GM][ns] chunk weights
  float *den = cw + GM * ns;                              // [GM] 1 / denominator
  // thread (w, d) = (tid / HD, tid % HD) of the gn heads; a warp holds one 32-block of one head.
  // Its first chunk outputs are requested now, with the maxima and sums below, so the two loads
  // share one round trip.
  const bool owner = tid < gn * HD;
  const int w = tid / HD, d = tid % HD;
  const size_t obase = (static_cast<size_t>(kvh) * p.n_split * G + g0 + w) * HD + d;
  constexpr int kBatch = 8;  // chunk loads in flight together
  float pv[kBatch];
#pragma unroll
  for (int j = 0; j < kBatch; ++j)
    pv[j] = owner ? __ldcg(p.part_o + obase + static_cast<size_t>(min(j, ns - 1)) * G * HD) : 0.f;
  if (warp < gn) {
    const size_t p0 = static_cast<size_t>(kvh) * p.n_split * G + g0 + warp;
    const bool one = lane < ns;
    const float m1 = one ? __ldcg(p.part_m + p0 + static_cast<size_t>(lane) * G) : -FLT_MAX;
    const float l1 = one ? __ldcg(p.part_l + p0 + static_cast<size_t>(lane) * G) : 0.f;
    float mx = m1;
    for (int sp = lane + 32; sp < ns; sp += 32) mx = fmaxf(mx, __ldcg(p.part_m + p0 + static_cast<size_t>(sp) * G));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float l = 0.f;
    if (one) {
      const float e = expf(m1 - mx);
      cw[warp * ns + lane] = e;
      l = e * l1;
    }
    for (int sp = lane + 32; sp < ns; sp += 32) {
      const size_t pi = p0 + static_cast<size_t>(sp) * G;
      const float e = expf(__ldcg(p.part_m + pi) - mx);
      cw[warp * ns + sp] = e;
      l += e * __ldcg(p.part_l + pi);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    if (lane == 0) den[warp] = 1.0f / l;
  }
  cbar();
  bool bad = false;
  if (owner) {
    float o = 0.f;
    for (int s0 = 0; s0 < ns; s0 += kBatch) {
      if (s0 > 0) {
#pragma unroll
        for (int j = 0; j < kBatch; ++j)
          pv[j] = __ldcg(p.part_o + obase + static_cast<size_t>(min(s0 + j, ns - 1)) * G * HD);
      }
#pragma unroll
      for (int j = 0; j < kBatch; ++j)
        if (s0 + j < ns) o += cw[w * ns + s0 + j] * pv[j];
    }
    const float v = o * den[w];
    const int blk = ((kvh * G + g0 + w) * HD + d) >> 5;
    bad = quant_block_tagged(v, lane, p.tatt + blk * kQ8TagWords, tag);
    if (TRACE && rec >= 0) {  // the same arithmetic again, into the trace
      uint8_t *tq = p.trace.at(rec, UGB_TRACE_ATT_XQ);
      p.trace.f32(rec, UGB_TRACE_ATT)[blk * 32 + lane] = v;
      quant_block(v, lane, reinterpret_cast<int8_t *>(tq), reinterpret_cast<float *>(tq + p.trace.d_q),
                  reinterpret_cast<int32_t *>(tq + p.trace.s_q), blk);
    }
  }
  if (bad && lane == 0) status_or(p.status, ST_NONFINITE_IN);
  cbar();  // the scratch is free for the next unit
}

// Every consumer thread: nb tagged Q8_1 blocks at w (written by other CTAs) into the shared
// activation, each word read until its tag is `tag`; false (on every consumer thread) when the
// step was aborted or the wait limit passed.  Words go in passes of kPer per thread, all of a
// pass in flight together.
__device__ bool load_q8_tagged(const TokenStep &p, uint8_t *smem, const unsigned long long *w, int nb, uint32_t tag) {
  const int tid = threadIdx.x;
  uint8_t *q = smem + p.o_xq;
  float *dd = reinterpret_cast<float *>(smem + p.o_xd);
  int32_t *ds = reinterpret_cast<int32_t *>(smem + p.o_xs);
  const int nw = nb * kQ8TagWords;
  constexpr int kPer = 8;
  bool ok = true;
  for (int i0 = 0; i0 < nw && ok; i0 += kPer * kCT) {
    unsigned long long v[kPer];
    uint32_t pend = 0;
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int i = i0 + k * kCT + tid;
      v[k] = i < nw ? ld_relaxed64(w + i) : 0ull;
      if (i < nw && static_cast<uint32_t>(v[k] >> 32) != tag) pend |= 1u << k;
    }
    if (pend) {
      const uint64_t t0 = globaltimer_ns();
      for (uint32_t it = 1; pend; ++it) {
#pragma unroll
        for (int k = 0; k < kPer; ++k)
          if (pend & (1u << k)) {
            v[k] = ld_relaxed64(w + i0 + k * kCT + tid);
            if (static_cast<uint32_t>(v[k] >> 32) == tag) pend &= ~(1u << k);
          }
        if (pend && (it & 15) == 0) {
          if (aborted(p)) {
            ok = false;
            break;
          }
          if (globaltimer_ns() - t0 > p.wait_ns) {
            abort_all(p);
            ok = false;
            break;
          }
        }
      }
    }
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int i = i0 + k * kCT + tid;
      if (i >= nw) continue;
      const int b = i / kQ8TagWords, j = i - b * kQ8TagWords;
      const uint32_t bits = static_cast<uint32_t>(v[k]);
      if (j < 8) {
        *reinterpret_cast<uint32_t *>(q + b * 32 + 4 * j) = bits;
      } else if (j == 8) {
        dd[b] = __uint_as_float(bits);
      } else {
        ds[b] = static_cast<int32_t>(bits);
      }
    }
  }
  return cbar_and(ok);
}

// The CTA's FFN blocks [b0, b1): h = SiLU(gate) * up (gateup_dp4a epilogue, gpu_dp4a.cu:63) from
// the shared gate / up rows, quantised per 32-block into the global hq buffer.
// Tracing (rec >= 0): every CTA writes its blocks of fields H and H_XQ of record rec.
template <bool TRACE>
__device__ void silu_quant(const TokenStep &p, uint8_t *smem, int b0, int b1, uint32_t tag, int rec) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float *gs = reinterpret_cast<const float *>(smem + p.o_gu);
  const float *us = gs + 32 * p.gu_blocks;
  bool bad = false;
  for (int b = b0 + warp; b < b1; b += kCW) {
    const int i = (b - b0) * 32 + lane;
    const float gv = gs[i], uv = us[i];
    const float h = (gv / (1.0f + expf(-gv))) * uv;
    bad |= quant_block_tagged(h, lane, p.thq + b * kQ8TagWords, tag);
    if (TRACE && rec >= 0) {  // the same arithmetic again, into the trace
      uint8_t *tq = p.trace.at(rec, UGB_TRACE_H_XQ);
      p.trace.f32(rec, UGB_TRACE_H)[b * 32 + lane] = h;
      quant_block(h, lane, reinterpret_cast<int8_t *>(tq), reinterpret_cast<float *>(tq + p.trace.d_f),
                  reinterpret_cast<int32_t *>(tq + p.trace.s_f), b);
    }
  }
  if (bad && lane == 0) status_or(p.status, ST_NONFINITE_IN);
}


// ---- the consumers' step -------------------------------------------------------------------

// Returns when the step is done or aborted; ms->consumed is not needed (the drain works from
// the producer's count).
template <int KIND, int HKIND, typename KV, bool TRACE>
__device__ void consumers(const TokenStep &p, uint8_t *smem, uint32_t base, TokMisc *ms, const TokLayer *layers) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int P = gridDim.x, cta = blockIdx.x;
  const uint32_t Pu = static_cast<uint32_t>(P);
  // Token and position: the previous step's greedy key when there is one, else the host's
  // token (embed_kernel's rule).  Every CTA reads the state; CTA 0 rewrites it once all have.
  if (tid == 0) {
    const unsigned long long key = __ldcg(&p.state->key[0]);
    int tok = key != 0 ? static_cast<int>(key_id(key)) : __ldcg(&p.state->token[0]);
    int pos = __ldcg(&p.state->pos) + (key != 0 ? 1 : 0);
    if (pos < 0 || pos >= p.n_ctx) {
      if (cta == 0) status_or(p.status, ST_BADARG);
      pos = pos < 0 ? 0 : p.n_ctx - 1;
    }
    if (tok < 0 || tok >= p.n_vocab) {
      if (cta == 0) status_or(p.status, ST_BADARG);
      tok = 0;
    }
    ms->tok = tok;
    ms->pos = pos;
    ms->epoch = ld_relaxed(p.sync + kEpochWord);
    atomicAdd(sync_word(p, kStart), 1u);
    ms->ok = 1;
    if (cta == 0) {
      if (spin_until(p, kStart, Pu)) {
        p.state->token[0] = tok;
        p.state->pos = pos;
        p.state->key[0] = 0;  // ordered before every CTA's head atomicMax by the phase counters
      } else {
        ms->ok = 0;
      }
    }
  }
  cbar();
  const int pos = ms->pos, tok = ms->tok;
  const uint32_t epoch = ms->epoch;
  unsigned long long *const tdx_o = p.tdx, *const tdx_d = p.tdx + p.n_embd;
  if (!cbar_and(ms->ok != 0)) return;
  float *x = reinterpret_cast<float *>(smem + p.o_xres);
  {  // x = the token's Q8_0 embedding row (embedding_q8, gpu_embedding.cu:3-9)
    const uint8_t *row = p.tok_embd + static_cast<uint64_t>(tok) * p.rb_tok;
    for (int i = tid; i < p.n_embd; i += kCT) {
      const uint8_t *blk = row + (i / 32) * 34;
      const uint32_t h = blk[0] | (static_cast<uint32_t>(blk[1]) << 8);
      x[i] = half_bits_to_float(h) * static_cast<float>(static_cast<int8_t>(blk[2 + (i & 31)]));
    }
  }
  cbar();
  const int qr = p.n_head * kHeadDim;
  const int nch = pos / kAttnChunk + 1;
  const int nsg = attn_subgroups(p.n_head / p.n_kv);
  const int units = p.n_kv * nch * nsg;  // (KV head, chunk, query subgroup)
  const TokPlan &pl = ms->plan;
  const int gb0 = pl.gb0, gb1 = pl.gb1;  // this CTA's FFN blocks
  float *gs = reinterpret_cast<float *>(smem + p.o_gu);
  float *us = gs + 32 * p.gu_blocks;
  Cursor cur;
  Slots sl;
  uint32_t *status = p.status;
  constexpr bool tracing = TRACE;
  const bool tr0 = TRACE && cta == 0;  // replicated values are traced by CTA 0
  for (int l = 0; l < p.n_layer; ++l) {
    const TokLayer &L = layers[l];
    // A: residual + norm + Q8_1, then Q/K/V
    // (the previous layer's down outputs are waited for inside the norm, by their tags)
    if (tid == 0)
      for (int u = cta; u < units; u += P)
        if (u % nsg == 0) prefetch_unit<KV>(p, l, u / nsg / nch, u / nsg % nch, pos);
    if (!norm_quant<TRACE>(p, smem, ms, l > 0 ? tdx_d : nullptr, dx_tag(epoch, l - 1), L.attn_norm, tr0 ? l : -1,
                           UGB_TRACE_ATTN_NORM))
      return;
    make_slots(p, base, p.n_embd, p.rb_e, sl);
    bool ok = consume<KIND>(p, base, cur, pl, L, kSlotQKV, p.rb_e, sl, [&](int row, float v) {
      st_tagged(p.tqkv + row, v, dx_tag(epoch, l));
      if (tracing) p.trace.f32(l, UGB_TRACE_QKV)[row] = v;
      if (!isfinite(v)) status_or(status, ST_NONFINITE_OUT);
    });
    if (!cbar_and(ok)) return;
    // B: attention partials
    // (no device-wide wait: a unit reads its Q/K/V rows by their tags)
    if (cta < units) {
      for (int u = cta; u < units; u += P) {
        if (!attn_unit<KV>(p, smem, L.bias, l, u / nsg / nch, u / nsg % nch, u % nsg, pos, dx_tag(epoch, l))) return;
        attn_finish<TRACE>(p, smem, ms, u / nsg / nch, u % nsg, nch, dx_tag(epoch, l), TRACE ? l : -1);
      }
    }
    // C: the quantised attention output (by its tags), then O.  p.unreachable > 0 (a test hook)
    // makes the first layer wait for a tag no CTA writes, so the wait ends only by its time limit.
    if (!load_q8_tagged(p, smem, p.tatt, qr / 32, dx_tag(epoch, l) ^ (l == 0 && p.unreachable ? 0x80000000u : 0u)))
      return;
    make_slots(p, base, qr, p.rb_q, sl);
    ok = consume<KIND>(p, base, cur, pl, L, kSlotO, p.rb_q, sl, [&](int row, float v) {
      st_tagged(tdx_o + row, v, dx_tag(epoch, l));
      if (tracing) p.trace.f32(l, UGB_TRACE_O)[row] = v;
      if (!isfinite(v)) status_or(status, ST_NONFINITE_OUT);
    });
    if (!cbar_and(ok)) return;
    // D: residual + norm + Q8_1, then gate and up of whole blocks, SiLU * up + Q8_1
    if (!norm_quant<TRACE>(p, smem, ms, tdx_o, dx_tag(epoch, l), L.ffn_norm, tr0 ? l : -1, UGB_TRACE_FFN_NORM))
      return;
    make_slots(p, base, p.n_embd, p.rb_e, sl);
    ok = consume<KIND>(p, base, cur, pl, L, kSlotGate, p.rb_e, sl, [&](int row, float v) {
      gs[row - 32 * gb0] = v;
      if (tracing) p.trace.f32(l, UGB_TRACE_GATE_UP)[row] = v;
      if (!isfinite(v)) status_or(status, ST_NONFINITE_OUT);
    });
    ok = consume<KIND>(p, base, cur, pl, L, kSlotUp, p.rb_e, sl, [&](int row, float v) {
      us[row - 32 * gb0] = v;
      if (tracing) p.trace.f32(l, UGB_TRACE_GATE_UP)[p.n_ff + row] = v;
      if (!isfinite(v)) status_or(status, ST_NONFINITE_OUT);
    }) && ok;
    if (!cbar_and(ok)) return;
    silu_quant<TRACE>(p, smem, gb0, gb1, dx_tag(epoch, l), TRACE ? l : -1);
    // E: hq (by its tags), then down
    if (!load_q8_tagged(p, smem, p.thq, p.n_ff / 32, dx_tag(epoch, l))) return;
    make_slots(p, base, p.n_ff, p.rb_f, sl);
    ok = consume<KIND>(p, base, cur, pl, L, kSlotDown, p.rb_f, sl, [&](int row, float v) {
      st_tagged(tdx_d + row, v, dx_tag(epoch, l));
      if (tracing) p.trace.f32(l, UGB_TRACE_DOWN)[row] = v;
      if (!isfinite(v)) status_or(status, ST_NONFINITE_OUT);
    });
    if (!cbar_and(ok)) return;
  }
  // Head: residual + output norm + Q8_1, logits of this CTA's rows, greedy key.
  if (!norm_quant<TRACE>(p, smem, ms, tdx_d, dx_tag(epoch, p.n_layer - 1), p.out_norm, tr0 ? p.n_layer : -1,
                         UGB_TRACE_ATTN_NORM))
    return;
  make_slots(p, base, p.n_embd, p.rb_h, sl);
  unsigned long long best = 0;
  const bool ok = consume<HKIND>(p, base, cur, pl, layers[0], kSlotHead, p.rb_h, sl, [&](int row, float v) {
    p.logits[row] = v;
    if (isfinite(v)) {
      best = max(best, static_cast<unsigned long long>(greedy_key(v, static_cast<uint32_t>(row))));
    } else {
      status_or(status, ST_NONFINITE_OUT);
    }
  });
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) best = max(best, __shfl_xor_sync(0xffffffffu, best, o));
  if (lane == 0) ms->key[warp] = best;
  if (!cbar_and(ok)) return;
  if (tid == 0) {
    unsigned long long b = 0;
    for (int w = 0; w < kCW; ++w) b = max(b, ms->key[w]);
    if (b) atomicMax(&p.state->key[0], b);
  }
}

template <int KIND, int HKIND, typename KV, bool TRACE>
__global__ void __launch_bounds__(kTT, 1) token_kernel(const TokenStep p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t base = smem_u32(smem);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  TokMisc *ms = reinterpret_cast<TokMisc *>(smem + 16 * kNS);
  TokLayer *layers = reinterpret_cast<TokLayer *>(smem + p.o_layers);
  if (tid == 0) {
    for (int s = 0; s < kNS; ++s) {
      mbar_init(base + 8 * s, 1);             // full: the producer's expect_tx + the copy
      mbar_init(base + 8 * (kNS + s), kCW);   // empty: one arrive per consumer warp
    }
    fence_mbar_init();
    ms->issued = 0;
    make_plan(p, ms->plan);
  }
  {  // the layer table into shared memory (read by every matrix of the step)
    static_assert(sizeof(TokLayer) % 8 == 0, "layer table copied as 64-bit words");
    const uint64_t *src = reinterpret_cast<const uint64_t *>(p.layers);
    uint64_t *dst = reinterpret_cast<uint64_t *>(layers);
    const int words = p.n_layer * static_cast<int>(sizeof(TokLayer) / 8);
    for (int i = tid; i < words; i += kTT) dst[i] = src[i];
  }
  __syncthreads();
  if (warp == kCW) {
    if (lane == 0) ms->issued = produce(p, base, ms->plan, layers);
    __syncwarp();
  } else {
    consumers<KIND, HKIND, KV, TRACE>(p, smem, base, ms, layers);
  }
  __syncthreads();
  if (tid == 0) {
    // Copies still in flight (an aborted step) land before the CTA leaves.
    const uint32_t n = ms->issued;
    for (uint32_t t = n > kNS ? n - kNS : 0; t < n; ++t)
      if (!mbar_wait_bounded(base + 8 * (t % kNS), (t / kNS) & 1)) status_or(p.status, ST_TIMEOUT);
    __threadfence();
    if (atomicAdd(sync_word(p, kExit), 1u) == gridDim.x - 1) {
      for (int i = 0; i < kNumSync; ++i) sync_word(p, i)[0] = 0;  // ready for the next launch
      for (int i = 0; i < kMaxTickets; ++i) p.sync[kTicket0 + i] = 0;  // (an aborted step may leave some)
      p.sync[kEpochWord] += 1;  // a new tag space for the next launch
      __threadfence();
    }
  }
}

}  // namespace

// ---- host ------------------------------------------------------------------------------------

namespace {

// Shared-memory layout of one CTA; false when it does not fit.
bool token_layout(const ugb_ctx *ctx, TokenStep &p) {
  const int qr = p.n_head * kHeadDim;
  const int kq = std::max({p.n_embd, qr, p.n_ff});
  const size_t xq_bytes = kq + 8 * static_cast<size_t>(kq / 32);
  const size_t attn = 4 * static_cast<size_t>(kPV * kMaxGroup * kHeadDim + 2 * kHeadDim + kMaxGroup * kAttnChunk);
  const size_t comb = 4 * static_cast<size_t>(kMaxGroup * p.n_split + kMaxGroup);  // attn_finish
  p.gu_blocks = (p.n_ff / 32 + ctx->sm_count - 1) / ctx->sm_count;
  size_t o = 16 * kNS + kMiscBytes;
  p.o_xres = static_cast<uint32_t>(o);
  o += round_up(4 * static_cast<size_t>(p.n_embd), 16);
  p.o_xq = static_cast<uint32_t>(o);
  p.o_xd = static_cast<uint32_t>(o + kq);
  p.o_xs = static_cast<uint32_t>(o + kq + 4 * (kq / 32));
  o += round_up(xq_bytes, 16);
  p.o_scr = static_cast<uint32_t>(o);  // attention unit and combine scratch
  o += round_up(std::max(attn, comb), 16);
  p.o_layers = static_cast<uint32_t>(o);  // the layer table
  o += round_up(sizeof(TokLayer) * static_cast<size_t>(p.n_layer), 16);
  p.o_gu = static_cast<uint32_t>(o);
  o += round_up(2 * 32 * 4 * static_cast<size_t>(p.gu_blocks), 16);
  o = round_up(o, 128);
  p.o_ring = static_cast<uint32_t>(o);
  // kRingSlack bytes after the ring: a Q8_0 unit is read as a 40-byte window from 8-byte
  // alignment, up to 6 bytes past the last unit of an item placed at the ring's end.
  if (ctx->smem_optin < o + 2 * kTokItemMax + kRingSlack) return false;
  p.ring_bytes = static_cast<uint32_t>((ctx->smem_optin - o - kRingSlack) & ~size_t(15));
  return true;
}

template <int KIND, int HKIND, typename KV>
ugb_status launch_kind(ugb_ctx *ctx, cudaStream_t stream, const TokenStep &p, size_t smem) {
  // a traced step runs its own instantiation: the trace stores stay out of the untraced kernel
  auto *k = p.trace.base ? token_kernel<KIND, HKIND, KV, true> : token_kernel<KIND, HKIND, KV, false>;
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) != cudaSuccess)
    return UGB_EBACKEND;
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, kTT, smem) != cudaSuccess || per_sm < 1)
    return UGB_ESHAPE;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(ctx->sm_count);
  cfg.blockDim = dim3(kTT);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident at once (they wait on each other)
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, k, p));
}

}  // namespace

bool token_supported(const ugb_ctx *ctx, uint32_t kind, uint32_t head_kind, TokenStep p) {
  if ((kind != UGB_Q8_0 && kind != UGB_Q4_K) || head_kind != UGB_Q8_0) return false;
  if (p.n_head % p.n_kv || p.n_head / p.n_kv > 8 || p.n_embd % 32 || p.n_ff % 32) return false;
  // one combine ticket per (KV head, subgroup)
  if (p.n_kv * attn_subgroups(p.n_head / p.n_kv) > kMaxTickets) return false;
  if (p.n_embd > 4096 || p.n_layer > kMaxTokLayers)
    return false;
  const uint32_t rbs[4] = {p.rb_e, p.rb_q, p.rb_f, p.rb_h};
  for (uint32_t rb : rbs)
    if (rb == 0 || rb % 16 || rb > kTokItemMax) return false;
  return token_layout(ctx, p);
}

ugb_status launch_token(ugb_ctx *ctx, cudaStream_t stream, uint32_t kind, uint32_t head_kind, TokenStep p) {
  if (!token_supported(ctx, kind, head_kind, p)) return UGB_ESHAPE;
  token_layout(ctx, p);
  const size_t smem = p.o_ring + p.ring_bytes + kRingSlack;
  if (kind == UGB_Q8_0)
    return p.kv16 ? launch_kind<UGB_Q8_0, UGB_Q8_0, __half>(ctx, stream, p, smem)
                  : launch_kind<UGB_Q8_0, UGB_Q8_0, float>(ctx, stream, p, smem);
  return p.kv16 ? launch_kind<UGB_Q4_K, UGB_Q8_0, __half>(ctx, stream, p, smem)
                : launch_kind<UGB_Q4_K, UGB_Q8_0, float>(ctx, stream, p, smem);
}

}  // namespace ugb
