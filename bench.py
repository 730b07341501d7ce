"""Benchmark of the B200 quantized decode hot path (libugb) -- one JSON line on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload c2|c1]

Workloads:
  c2  (default; the headline) greedy batch-1 decode of a random-init Qwen2.5-1.5B-shaped
      decoder with every linear weight in Q8_0 (28 layers, hidden 1536, FFN 8960, 12/2 heads
      of 128, vocab 151936, tied embeddings, context 512).  A step is one token: embedding,
      28 layers of norm+quant / QKV / attention / O / norm+quant / gate+up / SiLU+quant / down,
      final norm, head and greedy selection, replayed from one captured CUDA graph with the
      token state kept on the device.  The timed tokens are the last K positions of the
      512-position context.  1.655 GB of weights stream from HBM per token (> L2).
  c1  Q8_0 matvec 8960x1536 with block-32 activation quantisation; weights
      rotate over 24 copies (350 MB > L2).
  c4  greedy decode of a Qwen2.5-7B-shaped model, Q4_K weights, batch 1 / 4 / 8 (--batch),
      context 1024; under torchrun the head rows are split over the GPUs (config 4).
  c5  greedy decode of a 48-layer MoE (192 Q3_K experts, top-8), batch 1 / 8, context 2048;
      under torchrun the experts are split over the GPUs (config 5).
  c3  the linear layers of a 512-token Q8 prefill of the same model (config 3): per layer the
      fused Q/K/V, O, fused gate/up and down GEMMs, each a block-32 activation quant plus the
      tcgen05 INT8 GEMM; weights repacked once outside timing (as the reference does).

Multi-GPU: one process per GPU (torchrun), each an independent replica ("replicas only":
batch-1 decode of a dense model has no exchange step worth sharding); value = all ranks'
tokens / the slowest rank's time (max over ranks of CUDA-event time).

The reference arm (--impl reference) times the CPU restatement of the reference path
(oracle/; the reference Rust cannot be built here) on the host cores with all threads, on
the same workload, metric and unit.
"""
from __future__ import annotations

import argparse
import importlib
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

Q8_0 = 8
PATHS = {"auto": 0, "chain": 1, "token": 2}  # ugb_decoder_set_path values
KV_TYPES = {"f32": 0, "f16": 1}  # ugb_decoder_config.kv_type


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def load_traffic(key):
    """Per-launch DRAM bytes of the dominant kernel from the committed ncu summary."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    if not os.path.exists(path):
        return None
    with open(path) as f:
        return json.load(f).get(key)


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 20 ms from the start of the warm-up to
    the end of the timed region (the GPU is busy with the benchmark throughout)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.out = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "20"],
                stdout=self.out, stderr=subprocess.DEVNULL)
        except (FileNotFoundError, OSError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.out.flush()
        self.out.seek(0)
        rows = [r.split(",") for r in self.out.read().strip().splitlines() if r.strip()]
        os.unlink(self.out.name)
        sm, smax, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                smax = max(smax, float(r[2]))
                for n, v in zip(names, r[5:9]):
                    if v.strip().lower() == "active":
                        reasons.add(n)
            except (ValueError, IndexError):
                continue
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


def barrier(world, torch):
    if world > 1:
        torch.distributed.barrier()


def reduce_max(v: float, world: int, torch) -> float:
    if world == 1:
        return v
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


# ---- workload c2: Qwen2.5-1.5B-shaped Q8_0 decode ------------------------------------------

C2 = dict(n_layer=28, n_embd=1536, n_ff=8960, n_head=12, n_head_kv=2, head_dim=128, n_vocab=151936,
          n_ctx=512, rope_theta=1e6, norm_eps=1e-6, kind=Q8_0, head_kind=Q8_0)


def c2_shapes(c=C2):
    """(name, k, m) of every Q8_0 matrix of one layer (GGUF blk.N.* tensors)."""
    q, kv = c["n_head"] * c["head_dim"], c["n_head_kv"] * c["head_dim"]
    e, f = c["n_embd"], c["n_ff"]
    return [("wq", e, q), ("wk", e, kv), ("wv", e, kv), ("wo", q, e),
            ("w_gate", e, f), ("w_up", e, f), ("w_down", f, e)]


def q8_bytes(k, m):
    return m * (k // 32) * 34


def kv_elem_bytes(c):
    return 2 if c.get("kv_type", 0) == 1 else 4


def c2_token_bytes(c=C2, pos=None):
    """Algorithmic bytes of one token: every weight once (layers + tied head, the embedding row
    is 1.6 KB), plus the KV cache read at context `pos` (K and V of every layer, fp16 or fp32)."""
    layers = c["n_layer"] * sum(q8_bytes(k, m) for _, k, m in c2_shapes(c))
    head = q8_bytes(c["n_embd"], c["n_vocab"])
    if pos is None:
        pos = c["n_ctx"]
    kv = c["n_layer"] * 2 * c["n_head_kv"] * c["head_dim"] * kv_elem_bytes(c) * pos
    return layers + head + kv


def c2_launches_per_token(c=C2):
    # embed; per layer: rmsnorm+quant, QKV, attention partial, attention combine+quant, O,
    # rmsnorm+quant, gate/up, SiLU+quant, down; final rmsnorm+quant, head, greedy
    return 1 + 9 * c["n_layer"] + 3


def c2_device_weights(ctx, ugb, torch, seed, c=C2):
    """Seeded synthetic weights in device memory (GGUF layouts), bound to a decoder."""
    dev = torch.device("cuda", torch.cuda.current_device())
    rng = np.random.default_rng(seed)
    s = [seed * 100003]

    def mat(k, m):
        s[0] += 1
        t = torch.empty(q8_bytes(k, m), dtype=torch.uint8, device=dev)
        ctx.fill_synthetic(Q8_0, t, k, m, s[0])
        return t

    def vec(n, center, amp):
        return torch.from_numpy((center + amp * rng.uniform(-1, 1, n)).astype(np.float32)).to(dev)

    q, kv = c["n_head"] * c["head_dim"], c["n_head_kv"] * c["head_dim"]
    w = {"tok_embd": mat(c["n_embd"], c["n_vocab"]), "output_norm": vec(c["n_embd"], 1.0, 0.1)}
    w["output"] = w["tok_embd"]  # tied embeddings
    w["layers"] = []
    for _ in range(c["n_layer"]):
        L = {"attn_norm": vec(c["n_embd"], 1.0, 0.1), "ffn_norm": vec(c["n_embd"], 1.0, 0.1),
             "bq": vec(q, 0.0, 0.02), "bk": vec(kv, 0.0, 0.02), "bv": vec(kv, 0.0, 0.02)}
        for name, k, m in c2_shapes(c):
            L[name] = mat(k, m)
        w["layers"].append(L)
    torch.cuda.synchronize()
    return w


def c2_host_weights(seed, c=C2):
    """The same shapes and value distributions in host memory, for the CPU legs (quants uniform
    in [-127, 127], fp16 scales |N(0,1)| * 0.002)."""
    rng = np.random.default_rng(seed)

    def mat(k, m):
        nb = k // 32
        b = np.empty((m, nb, 34), dtype=np.uint8)
        b[:, :, 2:] = rng.integers(-127, 128, size=(m, nb, 32), dtype=np.int8).view(np.uint8)
        sc = (0.002 * np.abs(rng.standard_normal((m, nb)))).astype(np.float16)
        b[:, :, :2] = sc.view(np.uint8).reshape(m, nb, 2)
        return b.reshape(-1)

    def vec(n, center, amp):
        return (center + amp * rng.uniform(-1, 1, n)).astype(np.float32)

    q, kv = c["n_head"] * c["head_dim"], c["n_head_kv"] * c["head_dim"]
    w = {"tok_embd": mat(c["n_embd"], c["n_vocab"]), "output_norm": vec(c["n_embd"], 1.0, 0.1)}
    w["output"] = w["tok_embd"]
    w["layers"] = []
    for _ in range(c["n_layer"]):
        L = {"attn_norm": vec(c["n_embd"], 1.0, 0.1), "ffn_norm": vec(c["n_embd"], 1.0, 0.1),
             "bq": vec(q, 0.0, 0.02), "bk": vec(kv, 0.0, 0.02), "bv": vec(kv, 0.0, 0.02)}
        for name, k, m in c2_shapes(c):
            L[name] = mat(k, m)
        w["layers"].append(L)
    return w


def c2_cpu(budget_s: float, max_tokens: int, c=C2):
    """The oracle's decode forward (oracle/decode_ref.py; matvecs on all host threads) over the
    last positions of the context: (tok/s, tokens timed, threads)."""
    from oracle import pyoracle as orc
    from oracle.decode_ref import RefDecoder
    ref = RefDecoder(c, c2_host_weights(7), mt=True)
    n = c["n_ctx"]
    max_tokens = max(1, min(max_tokens, n - 2))
    tok = 1
    tok = ref.step(tok, n - max_tokens - 1)[1]  # warm (page in the weights)
    t0 = time.perf_counter()
    done = 0
    for p in range(n - max_tokens, n):
        tok = ref.step(tok, p)[1]
        done += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    return done / dt, done, orc.lib(True).orc_threads()


def c2_timed_tokens(args, ugb, ctx, torch, world, w, c, stream, cap, sampler=None):
    """A decoder of config c on weights w: K device-driven token replays of one captured step
    at the last K positions of the context, after W warm-up replays.  Returns (decoder, graph,
    path, kernels per token, max-over-ranks ms, timed positions, clocks)."""
    dec = ugb.Decoder(ctx, **c)
    dec.bind(w["tok_embd"], w["output_norm"], w["output"], w["layers"])
    active = dec.set_path(PATHS[args.path])
    n_ctx = c["n_ctx"]
    # One token step captured once; each replay reads the previous step's greedy token and
    # advances the position on the device (embedding kernel), so K replays decode K tokens.
    dec.set_state(1, 0, stream)
    graph = ctx.capture(lambda: dec.step(), cap)

    def run(first_pos, count, tok=1):
        """count replays starting at first_pos; re-seed the state when the context is full."""
        pos = first_pos
        dec.set_state(tok, pos, stream)
        for _ in range(count):
            if pos == n_ctx:
                pos = 0
                dec.set_state(tok, 0, stream)
            graph.launch(stream)
            pos += 1

    K, W = args.steps, args.warmup
    start = max(0, n_ctx - K)
    if sampler:
        sampler.start()
    run(max(0, start - W), W)
    stream.synchronize()
    code, bits = ctx.status_read(stream)
    assert code == ugb.OK, ("status after warm-up", code, bits)
    # -- timed region: K tokens, device time by CUDA events on the launching stream --
    barrier(world, torch)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    dec.set_state(1, start, stream)
    e0.record(stream)
    pos = start
    for _ in range(K):
        if pos == n_ctx:
            pos = 0
            dec.set_state(1, 0, stream)
        graph.launch(stream)
        pos += 1
    e1.record(stream)
    torch.cuda.synchronize()
    barrier(world, torch)
    clocks = sampler.stop() if sampler else None
    ms = e0.elapsed_time(e1)
    code, bits = ctx.status_read(stream)
    assert code == ugb.OK, ("status after timing", code, bits)
    return dec, graph, active, graph.kernels(), reduce_max(ms, world, torch), [(start + i) % n_ctx for i in range(K)], clocks


def c2_gpu(args, ugb, ctx, torch, rank, world, c=C2):
    dev = torch.device("cuda", torch.cuda.current_device())
    w = c2_device_weights(ctx, ugb, torch, seed=1 + rank, c=c)
    c = dict(c, kv_type=KV_TYPES[args.kv])
    n_ctx = c["n_ctx"]
    stream = torch.cuda.Stream()
    cap = torch.cuda.Stream()
    K = args.steps
    sampler = ClockSampler(int(os.environ.get("LOCAL_RANK", "0")) if world > 1 else torch.cuda.current_device())
    dec, graph, active, kernels_per_token, ms_max, timed_pos, clocks = c2_timed_tokens(
        args, ugb, ctx, torch, world, w, c, stream, cap, sampler)
    token_bytes = float(np.mean([c2_token_bytes(c, p + 1) for p in timed_pos]))

    # -- dominant kernel.  Token path: the step is one launch of the persistent token kernel, so
    # its CUDA-event time per launch is the step's and its algorithmic bytes are the token's.
    # Launch chain: the fused gate/up matvec (17920 x 1536 Q8_0, the largest launch of a layer),
    # all 28 layers' matrices back to back in one graph (each launch streams its own 29 MB from
    # HBM), timed by CUDA events on the launching stream --
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if active == ugb.PATH_TOKEN:
        kern_ms, kern_bytes, kgraph = ms_max / K, token_bytes, None
    else:
        kern_ms, kern_bytes, kgraph = c2_gateup_kernel(ugb, ctx, torch, dev, w, c, cap, stream, e0, e1)

    # -- end to end through the host-facing C-ABI call: ugb_decoder_token (host token and
    # position in: H2D of the state; graph replay; D2H of the state and the status word) --
    e2e_steps = min(max(K, 32), n_ctx)
    tok = 1
    for p in range(3):
        tok = dec.token(tok, n_ctx - e2e_steps - 3 + p, stream)
    t0 = time.perf_counter()
    for p in range(n_ctx - e2e_steps, n_ctx):
        tok = dec.token(tok, p, stream)
    e2e_s = (time.perf_counter() - t0) / e2e_steps
    e2e_s = reduce_max(e2e_s * 1e3, world, torch) / 1e3
    dec.close()
    graph.close()
    if kgraph is not None:
        kgraph.close()
    other = None
    if c["kv_type"] == 1:  # the reference's own fp32 cache, same weights and positions
        d2, g2, _, _, ms2, pos2, _ = c2_timed_tokens(args, ugb, ctx, torch, world, w, dict(c, kv_type=0), stream, cap)
        d2.close()
        g2.close()
        other = {"kv_cache": "fp32", "value": world * K / (ms2 / 1e3), "ms_per_step": ms2 / K,
                 "bytes_per_token": float(np.mean([c2_token_bytes(dict(c, kv_type=0), p + 1) for p in pos2]))}
    return {
        "value": world * K / (ms_max / 1e3), "ms_per_step": ms_max / K, "clocks": clocks,
        "gpu_launches": kernels_per_token * K, "path": active,
        "token_bytes": token_bytes, "kv_other": other,
        "kernel_ms": kern_ms, "kernel_bytes": kern_bytes,
        "e2e": {"value": world / e2e_s, "unit": "tok/s", "h2d_bytes_per_step": 16,
                "d2h_bytes_per_step": 16 + 4},
    }


def c2_gateup_kernel(ugb, ctx, torch, dev, w, c, cap, stream, e0, e1):
    """Per-launch time and algorithmic bytes of the launch chain's fused gate/up matvec."""
    xq = ugb.alloc_q8act(c["n_embd"], 1, device=dev)
    xv = torch.randn(c["n_embd"], device=dev)
    ctx.quant_q8_1(xv, xq, c["n_embd"], 1)
    gu = torch.empty(2 * c["n_ff"], dtype=torch.float32, device=dev)
    rb = ugb.row_bytes(Q8_0, c["n_embd"])
    ctx.set_pdl(True)
    kgraph = ctx.capture(lambda: [ctx.matvec_multi(Q8_0, [L["w_gate"], L["w_up"]], [c["n_ff"], c["n_ff"]], rb,
                                                   xq, gu, c["n_embd"], 1) for L in w["layers"]], cap)
    ctx.set_pdl(False)
    kgraph.launch(stream)
    stream.synchronize()
    reps = 8
    e0.record(stream)
    for _ in range(reps):
        kgraph.launch(stream)
    e1.record(stream)
    stream.synchronize()
    kern_ms = e0.elapsed_time(e1) / (reps * c["n_layer"])
    kern_bytes = 2 * q8_bytes(c["n_embd"], c["n_ff"]) + xq.numel() + gu.numel() * 4
    return kern_ms, kern_bytes, kgraph


# ---- workload c1 ----------------------------------------------------------------------------

C1_K, C1_M = 1536, 8960
C1_ROTATE = 24

# Algorithmic bytes of one step (quant_act + linear): the Q8_0 weights once, the fp32
# activation once and the fp32 output once (the 1.7 KB Q8_1 intermediate stays in L2).
C1_BYTES = (C1_M * (C1_K // 32) * 34          # 14,622,720 B of Q8_0 weights
            + C1_K * 4                           # fp32 activation
            + C1_M * 4)                          # fp32 output


def c1_gpu(args, ugb, ctx, torch, rank, world):
    dev = torch.device("cuda", torch.cuda.current_device())
    rb = ugb.row_bytes(Q8_0, C1_K)
    ws = [torch.empty(rb * C1_M, dtype=torch.uint8, device=dev) for _ in range(C1_ROTATE)]
    for i, w in enumerate(ws):
        ctx.fill_synthetic(Q8_0, w, C1_K, C1_M, seed=1000 + i)
    gen = torch.Generator(device="cpu").manual_seed(1234 + rank)
    xs = torch.randn((C1_ROTATE, C1_K), generator=gen).to(dev)
    xq = ugb.alloc_q8act(C1_K, 1, device=dev)
    y = torch.empty(C1_M, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream()

    def step(i):
        # quant_act + linear (gpu_graph.rs:74-80) as one call: at this shape (batch 1, the matrix
        # staged whole, one CTA per SM) the quantisation runs inside the matvec kernel, and each
        # step's weight copies start while the previous step computes (programmatic dependent
        # launch with two steps resident per SM)
        j = i % C1_ROTATE
        ctx.matvec_f32(Q8_0, ws[j], rb, xs[j], xq, y, C1_K, C1_M, 1)

    # The K timed steps are one CUDA graph (the reference submits its per-token command list
    # as one GPFIFO entry); kernels launch with programmatic dependent launch so each matvec
    # streams its weights while the previous kernel drains.
    ctx.set_pdl(True)
    cap = torch.cuda.Stream()
    graph = ctx.capture(lambda: [step(i) for i in range(args.steps)], cap)
    warm = ctx.capture(lambda: [step(i) for i in range(args.warmup)], cap)
    warm.launch(stream)
    code, bits = ctx.status_read()
    assert code == ugb.OK, ("status after warm-up", code, bits)

    # -- timed region: K steps, device time by CUDA events, max over ranks --
    sampler = ClockSampler(int(os.environ.get("LOCAL_RANK", "0")) if world > 1 else torch.cuda.current_device())
    barrier(world, torch)
    torch.cuda.synchronize()
    sampler.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    graph.launch(stream)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier(world, torch)
    clocks = sampler.stop()
    ms = e0.elapsed_time(e1)
    ms_max = reduce_max(ms, world, torch)
    launches = args.steps  # one fused quant + matvec kernel per step

    # -- the dominant kernel (the matvec) back to back in a graph, for the roofline --
    reps = max(args.steps, 96)
    kgraph = ctx.capture(lambda: [ctx.matvec(Q8_0, ws[i % C1_ROTATE], rb, xq, y, C1_K, C1_M, 1)
                                  for i in range(reps)], cap)
    kgraph.launch(stream)
    torch.cuda.synchronize()
    e0.record(stream)
    kgraph.launch(stream)
    e1.record(stream)
    torch.cuda.synchronize()
    kern_ms = e0.elapsed_time(e1) / reps
    ctx.set_pdl(False)
    code, bits = ctx.status_read()
    assert code == ugb.OK, ("status after timing", code, bits)

    # -- end to end through the host-buffer C-ABI call (ugb_linear: H2D x, D2H y) --
    x_host = [np.random.default_rng(7 + i).standard_normal(C1_K).astype(np.float32) for i in range(4)]
    for i in range(3):
        ctx.linear(Q8_0, ws[i], rb, x_host[i % 4], C1_K, C1_M)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    e2e_steps = max(args.steps, 20)
    for i in range(e2e_steps):
        ctx.linear(Q8_0, ws[i % C1_ROTATE], rb, x_host[i % 4], C1_K, C1_M)
    e2e_s = (time.perf_counter() - t0) / e2e_steps
    e2e_s = reduce_max(e2e_s * 1e3, world, torch) / 1e3

    per_step_s = ms_max / 1e3 / args.steps
    value = world * C1_BYTES / per_step_s / 1e9
    return {
        "value": value, "ms_per_step": ms_max / args.steps, "clocks": clocks,
        "gpu_launches": launches,
        "kernel_ms": kern_ms, "kernel_bytes": C1_M * (C1_K // 32) * 34 + C1_M * 4,
        "e2e": {"value": world * C1_BYTES / e2e_s / 1e9, "unit": "GB/s",
                "h2d_bytes_per_step": C1_K * 4, "d2h_bytes_per_step": C1_M * 4 + 4},
    }


def c1_cpu(samples: int, mt: bool = True):
    """The oracle (CPU restatement) on the same workload: quant_act + matvec per step."""
    from oracle import pyoracle as orc
    rng = np.random.default_rng(99)
    rb = C1_K // 32 * 34
    w = rng.integers(0, 256, size=rb * C1_M, dtype=np.uint8)
    blocks = w.reshape(-1, 34)
    blocks[:, 0] = 0x19
    blocks[:, 1] = 0x14
    x = rng.standard_normal(C1_K).astype(np.float32)
    lib = orc.lib(mt)
    q, d, s, _ = orc.quant_act(x)
    orc.matvec(Q8_0, w, rb, q, d, s, C1_K, C1_M, 1, mt=mt)  # warm
    t0 = time.perf_counter()
    for _ in range(samples):
        q, d, s, _ = orc.quant_act(x)
        orc.matvec(Q8_0, w, rb, q, d, s, C1_K, C1_M, 1, mt=mt)
    dt = (time.perf_counter() - t0) / samples
    return C1_BYTES / dt / 1e9, lib.orc_threads() if mt else 1




# ---- workload c3: Q8 prefill GEMMs of the 1.5B-shaped model -------------------------------

C3_TOKENS = 512


def c3_gemms(c=C2):
    """(name, n rows, k) of the four prefill GEMMs of a layer: fused Q/K/V, O, fused gate/up,
    down (the K and V rows are the 512 rows after the 1536 Q rows)."""
    q, kv = c["n_head"] * c["head_dim"], c["n_head_kv"] * c["head_dim"]
    return [("qkv", q + 2 * kv, c["n_embd"]), ("o", c["n_embd"], q),
            ("gate_up", 2 * c["n_ff"], c["n_embd"]), ("down", c["n_embd"], c["n_ff"])]


def c3_ops_per_step(c=C2, m=C3_TOKENS):
    return c["n_layer"] * sum(2 * m * n * k for _, n, k in c3_gemms(c))


def c3_attn_flops(c=C2, m=C3_TOKENS):
    """fp32 multiply-adds x 2 of the causal attention of an m-token prompt (scores and P.V)."""
    return c["n_layer"] * c["n_head"] * 2 * 2 * c["head_dim"] * m * (m + 1) // 2


def c3_gemm_kernel(ugb, ctx, torch, dev, cap, stream, c=C2, m=C3_TOKENS):
    """Per-launch time of the fused gate/up prefill GEMM (512 x 17920 x 1536) on its own
    operands, 28 launches back to back in one graph (each layer's weights are distinct)."""
    _, n, k = c3_gemms(c)[2]
    gen = torch.Generator(device="cpu").manual_seed(13)
    ops = []
    for li in range(c["n_layer"]):
        w = torch.empty(q8_bytes(k, n), dtype=torch.uint8, device=dev)
        ctx.fill_synthetic(Q8_0, w, k, n, seed=7000 + li)
        wp = ugb.alloc_prefill(n, k, device=dev)
        ctx.prefill_repack_q8_0(w, n, k, wp)
        del w
        xp = ugb.alloc_prefill(m, k, device=dev)
        ctx.prefill_quant(torch.randn((m, k), generator=gen).to(dev), m, k, xp)
        ops.append((wp, xp, torch.empty((m, n), dtype=torch.float32, device=dev)))
    torch.cuda.synchronize()
    ctx.set_pdl(True)
    kgraph = ctx.capture(lambda: [ctx.prefill_gemm(wp, xp, y, m, n, k) for wp, xp, y in ops], cap)
    ctx.set_pdl(False)
    kgraph.launch(stream)
    stream.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 4
    e0.record(stream)
    for _ in range(reps):
        kgraph.launch(stream)
    e1.record(stream)
    stream.synchronize()
    kgraph.close()
    return e0.elapsed_time(e1) / (reps * len(ops)), 2 * m * n * k


def int8_peak_tops(torch, dev):
    """Measured INT8 tensor peak on this GPU: cuBLAS int8 GEMM 8192^3 (torch._int_mm), burst."""
    a8 = torch.randint(-127, 127, (8192, 8192), dtype=torch.int8, device=dev)
    b8 = torch.randint(-127, 127, (8192, 8192), dtype=torch.int8, device=dev)
    for _ in range(3):
        torch._int_mm(a8, b8)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(10):
        torch._int_mm(a8, b8)
    e1.record()
    torch.cuda.synchronize()
    return 2 * 8192 ** 3 / (e0.elapsed_time(e1) / 10 / 1e3) / 1e12


def c3_gpu(args, ugb, ctx, torch, rank, world, c=C2, m=C3_TOKENS):
    """The whole 512-token prefill of the 1.5B model (ugb_decoder_prefill_async, replayed from one
    captured graph): embedding, 28 layers of norm / quant / Q-K-V GEMM / bias + RoPE + KV write /
    causal attention / quant / O GEMM / norm / quant / gate-up GEMM / SiLU / quant / down GEMM, and
    the last token through the output norm, the head and greedy selection."""
    dev = torch.device("cuda", torch.cuda.current_device())
    c = dict(c, kv_type=KV_TYPES[args.kv])
    w = c2_device_weights(ctx, ugb, torch, seed=11 + rank, c=c)
    dec = ugb.Decoder(ctx, **c)
    dec.bind(w["tok_embd"], w["output_norm"], w["output"], w["layers"])
    dec.prefill_prepare(m)  # one-time repack, outside timing (as the reference's init_swizzle)
    prompt = np.random.default_rng(5 + rank).integers(0, c["n_vocab"], size=m).astype(np.int32)
    toks = torch.from_numpy(prompt).to(dev)
    stream = torch.cuda.Stream()
    cap = torch.cuda.Stream()
    ctx.set_pdl(True)
    graph = ctx.capture(lambda: dec.prefill_async(toks, m, 0), cap)
    ctx.set_pdl(False)
    kernels = graph.kernels()
    sampler = ClockSampler(int(os.environ.get("LOCAL_RANK", "0")) if world > 1 else torch.cuda.current_device())
    sampler.start()
    for _ in range(args.warmup):
        graph.launch(stream)
    stream.synchronize()
    code, bits = ctx.status_read(stream)
    assert code == ugb.OK, ("status after warm-up", code, bits)
    barrier(world, torch)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        graph.launch(stream)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier(world, torch)
    clocks = sampler.stop()
    ms = e0.elapsed_time(e1)
    ms_max = reduce_max(ms, world, torch)
    code, bits = ctx.status_read(stream)
    assert code == ugb.OK, ("status after timing", code, bits)
    graph.close()
    # end to end through the host-facing call: ugb_decoder_prefill (host prompt in, greedy next
    # token out, status checked) every step
    e2e_steps = max(3, min(args.steps, 10))
    dec.prefill(list(prompt), 0)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        dec.prefill(list(prompt), 0)
    e2e_s = (time.perf_counter() - t0) / e2e_steps
    e2e_s = reduce_max(e2e_s * 1e3, world, torch) / 1e3
    dec.close()
    kern_ms, kern_ops = c3_gemm_kernel(ugb, ctx, torch, dev, cap, stream, c, m)
    return {
        "value": world * m * args.steps / (ms_max / 1e3), "ms_per_step": ms_max / args.steps, "clocks": clocks,
        "gpu_launches": kernels * args.steps,
        "kernel_ms": kern_ms, "kernel_ops": kern_ops, "int8_tops": int8_peak_tops(torch, dev),
        "step_gemm_ops": c3_ops_per_step(c, m), "step_attn_flops": c3_attn_flops(c, m),
        "e2e": {"value": world * m / e2e_s, "unit": "tok/s", "h2d_bytes_per_step": m * 4,
                "d2h_bytes_per_step": 104 + 4},
    }


def c3_cpu(budget_s: float, c=C2, kv_type=0):
    """The oracle's whole-prompt prefill of the full-depth model (oracle/decode_ref.py
    RefDecoder.prefill: batched oracle/ugb_oracle.c matvecs on POSIX threads, numpy glue) on a
    prompt of as many tokens as fit the budget: (tok/s, tokens, threads)."""
    from oracle import pyoracle as orc
    from oracle.decode_ref import RefDecoder
    cfg = dict(c, kv_type=kv_type)
    ref = RefDecoder(cfg, c2_host_weights(7, c), mt=True)
    rng = np.random.default_rng(3)
    tokens = 4
    while True:
        prompt = rng.integers(0, c["n_vocab"], size=tokens)
        t0 = time.perf_counter()
        ref.prefill(prompt, 0)
        dt = time.perf_counter() - t0
        if dt * 3 > budget_s or tokens >= C3_TOKENS:
            break
        tokens *= 2
    return tokens / dt, tokens, orc.lib(True).orc_threads()


# ---- workloads c4 / c5: batched and sharded decode of the larger configs ---------------------

Q3_K, Q4_K = 11, 12
KIND_BLOCK = {Q8_0: (32, 34), Q4_K: (256, 144), Q3_K: (256, 110)}

# Qwen2.5-7B-shaped, Q4_K linear weights, Q8_0 head (tied here: the
# same bytes stream per token), batch 1 / 4 / 8 at context 1024, head row-split over the GPUs.
C4 = dict(n_layer=28, n_embd=3584, n_ff=18944, n_head=28, n_head_kv=4, head_dim=128, n_vocab=152064,
          n_ctx=1024, rope_theta=1e6, norm_eps=1e-6, kind=Q4_K, head_kind=Q8_0)
# 48 layers, hidden 4096, 192 Q3_K experts of 1536 (top-8 softmax),
# 32 / 4 heads of 128, Q8_0 attention and router, vocab 151936, batch 1 / 8 at context 2048,
# expert-parallel over the GPUs.
C5 = dict(n_layer=48, n_embd=4096, n_ff=0, n_head=32, n_head_kv=4, head_dim=128, n_vocab=151936,
          n_ctx=2048, rope_theta=1e6, norm_eps=1e-6, kind=Q8_0, head_kind=Q8_0, n_expert=192, top_k=8,
          n_ff_expert=1536, expert_kind=Q3_K)


def kbytes(kind, k, m):
    e, b = KIND_BLOCK[kind]
    return m * (k // e) * b


def big_step_bytes(c, batch, pos, world=1, rank=0):
    """Algorithmic bytes one device streams per step: its weights once (dense layers; the
    routed experts actually selected by the batch -- top_k per token, at most every held
    expert -- at their expected distinct count under uniform routing), its head rows, and the
    batch's fp32 KV cache read at context `pos`."""
    q, kv = c["n_head"] * c["head_dim"], c["n_head_kv"] * c["head_dim"]
    e = c["n_embd"]
    attn = kbytes(c["kind"], e, q + 2 * kv) + kbytes(c["kind"], q, e)
    if c.get("n_expert", 0):
        ne, k_, ff = c["n_expert"], c["top_k"], c["n_ff_expert"]
        per_expert = 2 * kbytes(c["expert_kind"], e, ff) + kbytes(c["expert_kind"], ff, e)
        distinct = ne * (1 - (1 - k_ / ne) ** batch)           # expected distinct experts touched
        ffn = kbytes(c["kind"], e, ne) + distinct / world * per_expert
    else:
        ffn = kbytes(c["kind"], e, 2 * c["n_ff"]) + kbytes(c["kind"], c["n_ff"], e)
    layers = c["n_layer"] * (attn + ffn)
    vn = c.get("n_vocab_local") or c["n_vocab"]
    head = kbytes(c["head_kind"], e, vn)
    kvb = c["n_layer"] * 2 * kv * kv_elem_bytes(c) * pos * batch
    return layers + head + kvb


def shard_config(c, workload, rank, world):
    c = dict(c)
    if workload == "c4" and world > 1:
        per = -(-c["n_vocab"] // world)
        c["vocab0"] = rank * per
        c["n_vocab_local"] = min(per, c["n_vocab"] - c["vocab0"])
    if workload == "c5" and world > 1:
        per = c["n_expert"] // world
        c["expert0"] = rank * per
        c["n_expert_local"] = per if rank < world - 1 else c["n_expert"] - rank * per
    return c


def big_gpu(args, ugb, ctx, torch, rank, world, workload):
    base = dict(C4 if workload == "c4" else C5)
    if args.layers:
        base["n_layer"] = args.layers
    batch = args.batch or (8 if workload == "c4" else 1)
    c = shard_config(dict(base, batch=batch, kv_type=KV_TYPES[args.kv]), workload, rank, world)
    dec = ugb.Decoder(ctx, **c)
    dec.synthetic(11)
    comm = None
    if world > 1:
        uid = [ugb.comm_unique_id() if rank == 0 else None]
        torch.distributed.broadcast_object_list(uid, src=0)
        comm = ugb.Comm(ctx, rank, world, uid[0])
        dec.set_comm(comm)
    active = dec.set_path(PATHS[args.path])
    n_ctx = c["n_ctx"]
    stream = torch.cuda.Stream()
    cap = torch.cuda.Stream()
    K, W = args.steps, args.warmup
    if K + W > n_ctx - 1:
        K = max(1, n_ctx - 1 - W)
    start = n_ctx - K
    toks = [1 + b for b in range(batch)]
    dec.set_tokens(toks, 0, stream)
    barrier(world, torch)
    graph = ctx.capture(lambda: dec.step(), cap)
    kernels = graph.kernels()  # includes NCCL's kernels when the step holds collectives
    sampler = ClockSampler(int(os.environ.get("LOCAL_RANK", "0")) if world > 1 else torch.cuda.current_device())
    sampler.start()
    dec.set_tokens(toks, start - W, stream)
    for _ in range(W):
        graph.launch(stream)
    stream.synchronize()
    code, bits = ctx.status_read(stream)
    assert code == ugb.OK, ("status after warm-up", code, bits)
    barrier(world, torch)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(K):
        graph.launch(stream)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier(world, torch)
    clocks = sampler.stop()
    ms = e0.elapsed_time(e1)
    code, bits = ctx.status_read(stream)
    assert code == ugb.OK, ("status after timing", code, bits)
    ms_max = reduce_max(ms, world, torch)
    step_bytes = float(np.mean([big_step_bytes(c, batch, start + i + 1, world) for i in range(K)]))
    # end to end: host tokens in, next tokens out, every step (ugb_decoder_tokens)
    e2e_steps = max(3, min(K, 16))
    barrier(world, torch)
    nxt = toks
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        nxt = dec.tokens(nxt, n_ctx - e2e_steps + i, stream)
    e2e_s = (time.perf_counter() - t0) / e2e_steps
    e2e_s = reduce_max(e2e_s * 1e3, world, torch) / 1e3
    barrier(world, torch)
    collective = None
    if comm:
        # the step's collective alone, back to back on the stream: the MoE layer output (sum of
        # batch x hidden f32) or the greedy keys (max of batch u64)
        if workload == "c5":
            cbuf = torch.zeros(batch * c["n_embd"], dtype=torch.float32, device="cuda")
            call, what, per_step = comm.allreduce_f32, f"sum of {batch}x{c['n_embd']} f32", c["n_layer"]
        else:
            cbuf = torch.zeros(batch, dtype=torch.int64, device="cuda")
            call, what, per_step = comm.allreduce_max_u64, f"max of {batch} u64 greedy keys", 1
        for _ in range(5):
            call(cbuf, stream)
        stream.synchronize()
        barrier(world, torch)
        reps = 200
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        c0.record(stream)
        for _ in range(reps):
            call(cbuf, stream)
        c1.record(stream)
        torch.cuda.synchronize()
        us = reduce_max(c0.elapsed_time(c1) * 1e3 / reps, world, torch)
        collective = {"op": "ugb_comm one-shot all-reduce over NVLink peer memory: " + what, "us_per_call": us,
                      "calls_per_step": per_step, "share_of_step": per_step * us / 1e3 / (ms_max / K)}
        code, bits = ctx.status_read(stream)
        assert code == ugb.OK, ("status after the collective timing", code, bits)
        barrier(world, torch)
    graph.close()
    dec.close()  # releases the decoder's own captured graph before the communicator goes
    if comm:
        comm.close()
    return {
        "value": batch * K / (ms_max / 1e3), "ms_per_step": ms_max / K, "clocks": clocks,
        "gpu_launches": kernels * K, "step_bytes": step_bytes, "batch": batch, "path": active,
        "e2e": {"value": batch / e2e_s, "unit": "tok/s", "h2d_bytes_per_step": 8 * 4 + 8,
                "d2h_bytes_per_step": 112 + 4},
        "config": c, "collective": collective,
    }


SHARDED = (("c4_b8_head_rows_split", "c4", 8), ("c5_b1_experts_split", "c5", 1), ("c5_b8_experts_split", "c5", 8))


def sharded_gpu(args, ugb, ctx, torch, rank, world):
    """The configs that shard (BASELINE configs 4 and 5) at this process group's size: C4 batch 8
    with the head rows split over the GPUs, C5 batch 1 and 8 with the experts split.  tok/s of the
    whole group, per-step time, and the time of the step's collective measured alone."""
    import copy
    out = {}
    for name, wl, batch in SHARDED:
        a = copy.copy(args)
        a.batch, a.path, a.layers = batch, "auto", 0
        res = big_gpu(a, ugb, ctx, torch, rank, world, wl)
        out[name] = {"value": res["value"], "unit": "tok/s", "ms_per_step": res["ms_per_step"], "n_gpus": world,
                     "batch": batch, "roofline_frac": res["step_bytes"] / (res["ms_per_step"] / 1e3) / 1e9 /
                     load_peaks()[0], "collective": res["collective"],
                     "path": "token kernel" if res["path"] == ugb.PATH_TOKEN else "launch chain (captured graph)"}
        torch.cuda.empty_cache()
    return out


def host_quant_matrix(rng, kind, k, m):
    """Random GGUF blocks with sane fp16 scales (timing input for the CPU legs)."""
    e, bsz = KIND_BLOCK[kind]
    b = rng.integers(0, 256, size=(m, k // e, bsz), dtype=np.uint8)
    half = np.frombuffer(np.float16(0.002).tobytes(), np.uint8)
    if kind == Q8_0:
        b[:, :, 0:2] = half
    elif kind == Q4_K:
        b[:, :, 0:2] = half
        b[:, :, 2:4] = half
    else:
        b[:, :, 108:110] = half
    return b.reshape(-1)


def big_cpu(budget_s, workload, batch):
    """The oracle decode forward on the host cores: a 1-layer and a 2-layer model of the
    config's shapes, timed per token, extrapolated to the full depth (per-layer time = the
    difference).  The oracle decodes one sequence at a time, so its tok/s is the same for any
    batch."""
    from oracle import pyoracle as orc
    from oracle.decode_ref import RefDecoder
    base = dict(C4 if workload == "c4" else C5)
    rng = np.random.default_rng(5)
    e, q, kv = base["n_embd"], base["n_head"] * base["head_dim"], base["n_head_kv"] * base["head_dim"]
    kind = base["kind"]
    tok = host_quant_matrix(rng, Q8_0, e, base["n_vocab"])

    def layer():
        L = {"attn_norm": np.ones(e, np.float32), "ffn_norm": np.ones(e, np.float32),
             "wq": host_quant_matrix(rng, kind, e, q), "wk": host_quant_matrix(rng, kind, e, kv),
             "wv": host_quant_matrix(rng, kind, e, kv), "wo": host_quant_matrix(rng, kind, q, e)}
        if base.get("n_expert", 0):
            ek, ne, ff = base["expert_kind"], base["n_expert"], base["n_ff_expert"]
            L.update(router=host_quant_matrix(rng, kind, e, ne), gate_exps=host_quant_matrix(rng, ek, e, ff * ne),
                     up_exps=host_quant_matrix(rng, ek, e, ff * ne), down_exps=host_quant_matrix(rng, ek, ff, e * ne))
        else:
            L.update(w_gate=host_quant_matrix(rng, kind, e, base["n_ff"]),
                     w_up=host_quant_matrix(rng, kind, e, base["n_ff"]),
                     w_down=host_quant_matrix(rng, kind, base["n_ff"], e))
        return L

    layers = [layer(), layer()]
    times = []
    for n in (1, 2):
        cfg = dict(base, n_layer=n)
        ref = RefDecoder(cfg, {"tok_embd": tok, "output": tok, "output_norm": np.ones(e, np.float32),
                               "layers": layers[:n]}, mt=True)
        t = 1
        ref.step(t, 0)
        t0 = time.perf_counter()
        steps = 0
        while steps < 2 or (time.perf_counter() - t0 < budget_s / 4 and steps < 8):
            t = ref.step(t, steps + 1)[1]
            steps += 1
        times.append((time.perf_counter() - t0) / steps)
    per_layer = max(times[1] - times[0], 0.0)
    per_token = times[0] + (base["n_layer"] - 1) * per_layer
    return 1.0 / per_token, per_token, orc.lib(True).orc_threads()


# ---- driver -----------------------------------------------------------------------------------

def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["c2", "c1", "c3", "c4", "c5"], default="c2")
    ap.add_argument("--batch", type=int, default=0, help="c4 / c5 sequences (default 8 / 1)")
    ap.add_argument("--layers", type=int, default=0,
                    help="c4 / c5: decode this many layers instead of the config's (profiling captures only)")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--sharded", choices=["auto", "on", "off"], default="auto",
                    help="c2: also measure the sharding configs (c4 batch 8 head split, c5 batch 1 / 8 experts "
                         "split) at this --gpus; auto = when more than one GPU")
    ap.add_argument("--kv", choices=sorted(KV_TYPES), default="f16",
                    help="c2 / c4 / c5 KV cache element type (BASELINE config 2: fp16; the reference keeps fp32)")
    ap.add_argument("--path", choices=sorted(PATHS), default="auto",
                    help="c2 / c4 / c5 decoder path: persistent token kernel where it applies (auto), "
                         "the per-kernel launch chain, or the token kernel only")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    hbm_peak, _, peak_kind = load_peaks()
    if args.workload == "c2":
        config = {"workload": "c2: greedy batch-1 decode, Qwen2.5-1.5B-shaped, all linear weights Q8_0",
                  "layers": C2["n_layer"], "hidden": C2["n_embd"], "ffn": C2["n_ff"],
                  "heads": f"{C2['n_head']}/{C2['n_head_kv']}x{C2['head_dim']}", "vocab": C2["n_vocab"],
                  "context": C2["n_ctx"], "kv_cache": "fp16" if args.kv == "f16" else "fp32",
                  "timed_positions": f"last {min(args.steps, C2['n_ctx'])} of {C2['n_ctx']}",
                  "l2": "inputs larger than L2 (1.655 GB of weights per token)",
                  "parallelism": f"replicas x{world}"}
        base = {"metric": "decode tok/s", "unit": "tok/s", "dtype": "int8 x int8 -> int32 (Q8_0 x Q8_1), fp32 glue"}
    elif args.workload in ("c4", "c5"):
        big = C4 if args.workload == "c4" else C5
        bsz = args.batch or (8 if args.workload == "c4" else 1)
        if args.workload == "c4":
            name = "c4: greedy decode, Qwen2.5-7B-shaped, Q4_K linear weights, Q8_0 head"
            split = f"head rows split over {world} GPU(s), greedy keys all-reduced (max) over NVLink"
        else:
            name = "c5: greedy decode, 48-layer MoE (192 Q3_K experts of 1536, top-8), Q8_0 attention / router"
            split = f"experts split over {world} GPU(s) ({192 // world} each), layer outputs all-reduced over NVLink"
        config = {"workload": name, "batch": bsz, "layers": big["n_layer"], "hidden": big["n_embd"],
                  "heads": f"{big['n_head']}/{big['n_head_kv']}x{big['head_dim']}", "vocab": big["n_vocab"],
                  "context": big["n_ctx"], "kv_cache": "fp16" if args.kv == "f16" else "fp32",
                  "head": "tied to the Q8_0 token embedding",
                  "l2": "inputs larger than L2", "parallelism": split if world > 1 else "1 GPU"}
        base = {"metric": "decode tok/s", "unit": "tok/s",
                "dtype": "int8 x int8 -> int32 (K-quant / Q8_0 x Q8_1), fp32 glue"}
    elif args.workload == "c3":
        config = {"workload": "c3: Q8 prefill of the Qwen2.5-1.5B-shaped Q8_0 model, 512-token prompt of seeded "
                              "uniform token ids, the whole prefill graph",
                  "tokens": C3_TOKENS, "layers": C2["n_layer"], "context": C2["n_ctx"],
                  "kv_cache": "fp16" if args.kv == "f16" else "fp32",
                  "gemms_per_layer": "qkv 2048x1536, o 1536x1536, gate_up 17920x1536, down 1536x8960",
                  "per_gemm": "block-32 activation quant + tcgen05 INT8 GEMM with per-block fp32 rescale",
                  "glue": "embedding, RMSNorm, bias + RoPE + KV write, causal attention (fp32), SiLU * up; "
                          "the last token through the output norm, the head and greedy selection",
                  "l2": "inputs larger than L2 (1.4 GB of repacked weights per step)",
                  "parallelism": f"replicas x{world}"}
        base = {"metric": "prefill tok/s", "unit": "tok/s",
                "dtype": "int8 x int8 -> int32 per 32-block (tcgen05 kind::i8), fp32 rescale and glue"}
    else:
        config = {"workload": "c1: Q8_0 matvec 8960x1536 + block-32 activation quantisation",
                  "rows": C1_M, "k": C1_K, "weight_copies_rotated": C1_ROTATE,
                  "l2": "inputs larger than L2 (24 rotated weight copies, 351 MB)",
                  "parallelism": f"replicas x{world}"}
        base = {"metric": "quant matvec HBM GB/s", "unit": "GB/s", "dtype": "int8 x int8 -> int32, fp32 scale"}
    base.update({"n_gpus": world, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
                 "scaling": "strong" if args.workload in ("c4", "c5") else "weak", "vs_baseline": None,
                 "data": "synthetic (seeded random-init weights; quants uniform, fp16 scales |N(0,1)|*0.002)",
                 "config": config})

    if args.impl == "reference":
        if rank != 0:
            return
        t0 = time.perf_counter()
        line = dict(base)
        if args.workload == "c2":
            value, done, cores = c2_cpu(max(30.0, args.cpu_seconds), args.steps, dict(C2, kv_type=KV_TYPES[args.kv]))
            sample = (f"{done} decode tokens at the last positions of the 512 context, oracle/decode_ref.py "
                      f"(numpy glue, oracle/ugb_oracle.c matvecs on POSIX threads over rows)")
            ms = 1e3 / value
        elif args.workload in ("c4", "c5"):
            value, per_token, cores = big_cpu(max(30.0, args.cpu_seconds), args.workload, 1)
            sample = ("1- and 2-layer oracle models of the config's shapes (oracle/decode_ref.py, matvecs on POSIX "
                      "threads), per-token time extrapolated to the full depth; one sequence at a time")
            ms = per_token * 1e3
        elif args.workload == "c3":
            value, toks, cores = c3_cpu(max(30.0, args.cpu_seconds), kv_type=KV_TYPES[args.kv])
            sample = (f"a {toks}-token prompt through the full 28-layer prefill (oracle/decode_ref.py "
                      f"RefDecoder.prefill: batched oracle/ugb_oracle.c matvecs on POSIX threads, numpy glue)")
            ms = C3_TOKENS / value * 1e3
        else:
            value, cores = c1_cpu(300)
            sample = "300 steps of quant_act + Q8_0 matvec 8960x1536 (oracle/ugb_oracle.c, POSIX threads over rows)"
            ms = C1_BYTES / value / 1e6
        line.update({"impl": "reference", "value": value, "ms_per_step": ms,
                     "cpu_baseline": {"value": value, "unit": base["unit"], "cores": cores, "kind": "port",
                                      "sample": sample},
                     "e2e": {"value": value, "unit": base["unit"], "h2d_bytes_per_step": 0,
                             "d2h_bytes_per_step": 0},
                     "wall_s": time.perf_counter() - t0})
        print(json.dumps(line))
        return

    import torch
    if world > 1:
        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local)
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    ugb = importlib.import_module("uefi-gpu_b200")
    ctx = ugb.Context(torch.cuda.current_device())
    decoder_path = None
    if args.workload == "c2":
        res = c2_gpu(args, ugb, ctx, torch, rank, world)
        if res["path"] == ugb.PATH_TOKEN:
            kernel = "token_kernel<Q8_0,Q8_0> (the whole decode step, one persistent launch per token)"
            traffic = load_traffic("c2_token")
            decoder_path = "token kernel: one persistent cooperative launch per token, 1 CTA per SM"
        else:
            kernel = "mv_rows_kernel<Q8_0> (fused gate/up, 17920x1536)"
            traffic = load_traffic("c2_gate_up")
            decoder_path = "launch chain: 256 kernels per token, captured as one CUDA graph"
    elif args.workload in ("c4", "c5"):
        res = big_gpu(args, ugb, ctx, torch, rank, world, args.workload)
        kernel = None
        traffic = None
        decoder_path = ("token kernel: one persistent cooperative launch per token" if res["path"] == ugb.PATH_TOKEN
                        else "launch chain captured as one CUDA graph")
    elif args.workload == "c3":
        res = c3_gpu(args, ugb, ctx, torch, rank, world)
        kernel = "prefill_gemm_kernel<128> (fused gate/up, 512 x 17920 x 1536)"
        traffic = load_traffic("c3_gate_up")
    else:
        res = c1_gpu(args, ugb, ctx, torch, rank, world)
        kernel = "mv_rows_kernel<Q8_0, burst> (8960x1536, ugb_matvec back to back under PDL)"
        traffic = load_traffic("c1_matvec")

    line = dict(base)
    if "step_bytes" in res:
        achieved = res["step_bytes"] / (res["ms_per_step"] / 1e3) / 1e9
        roof = {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                "frac": achieved / hbm_peak, "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
                "kernel": "whole decode step (one device)", "bytes_per_step": res["step_bytes"],
                "traffic": None}
    elif "kernel_ops" in res:
        achieved = res["kernel_ops"] / (res["kernel_ms"] / 1e3) / 1e12
        roof = {"bound": "tensor", "achieved": achieved, "peak": res["int8_tops"], "unit": "TOPS (int8)",
                "frac": achieved / res["int8_tops"],
                "peak_source": "measured in this run: cuBLAS int8 GEMM 8192^3 (torch._int_mm), burst",
                "kernel": kernel, "kernel_ms": res["kernel_ms"], "ops_per_launch": res["kernel_ops"],
                "traffic": traffic}
        if "step_gemm_ops" in res:  # the GEMMs' share of the whole prefill step
            step_tops = res["step_gemm_ops"] / (res["ms_per_step"] / 1e3) / 1e12
            roof["step"] = {"gemm_int8_ops": res["step_gemm_ops"], "attention_fp32_flops": res["step_attn_flops"],
                            "gemm_tops_over_step": step_tops, "frac": step_tops / res["int8_tops"]}
    else:
        achieved = res["kernel_bytes"] / (res["kernel_ms"] / 1e3) / 1e9
        roof = {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                "frac": achieved / hbm_peak, "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)"
                if peak_kind == "measured" else "fallback 6650 GB/s",
                "kernel": kernel, "kernel_ms": res["kernel_ms"], "bytes_per_launch": res["kernel_bytes"],
                "traffic": traffic}
    line.update({
        "value": res["value"], "ms_per_step": res["ms_per_step"], "roofline": roof,
        "e2e": res["e2e"], "gpu_launches": res["gpu_launches"], "clocks": res["clocks"],
    })
    if decoder_path:
        line["decoder_path"] = decoder_path
    if res.get("kv_other"):
        line["kv_fp32"] = res["kv_other"]
    if args.workload == "c2" and (args.sharded == "on" or (args.sharded == "auto" and world > 1)):
        line["sharded"] = sharded_gpu(args, ugb, ctx, torch, rank, world)
    if "token_bytes" in res:
        step_gbs = res["token_bytes"] / (res["ms_per_step"] / 1e3) / 1e9
        line["roofline"]["step"] = {"bytes_per_token": res["token_bytes"], "achieved": step_gbs,
                                    "frac": step_gbs / hbm_peak}
    if rank == 0 and world == 1:
        if args.workload == "c2":
            v, done, cores = c2_cpu(args.cpu_seconds, 64, dict(C2, kv_type=KV_TYPES[args.kv]))
            sample = f"{done} decode tokens (oracle/decode_ref.py; matvecs on the host threads)"
        elif args.workload in ("c4", "c5"):
            v, _, cores = big_cpu(args.cpu_seconds, args.workload, 1)
            sample = "1- and 2-layer oracle models, per-token time extrapolated to the full depth"
        elif args.workload == "c3":
            v, toks, cores = c3_cpu(args.cpu_seconds, kv_type=KV_TYPES[args.kv])
            sample = f"a {toks}-token prompt through the full 28-layer oracle prefill on the host threads"
        else:
            v, cores = c1_cpu(100)
            sample = "100 steps of quant_act + Q8_0 matvec 8960x1536 on the host cores"
        line["cpu_baseline"] = {"value": v, "unit": base["unit"], "cores": cores, "kind": "port",
                                "sample": sample}
    if rank == 0:
        print(json.dumps(line))
    ctx.close()
    if world > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
