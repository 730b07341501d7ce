"""Benchmark of the B200 quantized linear-layer hot path (libugb) -- one JSON line on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload W]

Workloads:
  c1  Q8_0 matvec 8960x1536 with block-32 activation quantisation.  A step is
      quant_act + linear on one fp32 vector; weights rotate over 24 copies (350 MB > L2) so
      every step streams its matrix from HBM.

Multi-GPU: one process per GPU (torchrun), each an independent replica of the workload
("replicas only": a single matvec has no exchange step); value = all ranks' units / the
slowest rank's time (max over ranks of CUDA-event time).

The reference arm (--impl reference) times the CPU restatement of the reference path
(oracle/, the reference Rust cannot be built here) on the host cores with all threads, on
the same workload, metric and unit.
"""
from __future__ import annotations

import argparse
import ctypes
import importlib
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

Q8_0 = 8
C1_K, C1_M = 1536, 8960
C1_ROTATE = 24


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
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

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
                 "--format=csv,noheader,nounits", "-lms", "200"],
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


# ---- workload c1 ----------------------------------------------------------------------------

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
        # quant_act + linear (gpu_graph.rs:74-80); the matvec prefetches its weights while the
        # quantiser runs (programmatic dependent launch)
        j = i % C1_ROTATE
        ctx.quant_q8_1(xs[j], xq, C1_K, 1)
        ctx.matvec(Q8_0, ws[j], rb, xq, y, C1_K, C1_M, 1)

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
    launches = 2 * args.steps  # quant_q8_1 + matvec per step

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


# ---- plumbing ---------------------------------------------------------------------------------

def barrier(world, torch):
    if world > 1:
        torch.distributed.barrier()


def reduce_max(v: float, world: int, torch) -> float:
    if world == 1:
        return v
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["c1"], default="c1")
    ap.add_argument("--cpu-samples", type=int, default=300)
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    hbm_peak, _, peak_kind = load_peaks()
    config = {"workload": "c1: Q8_0 matvec 8960x1536 + block-32 activation quantisation",
              "rows": C1_M, "k": C1_K, "weight_copies_rotated": C1_ROTATE,
              "l2": "inputs larger than L2 (24 rotated weight copies, 351 MB)",
              "parallelism": f"replicas x{world}"}
    base = {"metric": "quant matvec HBM GB/s", "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8 x int8 -> int32, fp32 scale",
            "data": "synthetic (seeded; quants uniform, fp16 scales |N(0,1)|*0.002)",
            "config": config}

    if args.impl == "reference":
        if rank != 0:
            return
        t0 = time.perf_counter()
        value, cores = c1_cpu(args.cpu_samples)
        steps = args.steps
        line = dict(base)
        line.update({"impl": "reference", "value": value, "n_gpus": world,
                     "ms_per_step": C1_BYTES / value / 1e6,
                     "cpu_baseline": {"value": value, "unit": "GB/s", "cores": cores,
                                      "kind": "port",
                                      "sample": f"{args.cpu_samples} steps of quant_act + Q8_0 matvec 8960x1536 "
                                                f"(oracle/ugb_oracle.c, POSIX threads over rows)"},
                     "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0,
                             "d2h_bytes_per_step": 0},
                     "wall_s": time.perf_counter() - t0})
        line["steps"] = steps
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
    res = c1_gpu(args, ugb, ctx, torch, rank, world)

    kern_bytes = res["kernel_bytes"]
    achieved = kern_bytes / (res["kernel_ms"] / 1e3) / 1e9
    line = dict(base)
    line.update({
        "value": res["value"], "ms_per_step": res["ms_per_step"],
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                     "frac": achieved / hbm_peak, "peak_source": peak_kind,
                     "kernel": "mv_rows_kernel<Q8_0>", "kernel_ms": res["kernel_ms"],
                     "traffic": load_traffic("c1_matvec")},
        "e2e": res["e2e"], "gpu_launches": res["gpu_launches"], "clocks": res["clocks"],
    })
    if rank == 0 and world == 1:
        v, cores = c1_cpu(max(20, args.cpu_samples // 3))
        line["cpu_baseline"] = {"value": v, "unit": "GB/s", "cores": cores, "kind": "port",
                                "sample": f"{max(20, args.cpu_samples // 3)} steps of quant_act + "
                                          f"Q8_0 matvec 8960x1536 on the host cores"}
    if rank == 0:
        print(json.dumps(line))
    ctx.close()
    if world > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
