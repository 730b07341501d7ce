"""Host logic of the sharded paths on CPU, as two gloo ranks (no GPU):

* the shard ranges bench.py gives each rank cover the vocabulary / the experts exactly once;
* expert parallelism: every rank's partial MoE sum (the oracle's expert FFN restricted to the
  experts it holds), all-reduced, equals the single-device result;
* vocabulary split: every rank's greedy key over its head rows (the (value, complemented id)
  order the kernels use), all-reduced with max, decodes to the global first maximum.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

Q8_0, Q3_K = 8, 11


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def greedy_key(v: np.float32, i: int) -> int:
    """The device's order-preserving 64-bit greedy key (value bits, complemented id)."""
    b = int(np.float32(v).view(np.uint32))
    b = (~b & 0xFFFFFFFF) if b & 0x80000000 else (b | 0x80000000)
    return (b << 32) | (~i & 0xFFFFFFFF)


def _q8_matrix(rng, k, m):
    b = np.empty((m, k // 32, 34), np.uint8)
    b[:, :, 2:] = rng.integers(-127, 128, (m, k // 32, 32), dtype=np.int8).view(np.uint8)
    b[:, :, :2] = (0.002 * np.abs(rng.standard_normal((m, k // 32)))).astype(np.float16).view(np.uint8).reshape(m, -1, 2)
    return b.reshape(-1)


def _moe_layer(seed, d, ne, ff):
    rng = np.random.default_rng(seed)
    return {"router": _q8_matrix(rng, d, ne), "gate_exps": _q8_matrix(rng, d, ff * ne),
            "up_exps": _q8_matrix(rng, d, ff * ne), "down_exps": _q8_matrix(rng, ff, d * ne)}


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=60))
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import bench
    from oracle.decode_ref import RefDecoder
    ok = {}
    # shard ranges
    c4 = bench.shard_config(dict(bench.C4), "c4", rank, world)
    c5 = bench.shard_config(dict(bench.C5), "c5", rank, world)
    spans = [None] * world
    dist.all_gather_object(spans, ((c4["vocab0"], c4["n_vocab_local"]), (c5["expert0"], c5["n_expert_local"])))
    v = sorted(s[0] for s in spans)
    e = sorted(s[1] for s in spans)
    ok["vocab_cover"] = v[0][0] == 0 and all(a[0] + a[1] == b[0] for a, b in zip(v, v[1:])) and \
        v[-1][0] + v[-1][1] == bench.C4["n_vocab"]
    ok["expert_cover"] = e[0][0] == 0 and all(a[0] + a[1] == b[0] for a, b in zip(e, e[1:])) and \
        e[-1][0] + e[-1][1] == bench.C5["n_expert"]
    # expert parallelism: partial sums add up to the full MoE FFN
    d, ne, ff = 256, 8, 64
    cfg = dict(n_layer=1, n_embd=d, n_head=2, n_head_kv=1, head_dim=128, n_vocab=16, n_ctx=4, rope_theta=1e6,
               norm_eps=1e-6, kind=Q8_0, head_kind=Q8_0, n_expert=ne, top_k=3, n_ff_expert=ff, expert_kind=Q8_0)
    ref = RefDecoder(cfg, {"layers": []})
    L = _moe_layer(5, d, ne, ff)
    xn = np.random.default_rng(6).standard_normal(d).astype(np.float32)
    per = ne // world
    mine = range(rank * per, ne if rank == world - 1 else (rank + 1) * per)
    part = torch.from_numpy(ref.moe_ffn(L, xn, mine))
    dist.all_reduce(part)
    full = ref.moe_ffn(L, xn)
    ok["ep_sum"] = bool(np.allclose(part.numpy(), full, rtol=1e-5, atol=1e-6 * np.abs(full).max()))
    # vocabulary split: max over the ranks' keys is the global first maximum
    logits = np.random.default_rng(7).standard_normal(1000).astype(np.float32)
    logits[[123, 777]] = logits.max() + 1  # a tie across the two halves: the lower id must win
    vper = -(-1000 // world)
    lo, hi = rank * vper, min(1000, (rank + 1) * vper)
    key = max(greedy_key(logits[i], i) for i in range(lo, hi))
    t = torch.tensor([key ^ (1 << 63)], dtype=torch.int64)  # signed compare == unsigned compare
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    won = (int(t.item()) ^ (1 << 63)) & 0xFFFFFFFFFFFFFFFF
    ok["vocab_argmax"] = (~won & 0xFFFFFFFF) == int(np.argmax(logits)) == 123
    out[rank] = ok
    dist.destroy_process_group()


def test_sharding_host_logic_two_ranks():
    world = 2
    port = _free_port()
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    for p in procs:
        if p.is_alive():
            p.kill()
            pytest.fail("gloo rank did not finish")
        assert p.exitcode == 0
    for r in range(world):
        assert out[r] == {"vocab_cover": True, "expert_cover": True, "ep_sum": True, "vocab_argmax": True}, out[r]
