"""Two-GPU parity of the sharded decoder (skipped with fewer than two GPUs).

Each rank is a process on its own GPU with the library's NCCL communicator; a gloo process
group carries the communicator id and a barrier (with a timeout) before every step, so a rank
that fails is noticed on the host before the other enters a collective.
* the library's own all-reduce over NVLink peer memory (sum f32, max u64) gives every rank the
  rank-order result bit for bit, across repeated calls and sizes up to 32768 values;
* vocabulary split: each rank holds half of the head rows; the greedy keys are all-reduced
  inside the token step.  The next tokens equal a single-GPU decoder's, and each rank's
  logits equal that decoder's logits over the held rows, bit for bit.
* expert parallelism: each rank holds half of every MoE layer's experts; the layer outputs
  are all-reduced inside the step.  The sum is associated differently from one device's
  rank-order sum, so (as in the oracle comparisons) most steps agree within 1e-4 and every step
  within 5e-2.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

Q8_0, Q3_K = 8, 11
SMALL = dict(n_layer=2, n_embd=256, n_ff=512, n_head=4, n_head_kv=2, head_dim=128, n_vocab=1000,
             n_ctx=64, rope_theta=1e6, norm_eps=1e-6, kind=Q8_0, head_kind=Q8_0)
MOE = dict(SMALL, n_ff=0, n_expert=8, top_k=2, n_ff_expert=256, expert_kind=Q3_K)


def _gpus() -> int:
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    import datetime
    import importlib
    import sys
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    ugb = importlib.import_module("uefi-gpu_b200")
    ctx = ugb.Context(rank)
    uid = [ugb.comm_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    comm = ugb.Comm(ctx, rank, world, uid[0])
    res = {}
    # -- the collectives themselves: every rank gets the rank-order sum / maximum, bit for bit,
    # over several calls (both buffer parities), unaligned and multi-slice sizes included --
    ok_sum, ok_max = True, True
    for call, n in enumerate([1, 4096, 4099, 32768, 7, 4096]):
        data = [np.random.default_rng(100 * call + r).standard_normal(n).astype(np.float32) for r in range(world)]
        want = data[0].copy()
        for r in range(1, world):
            want = (want + data[r]).astype(np.float32)
        buf = torch.from_numpy(data[rank].copy()).cuda()
        comm.allreduce_f32(buf)
        ok_sum &= bool(np.array_equal(buf.cpu().numpy().view(np.uint32), want.view(np.uint32)))
        keys = [np.random.default_rng(7 * call + r).integers(0, 2 ** 62, size=max(1, n // 1024)) for r in range(world)]
        kbuf = torch.from_numpy(keys[rank].copy()).cuda()
        comm.allreduce_max_u64(kbuf)
        ok_max &= bool(np.array_equal(kbuf.cpu().numpy(), np.max(np.stack(keys), axis=0)))
    res["allreduce_sum"], res["allreduce_max"] = ok_sum, ok_max
    # -- vocabulary split --
    half = SMALL["n_vocab"] // world
    shard = ugb.Decoder(ctx, **dict(SMALL, vocab0=rank * half, n_vocab_local=half))
    shard.synthetic(5)
    shard.set_comm(comm)
    full = ugb.Decoder(ctx, **SMALL)
    full.synthetic(5)
    full.set_path(ugb.PATH_CHAIN)  # the sharded head runs the launch chain: compare like with like
    tok, same_tok, same_logits = 3, True, True
    for pos in range(10):
        dist.barrier()
        nxt = shard.token(tok, pos)
        ref = full.token(tok, pos)
        same_tok &= nxt == ref
        same_logits &= bool(np.array_equal(shard.logits().view(np.uint32),
                                           full.logits()[rank * half:(rank + 1) * half].view(np.uint32)))
        tok = ref
    res["vocab_tokens"], res["vocab_logits"] = same_tok, same_logits
    shard.close()
    full.close()
    # -- expert parallelism --
    per = MOE["n_expert"] // world
    ep = ugb.Decoder(ctx, **dict(MOE, expert0=rank * per, n_expert_local=per))
    ep.synthetic(6)
    ep.set_comm(comm)
    full = ugb.Decoder(ctx, **MOE)
    full.synthetic(6)
    errs = []
    rng = np.random.default_rng(1)
    for pos in range(16):
        t = int(rng.integers(0, SMALL["n_vocab"]))
        dist.barrier()
        ep.token(t, pos)
        full.token(t, pos)
        a, b = ep.logits().astype(np.float64), full.logits().astype(np.float64)
        errs.append(float(np.linalg.norm(a - b) / np.linalg.norm(b)))
    res["ep_errs"] = errs
    res["status"] = ctx.status_read()[1]
    dist.barrier()
    ep.close()
    full.close()
    comm.close()
    ctx.close()
    out[rank] = res
    dist.destroy_process_group()


@pytest.mark.skipif(_gpus() < 2, reason="needs two GPUs")
def test_sharded_decoder_two_gpus():
    import torch.multiprocessing as mp
    world = 2
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=400)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    for r in range(world):
        res = out[r]
        assert res["allreduce_sum"] and res["allreduce_max"], res
        assert res["vocab_tokens"] and res["vocab_logits"], res
        errs = np.array(res["ep_errs"])
        assert errs.max() <= 5e-2 and (errs <= 1e-4).mean() >= 0.6, errs
        assert res["status"] == 0
