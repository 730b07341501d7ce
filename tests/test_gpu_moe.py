"""GPU parity of the MoE expert path against the CPU oracle, through the C ABI.

* ugb_matvec_jobs (the FrontierJob table): every job equals the same matvec launched alone,
  bit for bit, and the oracle within 1e-3 per row; mixed kinds and row lengths in one table;
  the reference packer's rejections (overlapping outputs, inconsistent row_bytes, > 32 jobs).
* ugb_moe_route: expert ids equal the oracle's softmax / top-k (ties to the lower id), weights
  within 1e-6 relative.
* ugb_moe_experts: checked stage by stage from the workspace (each stage against the oracle
  applied to the GPU's previous stage, so one activation rounding flip cannot cascade): gate/up
  rows within 1e-3, the SiLU quants equal up to one step where exp's last ulp decides a
  rounding (scales within 1e-6), the down rows within 1e-3, the combine bit-exact.
  Expert-parallel shards (accumulate) sum to the single-device result.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import assert_rows_close

pytestmark = pytest.mark.gpu

Q8_0, Q3_K, Q4_K = 8, 11, 12
Q6_K, IQ3_XXS, IQ4_NL, IQ4_XS = 14, 18, 20, 23


def _torch():
    import torch
    return torch


def synth(ctx, ugb, kind, k, m, seed):
    torch = _torch()
    w = torch.empty(ugb.row_bytes(kind, k) * m, dtype=torch.uint8, device="cuda")
    ctx.fill_synthetic(kind, w, k, m, seed)
    return w


def quantized(ctx, ugb, x_np):
    torch = _torch()
    batch, k = x_np.shape
    xq = ugb.alloc_q8act(k, batch)
    ctx.quant_q8_1(torch.from_numpy(np.ascontiguousarray(x_np, np.float32)).cuda(), xq, k, batch)
    return xq


def host_act(ugb, xq, k, batch):
    q, d, s = ugb.split_q8act(xq, k, batch)
    nb = k // 32
    return (q.cpu().numpy(), np.ascontiguousarray(d[:, :nb].cpu().numpy()),
            np.ascontiguousarray(s[:, :nb].cpu().numpy()))


def oracle_mv(orc, ugb, kind, w_np, k, m, q, d, s, batch=1):
    return orc.matvec(kind, w_np, ugb.row_bytes(kind, k), q, d, s, k, m, batch)


# ---- job table ----------------------------------------------------------------------------------

@pytest.mark.parametrize("batch", [1, 3])
def test_jobs_equal_single_launches(ctx, ugb, orc, batch):
    torch = _torch()
    shapes = [(Q8_0, 1536, 300), (Q3_K, 4096, 1536), (Q4_K, 1536, 700), (Q8_0, 1536, 8), (Q3_K, 4096, 96),
              (Q3_K, 1536, 4096), (Q6_K, 4096, 200), (IQ3_XXS, 1536, 300), (IQ4_NL, 1536, 64),
              (IQ4_XS, 4096, 96)]
    rng = np.random.default_rng(batch)
    jobs, outs, singles, xs = [], [], [], {}
    for i, (kind, k, m) in enumerate(shapes):
        w = synth(ctx, ugb, kind, k, m, seed=100 + i)
        if k not in xs:
            x = rng.standard_normal((batch, k)).astype(np.float32)
            xs[k] = (x, quantized(ctx, ugb, x))
        xq = xs[k][1]
        y = torch.full((batch, m), float("nan"), device="cuda")
        y1 = torch.empty((batch, m), device="cuda")
        ctx.matvec(kind, w, ugb.row_bytes(kind, k), xq, y1, k, m, batch)
        jobs.append(ugb.Job(w.data_ptr(), xq.data_ptr(), y.data_ptr(), kind, k, m, ugb.row_bytes(kind, k), 0, 0))
        outs.append((kind, k, m, w, y))
        singles.append(y1)
    ctx.matvec_jobs(jobs, batch)
    torch.cuda.synchronize()
    for (kind, k, m, w, y), y1 in zip(outs, singles):
        got = y.cpu().numpy()
        np.testing.assert_array_equal(got.view(np.uint32), y1.cpu().numpy().view(np.uint32))
        q, d, s = host_act(ugb, xs[k][1], k, batch)
        want = oracle_mv(orc, ugb, kind, w.cpu().numpy(), k, m, q, d, s, batch)
        for b in range(batch):
            assert_rows_close(got[b], want[b])
    assert ctx.status_read()[1] == 0


def test_jobs_rejections(ctx, ugb):
    torch = _torch()
    w = synth(ctx, ugb, Q8_0, 64, 16, seed=1)
    xq = quantized(ctx, ugb, np.ones((1, 64), np.float32))
    y = torch.empty(64, device="cuda")
    rb = ugb.row_bytes(Q8_0, 64)
    ok = ugb.Job(w.data_ptr(), xq.data_ptr(), y.data_ptr(), Q8_0, 64, 16, rb, 0, 0)
    overlap = ugb.Job(w.data_ptr(), xq.data_ptr(), y.data_ptr() + 32, Q8_0, 64, 16, rb, 0, 0)
    bad_rb = ugb.Job(w.data_ptr(), xq.data_ptr(), y.data_ptr() + 128, Q8_0, 64, 16, rb + 1, 0, 0)
    empty = ugb.Job(w.data_ptr(), xq.data_ptr(), y.data_ptr() + 128, Q8_0, 64, 0, rb, 0, 0)
    for table in ([ok, overlap], [ok, bad_rb], [ok, empty], [ok] * 33):
        with pytest.raises(ugb.UgbError):
            ctx.matvec_jobs(table)
    ctx.matvec_jobs([ok])


# ---- routing --------------------------------------------------------------------------------------

@pytest.mark.parametrize("n_expert,top_k,batch", [(192, 8, 8), (512, 10, 1), (16, 4, 3)])
def test_route_matches_oracle(ctx, ugb, orc, n_expert, top_k, batch):
    torch = _torch()
    rng = np.random.default_rng(n_expert + top_k)
    logits = (rng.standard_normal((batch, n_expert)) * 3).astype(np.float32)
    if batch > 1:
        logits[1, 5] = logits[1, 9] = logits[1, 200 % n_expert] = logits[1].max() + 1  # exact ties
    ids = torch.empty((batch, top_k), dtype=torch.int32, device="cuda")
    wts = torch.empty((batch, top_k), dtype=torch.float32, device="cuda")
    ctx.moe_route(torch.from_numpy(logits).cuda(), n_expert, top_k, batch, ids, wts)
    ids, wts = ids.cpu().numpy(), wts.cpu().numpy()
    for t in range(batch):
        oid, ow = orc.moe_route(logits[t], top_k)
        np.testing.assert_array_equal(ids[t], oid)
        np.testing.assert_allclose(wts[t], ow, rtol=1e-6, atol=0)
    if batch > 1:
        tied = sorted({5, 9, 200 % n_expert})
        assert list(ids[1, :len(tied)]) == tied


def test_route_nonfinite(ctx, ugb):
    torch = _torch()
    logits = torch.zeros((2, 16), device="cuda")
    logits[1, 3] = float("inf")
    ids = torch.empty((2, 4), dtype=torch.int32, device="cuda")
    wts = torch.empty((2, 4), device="cuda")
    ctx.moe_route(logits, 16, 4, 2, ids, wts)
    code, bits = ctx.status_read()
    assert bits & ugb.STATUS_NONFINITE_IN
    assert (ids[1] == -1).all() and (ids[0] >= 0).all()


# ---- routed experts ---------------------------------------------------------------------------------

def run_experts(ctx, ugb, kind, hidden, ffn, n_total, top_k, batch, shards, seed):
    """Stacked expert tensors, routing of random logits, and ugb_moe_experts over `shards`
    (list of (expert0, n_expert)) accumulating into one output."""
    torch = _torch()
    gate = synth(ctx, ugb, kind, hidden, ffn * n_total, seed)
    up = synth(ctx, ugb, kind, hidden, ffn * n_total, seed + 1)
    down = synth(ctx, ugb, kind, ffn, hidden * n_total, seed + 2)
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((batch, hidden)).astype(np.float32)
    xq = quantized(ctx, ugb, x)
    logits = torch.from_numpy(rng.standard_normal((batch, n_total)).astype(np.float32)).cuda()
    ids = torch.empty((batch, top_k), dtype=torch.int32, device="cuda")
    wts = torch.empty((batch, top_k), device="cuda")
    ctx.moe_route(logits, n_total, top_k, batch, ids, wts)
    out = torch.full((batch, hidden), float("nan"), device="cuda")
    wsb = ugb.moe_workspace_bytes(hidden, ffn, top_k, batch)
    wss = []
    for i, (e0, n) in enumerate(shards):
        ws = torch.full((wsb,), 255, dtype=torch.uint8, device="cuda")
        rbi, rbf = ugb.row_bytes(kind, hidden), ugb.row_bytes(kind, ffn)
        args = ugb.MoeArgs(kind, 1 if i else 0, hidden, ffn, top_k, batch, n, e0, n_total,
                           gate.data_ptr() + e0 * ffn * rbi, up.data_ptr() + e0 * ffn * rbi,
                           down.data_ptr() + e0 * hidden * rbf, xq.data_ptr(), ids.data_ptr(), wts.data_ptr(),
                           out.data_ptr(), ws.data_ptr(), wsb)
        ctx.moe_experts(args)
        wss.append(ws)
    torch.cuda.synchronize()
    return dict(gate=gate, up=up, down=down, xq=xq, ids=ids.cpu().numpy(), wts=wts.cpu().numpy(),
                out=out.cpu().numpy(), ws=[w.cpu().numpy() for w in wss])


@pytest.mark.parametrize("kind,hidden,ffn,n_total,top_k,batch", [
    (Q3_K, 1024, 512, 16, 4, 1), (Q3_K, 1024, 512, 16, 4, 3), (Q8_0, 512, 256, 8, 2, 8),
    (Q4_K, 512, 256, 12, 3, 2), (IQ3_XXS, 1024, 512, 16, 4, 1), (Q6_K, 512, 256, 8, 2, 3),
    (IQ4_XS, 512, 256, 8, 2, 2), (IQ4_NL, 512, 256, 8, 2, 1)])
def test_moe_experts_stagewise(ctx, ugb, orc, kind, hidden, ffn, n_total, top_k, batch):
    r = run_experts(ctx, ugb, kind, hidden, ffn, n_total, top_k, batch, [(0, n_total)], seed=7)
    lay = ugb.moe_workspace_layout(hidden, ffn, top_k, batch)
    slots = lay["slots"]
    ws = r["ws"][0]
    gu = ws[lay["gu"]:lay["gu"] + slots * 2 * ffn * 4].view(np.float32).reshape(slots, 2 * ffn)
    hq_buf = ws[lay["hq"]:lay["hq"] + ugb.q8act_bytes(ffn, slots)]
    values = ws[lay["values"]:lay["values"] + slots * hidden * 4].view(np.float32).reshape(slots, hidden)
    q, d, s = host_act(ugb, r["xq"], hidden, batch)
    rbi, rbf = ugb.row_bytes(kind, hidden), ugb.row_bytes(kind, ffn)
    gate, up, down = r["gate"].cpu().numpy(), r["up"].cpu().numpy(), r["down"].cpu().numpy()
    # stage 1: gate / up rows of each slot's expert
    for sl in range(slots):
        t, e = sl // top_k, int(r["ids"].flat[sl])
        g = oracle_mv(orc, ugb, kind, gate[e * ffn * rbi:(e + 1) * ffn * rbi], hidden, ffn, q[t:t + 1], d[t:t + 1], s[t:t + 1])
        u = oracle_mv(orc, ugb, kind, up[e * ffn * rbi:(e + 1) * ffn * rbi], hidden, ffn, q[t:t + 1], d[t:t + 1], s[t:t + 1])
        assert_rows_close(gu[sl], np.concatenate([g[0], u[0]]))
    # stage 2: SiLU(gate) * up quantised from the GPU's own gate/up.  numpy's exp and CUDA's
    # expf may differ by an ulp, so a scale may move by an ulp and a quant on a rounding
    # boundary by one step; everything else is exact.
    g32, u32 = gu[:, :ffn], gu[:, ffn:]
    with np.errstate(over="ignore"):
        h = (g32 / (np.float32(1) + np.exp(-g32)) * u32).astype(np.float32)
    qh, dh, _, _ = orc.quant_act(h)
    nbh = ffn // 32
    nbp = (nbh + 3) // 4 * 4
    hq_q = hq_buf[:slots * ffn].view(np.int8).reshape(slots, ffn)
    d_off = (slots * ffn + 255) // 256 * 256
    s_off = d_off + (slots * nbp * 4 + 255) // 256 * 256
    hq_d = np.ascontiguousarray(hq_buf[d_off:d_off + slots * nbp * 4].view(np.float32).reshape(slots, nbp)[:, :nbh])
    hq_s = np.ascontiguousarray(hq_buf[s_off:s_off + slots * nbp * 4].view(np.int32).reshape(slots, nbp)[:, :nbh])
    diff = np.abs(hq_q.astype(np.int32) - qh.astype(np.int32))
    assert diff.max() <= 1 and (diff > 0).sum() <= max(2, diff.size // 10000)
    np.testing.assert_allclose(hq_d, dh, rtol=1e-6, atol=0)
    np.testing.assert_array_equal(hq_s, hq_q.reshape(slots, nbh, 32).astype(np.int32).sum(-1))
    # stage 3: down rows from the GPU's own quantised h
    for sl in range(slots):
        e = int(r["ids"].flat[sl])
        v = oracle_mv(orc, ugb, kind, down[e * hidden * rbf:(e + 1) * hidden * rbf], ffn, hidden,
                      np.ascontiguousarray(hq_q[sl:sl + 1]), hq_d[sl:sl + 1], hq_s[sl:sl + 1])
        assert_rows_close(values[sl], v[0])
    # stage 4: combine in rank order, separate multiply and add
    want = np.zeros((batch, hidden), np.float32)
    for t in range(batch):
        for k in range(top_k):
            want[t] = want[t] + np.float32(r["wts"][t, k]) * values[t * top_k + k]
    np.testing.assert_array_equal(r["out"].view(np.uint32), want.view(np.uint32))
    assert ctx.status_read()[1] == 0


def test_moe_expert_parallel_shards_sum(ctx, ugb):
    kind, hidden, ffn, n_total, top_k, batch = Q3_K, 1024, 512, 16, 4, 3
    full = run_experts(ctx, ugb, kind, hidden, ffn, n_total, top_k, batch, [(0, n_total)], seed=3)
    split = run_experts(ctx, ugb, kind, hidden, ffn, n_total, top_k, batch, [(0, 5), (5, 7), (12, 4)], seed=3)
    np.testing.assert_array_equal(full["ids"], split["ids"])
    np.testing.assert_allclose(split["out"], full["out"], rtol=2e-6, atol=1e-6 * np.abs(full["out"]).max())
    assert ctx.status_read()[1] == 0
