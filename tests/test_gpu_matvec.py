"""GPU parity of the decode hot path against the CPU oracle, through the C ABI.

Integer block dots must be bit-exact; fp32 rows within 1e-3 relative (assert_rows_close);
activation quants and scales bit-exact.  Shapes cover the configs (C1 8960x1536 Q8_0, the
1.5B / 7B / MoE matrices) and ragged edges: row counts that are not a multiple of the row
group, rows whose byte length is not a multiple of 16 (tail bytes past the last 16-byte
boundary), single-block rows, and batches 1..8 including non-powers of two.  The reference's
other formats (Q6_K, IQ3_XXS, IQ4_NL, IQ4_XS; frontier_core.rs:80-101) take the same checks.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import assert_rows_close, golden

pytestmark = pytest.mark.gpu

Q8_0, Q3_K, Q4_K = 8, 11, 12
Q6_K, IQ3_XXS, IQ4_NL, IQ4_XS = 14, 18, 20, 23
ELEMS = {Q8_0: 32, Q4_K: 256, Q3_K: 256, Q6_K: 256, IQ3_XXS: 256, IQ4_NL: 32, IQ4_XS: 256}


def _torch():
    import torch
    return torch


def make_weights(ctx, ugb, kind, k, m, seed):
    torch = _torch()
    rb = ugb.row_bytes(kind, k)
    w = torch.empty(rb * m + 64, dtype=torch.uint8, device="cuda")[: rb * m]
    ctx.fill_synthetic(kind, w, k, m, seed)
    return w, rb


def quantize(ctx, ugb, x_np):
    torch = _torch()
    batch, k = x_np.shape
    x = torch.from_numpy(np.ascontiguousarray(x_np, dtype=np.float32)).cuda()
    xq = ugb.alloc_q8act(k, batch)
    ctx.quant_q8_1(x, xq, k, batch)
    return xq


def host_act(ugb, xq, k, batch):
    q, d, s = ugb.split_q8act(xq, k, batch)
    nb = k // 32
    return (q.cpu().numpy(), np.ascontiguousarray(d[:, :nb].cpu().numpy()),
            np.ascontiguousarray(s[:, :nb].cpu().numpy()))


def test_quant_bit_exact_golden(ctx, ugb, orc):
    g = golden("quant_act.npz")
    x = g["x"].reshape(1, -1)
    k = x.shape[1]
    xq = quantize(ctx, ugb, x)
    q, d, s = host_act(ugb, xq, k, 1)
    np.testing.assert_array_equal(q[0], g["q"])
    np.testing.assert_array_equal(d[0].view(np.uint32), g["d"].view(np.uint32))
    np.testing.assert_array_equal(s[0], g["s"])
    assert ctx.status_read()[1] == 0


@pytest.mark.parametrize("k,batch", [(1536, 1), (8960, 3), (96, 8), (18944, 2)])
def test_quant_bit_exact_random(ctx, ugb, orc, k, batch):
    rng = np.random.default_rng(k + batch)
    x = (rng.standard_normal((batch, k)) * rng.uniform(0.01, 100)).astype(np.float32)
    xq = quantize(ctx, ugb, x)
    q, d, s = host_act(ugb, xq, k, batch)
    qo, do, so, bad = orc.quant_act(x)
    assert bad == 0
    np.testing.assert_array_equal(q, qo)
    np.testing.assert_array_equal(d.view(np.uint32), do.view(np.uint32))
    np.testing.assert_array_equal(s, so)


def test_quant_nonfinite_sets_status(ctx, ugb):
    x = np.ones((1, 64), dtype=np.float32)
    x[0, 5] = np.nan
    quantize(ctx, ugb, x)
    code, bits = ctx.status_read()
    assert code == ugb.ENONFINITE and bits & 1


SHAPES = [
    (Q8_0, 1536, 8960),    # C1 / gate,up of the 1.5B model
    (Q8_0, 8960, 1536),    # 1.5B down projection
    (Q8_0, 1536, 2048),    # fused QKV rows
    (Q8_0, 96, 13),        # 3 blocks per row: 102-byte rows, ragged row group, tail bytes
    (Q8_0, 32, 1),         # single block, single row
    (Q8_0, 1184, 37),      # 37 blocks: two chunks, odd block count
    (Q4_K, 3584, 300),     # 7B hidden
    (Q4_K, 18944, 77),     # 7B down projection (19 chunks)
    (Q4_K, 256, 5),
    (Q3_K, 4096, 200),     # MoE expert gate/up
    (Q3_K, 1536, 129),     # MoE expert down: 660-byte rows (not 16-byte multiples)
    (Q3_K, 256, 3),        # 110-byte rows
    (Q8_0, 32768, 21),     # rows longer than a pipeline stage: K split into 12 chunks
    (Q4_K, 24576, 9),      # K-chunked, ragged row group
    (Q3_K, 65536, 5),      # K-chunked Q3_K at UGB_MAX_K
    (Q8_0, 3584, 100),     # 7B output-head row length
    (Q8_0, 8960, 37),      # rows spread over all lanes, two per item, ragged last item
    (Q6_K, 4096, 200),     # the reference's other formats: Q6_K
    (Q6_K, 1536, 37),      # 1260-byte rows (not 16-byte multiples), ragged row group
    (IQ4_NL, 1536, 300),   # IQ4_NL: 18-byte blocks
    (IQ4_NL, 96, 13),      # 54-byte rows, tail bytes
    (IQ4_NL, 32768, 9),    # K-chunked IQ4_NL
    (IQ4_XS, 4096, 129),   # IQ4_XS: 136-byte super-blocks
    (IQ3_XXS, 1536, 129),  # IQ3_XXS: 588-byte rows
    (IQ3_XXS, 65536, 5),   # K-chunked IQ3_XXS at UGB_MAX_K
]


@pytest.mark.parametrize("kind,k,m", SHAPES)
def test_block_dots_bit_exact(ctx, ugb, orc, kind, k, m):
    torch = _torch()
    w, rb = make_weights(ctx, ugb, kind, k, m, seed=k * 7 + m)
    rng = np.random.default_rng(m)
    x = rng.standard_normal((1, k)).astype(np.float32)
    xq = quantize(ctx, ugb, x)
    out = torch.empty(m * (k // 32), dtype=torch.int32, device="cuda")
    ctx.block_dots(kind, w, rb, xq, out, k, m)
    got = out.cpu().numpy().reshape(m, k // 32)
    wh = w.cpu().numpy()
    q, d, s = host_act(ugb, xq, k, 1)
    for r in range(m):
        want = orc.block_dots(kind, wh[r * rb:(r + 1) * rb], q[0])
        np.testing.assert_array_equal(got[r], want, err_msg=f"row {r}")


@pytest.mark.parametrize("kind,k,m", SHAPES)
@pytest.mark.parametrize("batch", [1, 3, 8])
def test_matvec_rows_close(ctx, ugb, orc, kind, k, m, batch):
    torch = _torch()
    w, rb = make_weights(ctx, ugb, kind, k, m, seed=k + m)
    rng = np.random.default_rng(k * m + batch)
    x = rng.standard_normal((batch, k)).astype(np.float32)
    xq = quantize(ctx, ugb, x)
    y = torch.full((batch, m), float("nan"), dtype=torch.float32, device="cuda")
    ctx.matvec(kind, w, rb, xq, y, k, m, batch)
    got = y.cpu().numpy()
    q, d, s = host_act(ugb, xq, k, batch)
    ref = orc.matvec(kind, w.cpu().numpy(), rb, q, d, s, k, m, batch)
    assert_rows_close(got, ref)
    code, bits = ctx.status_read()
    assert code == ugb.OK, bits


def test_matvec_deterministic(ctx, ugb):
    torch = _torch()
    k, m = 1536, 8960
    w, rb = make_weights(ctx, ugb, Q8_0, k, m, seed=11)
    xq = quantize(ctx, ugb, np.random.default_rng(0).standard_normal((2, k)).astype(np.float32))
    ys = []
    for _ in range(3):
        y = torch.empty((2, m), dtype=torch.float32, device="cuda")
        ctx.matvec(Q8_0, w, rb, xq, y, k, m, 2)
        ys.append(y.cpu().numpy())
    assert np.array_equal(ys[0].view(np.uint32), ys[1].view(np.uint32))
    assert np.array_equal(ys[0].view(np.uint32), ys[2].view(np.uint32))


def test_matvec_head_full_size(ctx, ugb, orc):
    """The 1.5B tied output head, 151936 x 1536 Q8_0, against the oracle at full size."""
    torch = _torch()
    k, m = 1536, 151936
    w, rb = make_weights(ctx, ugb, Q8_0, k, m, seed=5)
    x = np.random.default_rng(9).standard_normal((1, k)).astype(np.float32)
    xq = quantize(ctx, ugb, x)
    y = torch.empty((1, m), dtype=torch.float32, device="cuda")
    ctx.matvec(Q8_0, w, rb, xq, y, k, m, 1)
    q, d, s = host_act(ugb, xq, k, 1)
    ref = orc.matvec(Q8_0, w.cpu().numpy(), rb, q, d, s, k, m, 1, mt=True)
    assert_rows_close(y.cpu().numpy(), ref)


def test_linear_host_api_matches_device_path(ctx, ugb, orc):
    """ugb_linear (Gpu::matvec / Weights::linear form) equals quant + matvec."""
    torch = _torch()
    k, m = 1536, 2048
    w, rb = make_weights(ctx, ugb, Q8_0, k, m, seed=3)
    x = ((np.arange(k) % 17) - 8).astype(np.float32) / 16  # llm.rs:302 check input
    y_host = ctx.linear(Q8_0, w, rb, x, k, m)
    xq = quantize(ctx, ugb, x.reshape(1, k))
    y = torch.empty((1, m), dtype=torch.float32, device="cuda")
    ctx.matvec(Q8_0, w, rb, xq, y, k, m, 1)
    np.testing.assert_array_equal(y_host.view(np.uint32), y.cpu().numpy()[0].view(np.uint32))
    # Parity against the oracle on the reference's check rows {0,1,17,127,1535}
    # (llm.rs:305).  The reference's 0.002 absolute gate there compares its fp32-activation
    # kernel (matvec_q8) with an fp32 dequant-dot; this path quantises activations per block
    # (quant_act), so it is held to the quantised oracle instead.
    q, d, s = host_act(ugb, xq, k, 1)
    ref = orc.matvec(Q8_0, w.cpu().numpy(), rb, q, d, s, k, m, 1)[0]
    rows = [0, 1, 17, 127, 1535]
    assert_rows_close(y_host[rows], ref[rows])


def test_linear_rejects_nonfinite(ctx, ugb):
    k, m = 256, 16
    w, rb = make_weights(ctx, ugb, Q8_0, k, m, seed=1)
    x = np.ones(k, dtype=np.float32)
    x[9] = np.inf
    with pytest.raises(ugb.UgbError) as e:
        ctx.linear(Q8_0, w, rb, x, k, m)
    assert e.value.code == ugb.ENONFINITE


def test_shape_and_alignment_errors(ctx, ugb):
    torch = _torch()
    k, m = 256, 16
    w, rb = make_weights(ctx, ugb, Q8_0, k, m, seed=1)
    xq = ugb.alloc_q8act(k, 1)
    y = torch.empty(m, dtype=torch.float32, device="cuda")
    lib = ugb.lib()
    s = torch.cuda.current_stream().cuda_stream
    assert lib.ugb_matvec(ctx.handle, s, Q8_0, w.data_ptr(), rb + 1, xq.data_ptr(), y.data_ptr(), k, m, 1) == ugb.ESHAPE
    assert lib.ugb_matvec(ctx.handle, s, 99, w.data_ptr(), rb, xq.data_ptr(), y.data_ptr(), k, m, 1) == ugb.EQUANT
    assert lib.ugb_matvec(ctx.handle, s, Q8_0, w.data_ptr() + 2, rb, xq.data_ptr(), y.data_ptr(), k, m, 1) == ugb.EALIGN
    assert lib.ugb_matvec(ctx.handle, s, Q8_0, w.data_ptr(), rb, xq.data_ptr(), y.data_ptr(), k, m, 9) == ugb.ESHAPE
    assert lib.ugb_matvec(ctx.handle, s, Q8_0, w.data_ptr(), rb, xq.data_ptr(), y.data_ptr(), 48, m, 1) == ugb.ESHAPE


@pytest.mark.parametrize("kind,k,rows,batch", [
    (Q8_0, 1536, (1536, 256, 256), 1),   # fused Q/K/V of the 1.5B model (qkv_dp4a)
    (Q8_0, 1536, (8960, 8960), 1),       # fused gate/up (gateup_dp4a)
    (Q8_0, 1536, (100, 37, 5), 3),       # matrices that do not hold whole items: split launches
    (Q4_K, 3584, (3584, 512, 512), 2),   # 7B Q/K/V
    (Q8_0, 8960, (64, 48), 1),           # long rows, two rows per item
])
def test_matvec_multi_equals_separate(ctx, ugb, kind, k, rows, batch):
    """ugb_matvec_multi == one ugb_matvec per matrix, bit for bit (Gpu::batch semantics)."""
    torch = _torch()
    ws = []
    for i, m in enumerate(rows):
        w, rb = make_weights(ctx, ugb, kind, k, m, seed=100 + i)
        ws.append(w)
    x = np.random.default_rng(7).standard_normal((batch, k)).astype(np.float32)
    xq = quantize(ctx, ugb, x)
    total = sum(rows)
    y = torch.full((batch, total), float("nan"), dtype=torch.float32, device="cuda")
    ctx.matvec_multi(kind, ws, rows, rb, xq, y, k, batch)
    parts = []
    for w, m in zip(ws, rows):
        yi = torch.empty((batch, m), dtype=torch.float32, device="cuda")
        ctx.matvec(kind, w, rb, xq, yi, k, m, batch)
        parts.append(yi)
    want = torch.cat(parts, dim=1).cpu().numpy()
    assert np.array_equal(y.cpu().numpy().view(np.uint32), want.view(np.uint32))
    assert ctx.status_read()[0] == ugb.OK


@pytest.mark.parametrize("kind,k,m", SHAPES)
@pytest.mark.parametrize("batch", [1, 3])
def test_matvec_f32_equals_two_calls(ctx, ugb, kind, k, m, batch):
    """ugb_matvec_f32 (quantise inside the matvec when fused) gives exactly quant + matvec."""
    torch = _torch()
    w, rb = make_weights(ctx, ugb, kind, k, m, seed=3 * k + m)
    rng = np.random.default_rng(k + 5 * m + batch)
    x_np = (rng.standard_normal((batch, k)) * rng.uniform(0.1, 10)).astype(np.float32)
    x = torch.from_numpy(x_np).cuda()
    xq = ugb.alloc_q8act(k, batch)
    ctx.quant_q8_1(x, xq, k, batch)
    y2 = torch.full((batch, m), float("nan"), dtype=torch.float32, device="cuda")
    ctx.matvec(kind, w, rb, xq, y2, k, m, batch)
    scratch = ugb.alloc_q8act(k, batch)
    y1 = torch.full((batch, m), float("nan"), dtype=torch.float32, device="cuda")
    ctx.matvec_f32(kind, w, rb, x, scratch, y1, k, m, batch)
    np.testing.assert_array_equal(y1.cpu().numpy().view(np.uint32), y2.cpu().numpy().view(np.uint32))
    code, bits = ctx.status_read()
    assert code == ugb.OK, bits


def test_matvec_f32_fuses_c1(ctx, ugb, orc):
    """At the C1 shape (batch 1) the quantisation runs inside the matvec: the scratch buffer is
    never written, and the rows match the oracle on the scratch-free path."""
    torch = _torch()
    k, m = 1536, 8960
    w, rb = make_weights(ctx, ugb, Q8_0, k, m, seed=11)
    x_np = np.random.default_rng(12).standard_normal((1, k)).astype(np.float32)
    x = torch.from_numpy(x_np).cuda()
    scratch = ugb.alloc_q8act(k, 1)
    scratch.fill_(0x5A)
    y = torch.full((1, m), float("nan"), dtype=torch.float32, device="cuda")
    ctx.matvec_f32(Q8_0, w, rb, x, scratch, y, k, m, 1)
    torch.cuda.synchronize()
    assert bool((scratch == 0x5A).all()), "the fused path must not use the scratch buffer"
    qo, do, so, bad = orc.quant_act(x_np)
    ref = orc.matvec(Q8_0, w.cpu().numpy(), rb, qo, do, so, k, m, 1)
    assert_rows_close(y.cpu().numpy(), ref)
    assert ctx.status_read()[0] == ugb.OK


def test_matvec_f32_nonfinite_sets_status(ctx, ugb):
    torch = _torch()
    k, m = 1536, 64
    w, rb = make_weights(ctx, ugb, Q8_0, k, m, seed=13)
    x = torch.ones((1, k), dtype=torch.float32, device="cuda")
    x[0, 77] = float("inf")
    scratch = ugb.alloc_q8act(k, 1)
    y = torch.empty((1, m), dtype=torch.float32, device="cuda")
    ctx.matvec_f32(Q8_0, w, rb, x, scratch, y, k, m, 1)
    code, bits = ctx.status_read()
    assert code == ugb.ENONFINITE and bits & 1


@pytest.mark.parametrize("k,rows,batch", [
    (3584, (3584, 512, 512), 8),   # 7B Q/K/V: 36 tiles, K split into 4 chunks
    (3584, (18944, 18944), 8),     # 7B gate/up: 296 tiles, whole rows per CTA
    (18944, (3584,), 8),           # 7B down: 28 tiles x 5 chunks of 15 super-blocks
    (3584, (3584,), 5),            # O projection with 5 vectors
    (4096, (1024, 77), 6),         # a matrix boundary on a tile edge, ragged last tile, 16 chunks
    (4096, (1000, 77), 6),         # a matrix boundary inside a tile: the dp4a kernels serve it
    (256, (130,), 7),              # one super-block per row, two tiles
    (24576, (9,), 8),              # one tile of 9 rows, 96 chunks of one super-block
])
def test_matvec_tc_q4k(ctx, ugb, orc, k, rows, batch):
    """Q4_K batches of 5..8 vectors run on the tensor cores (mv_tc.cu): every row against the
    oracle, and the same bits on a second run (the K-split partials add in a fixed order)."""
    torch = _torch()
    ws = []
    for i, m in enumerate(rows):
        w, rb = make_weights(ctx, ugb, Q4_K, k, m, seed=k + 31 * i + m)
        ws.append(w)
    rng = np.random.default_rng(k + batch)
    x = (rng.standard_normal((batch, k)) * rng.uniform(0.1, 10)).astype(np.float32)
    xq = quantize(ctx, ugb, x)
    total = sum(rows)
    outs = []
    for _ in range(2):
        y = torch.full((batch, total), float("nan"), dtype=torch.float32, device="cuda")
        if len(rows) == 1:
            ctx.matvec(Q4_K, ws[0], rb, xq, y, k, rows[0], batch)
        else:
            ctx.matvec_multi(Q4_K, ws, rows, rb, xq, y, k, batch)
        outs.append(y.cpu().numpy())
        code, bits = ctx.status_read()
        assert code == ugb.OK, bits
    assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))
    q, d, s = host_act(ugb, xq, k, batch)
    r0 = 0
    for w, m in zip(ws, rows):
        ref = orc.matvec(Q4_K, w.cpu().numpy(), rb, q, d, s, k, m, batch)
        assert_rows_close(outs[0][:, r0:r0 + m], ref)
        r0 += m
