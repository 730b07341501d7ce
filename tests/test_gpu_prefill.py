"""GPU parity of the Q8 prefill path (repack, token-batched quant, tcgen05 INT8 GEMM) against
the CPU oracle, through the C ABI.

* The repack is lossless: un-permuting the packed tiles gives back every quant and the exact
  f32 of every fp16 scale (oracle orc_prefill_repack_q8_0).
* The packed activation holds the quant_act quants and scales bit for bit.
* Every int32 block dot the tensor cores produce equals the integer dot computed on the host.
* y equals the oracle's fmaf((float)dot, dw*dx, acc) accumulation in block order bit for bit
  (same operations in the same order), and within 1e-3 per row in any case.
Shapes: the config-3 matrices (K 1536 / 8960; N 2048 / 1536 / 17920) at reduced token counts,
both CTA widths (128-row tiles, and 64-row halves when 128-row tiling leaves SMs idle), and ragged edges (tokens and rows not multiples of the 128-row tile, a single K-block, K
whose block count is not a multiple of the 4-block stage).
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import assert_rows_close

pytestmark = pytest.mark.gpu

Q8_0 = 8
TILE = 128


def _canon_index():
    r = np.arange(TILE)[:, None]
    j = np.arange(32)[None, :]
    return (r // 8) * 256 + (j // 16) * 128 + (r % 8) * 16 + (j % 16)


CANON = _canon_index()


def unpack(buf: np.ndarray, rows: int, k: int):
    """Packed prefill operand -> (quants int8 [tiles*128][k], scales f32 [k/32][tiles*128])."""
    tiles, nb = -(-rows // TILE), k // 32
    qbytes = tiles * nb * TILE * 32
    qt = buf[:qbytes].view(np.int8).reshape(tiles, nb, TILE * 32)
    q = qt[:, :, CANON]                      # [tiles][nb][128][32]
    q = q.transpose(0, 2, 1, 3).reshape(tiles * TILE, k)
    s = buf[qbytes:].view(np.float32).reshape(tiles, nb, TILE).transpose(1, 0, 2).reshape(nb, tiles * TILE)
    return q, s


def synth_q8_0(ctx, ugb, k, n, seed):
    import torch
    rb = ugb.row_bytes(Q8_0, k)
    w = torch.empty(rb * n, dtype=torch.uint8, device="cuda")
    ctx.fill_synthetic(Q8_0, w, k, n, seed)
    return w


def run_prefill(ctx, ugb, w, x_np, n, k, dots=False):
    import torch
    m = x_np.shape[0]
    wp = ugb.alloc_prefill(n, k)
    xp = ugb.alloc_prefill(m, k)
    ctx.prefill_repack_q8_0(w, n, k, wp)
    x = torch.from_numpy(np.ascontiguousarray(x_np, dtype=np.float32)).cuda()
    ctx.prefill_quant(x, m, k, xp)
    y = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
    d = None
    if dots:
        d = torch.zeros((k // 32, m, n), dtype=torch.int32, device="cuda")
        ctx.prefill_block_dots(wp, xp, d, y, m, n, k)
    else:
        ctx.prefill_gemm(wp, xp, y, m, n, k)
    torch.cuda.synchronize()
    return wp, xp, y.cpu().numpy(), (d.cpu().numpy() if dots else None)


@pytest.mark.parametrize("n,k", [(300, 256), (128, 32), (2048, 1536)])
def test_repack_lossless(ctx, ugb, orc, n, k):
    w = synth_q8_0(ctx, ugb, k, n, seed=n + k)
    wp = ugb.alloc_prefill(n, k)
    ctx.prefill_repack_q8_0(w, n, k, wp)
    q, s = unpack(wp.cpu().numpy(), n, k)
    n_pad = q.shape[0]
    qa, sa = orc.prefill_repack_q8_0(w.cpu().numpy(), n, k, n_pad)
    np.testing.assert_array_equal(q, qa)
    np.testing.assert_array_equal(s.view(np.uint32), sa.view(np.uint32))


@pytest.mark.parametrize("m,k", [(200, 256), (1, 32), (512, 1536)])
def test_prefill_quant_bit_exact(ctx, ugb, orc, m, k):
    import torch
    rng = np.random.default_rng(m + k)
    x = (rng.standard_normal((m, k)) * rng.uniform(0.1, 10, (m, 1))).astype(np.float32)
    xp = ugb.alloc_prefill(m, k)
    ctx.prefill_quant(torch.from_numpy(x).cuda(), m, k, xp)
    q, s = unpack(xp.cpu().numpy(), m, k)
    qo, do, _, bad = orc.quant_act(x)
    assert bad == 0
    np.testing.assert_array_equal(q[:m], qo)
    assert not q[m:].any()
    np.testing.assert_array_equal(s[:, :m].T.view(np.uint32), do.view(np.uint32))
    assert not s[:, m:].any()


@pytest.mark.parametrize("m,n,k", [(200, 300, 256), (128, 128, 32), (37, 256, 416), (256, 18944, 64)])
def test_block_dots_bit_exact(ctx, ugb, orc, m, n, k):
    rng = np.random.default_rng(7 * m + n)
    x = rng.standard_normal((m, k)).astype(np.float32)
    w = synth_q8_0(ctx, ugb, k, n, seed=m * n)
    _, _, y, dots = run_prefill(ctx, ugb, w, x, n, k, dots=True)
    nb = k // 32
    qx, _, _, _ = orc.quant_act(x)
    wq = w.cpu().numpy().reshape(n, nb, 34)[:, :, 2:].view(np.int8).astype(np.int32)  # [n][nb][32]
    want = np.einsum("tbj,nbj->btn", qx.reshape(m, nb, 32).astype(np.int32), wq)
    np.testing.assert_array_equal(dots, want)
    yo = orc.prefill_gemm_q8_0(w.cpu().numpy(), n, k, x)
    np.testing.assert_array_equal(y.view(np.uint32), yo.view(np.uint32))


@pytest.mark.parametrize("m,n,k", [(512, 2048, 1536), (96, 1536, 8960), (300, 17920, 1536), (129, 256, 1536)])
def test_prefill_gemm_matches_oracle(ctx, ugb, orc, m, n, k):
    rng = np.random.default_rng(m + n + k)
    x = rng.standard_normal((m, k)).astype(np.float32)
    w = synth_q8_0(ctx, ugb, k, n, seed=n ^ k)
    _, _, y, _ = run_prefill(ctx, ugb, w, x, n, k)
    yo = orc.prefill_gemm_q8_0(w.cpu().numpy(), n, k, x)
    for t in range(m):
        assert_rows_close(y[t], yo[t])
    assert np.array_equal(y.view(np.uint32), yo.view(np.uint32))
    assert ctx.status_read()[1] == 0


def test_prefill_rejects_bad_shapes(ctx, ugb):
    import torch
    w = synth_q8_0(ctx, ugb, 64, 8, seed=1)
    wp = ugb.alloc_prefill(8, 64)
    with pytest.raises(ugb.UgbError):
        ctx.prefill_repack_q8_0(w, 8, 48, wp)
    xp = ugb.alloc_prefill(4, 64)
    y = torch.empty((4, 8), dtype=torch.float32, device="cuda")
    with pytest.raises(ugb.UgbError):
        ctx.prefill_gemm(wp, xp, y, 4, 8, 64, ldy=4)
    with pytest.raises(ugb.UgbError):
        ctx.prefill_gemm(wp, xp, y, 0, 8, 64)
