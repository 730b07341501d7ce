"""ugb_linear_static: the host-buffer linear layer for callers that cannot let a library
allocate device memory (hosts that plan every byte of device memory up front, or loops that
must not meet the synchronisation or late out-of-memory failure of a first-use cudaMalloc).
Its scratch is a fixed array compiled into libugb.

Checked through the C ABI:
* on a fresh context, before any ugb_linear call, it allocates nothing: the device's free
  memory and the caching allocator's usage are unchanged across calls (positive control:
  ugb_linear's first call on another fresh context does allocate its workspace);
* its rows equal ugb_linear's bit for bit (the same quantiser and matvec run on the same data)
  and the oracle's within 1e-3 per row, on two calls in a row (the second call reuses the
  scratch the first left behind);
* sizes beyond the fixed scratch are refused with UGB_ESHAPE, and the context stays usable.

Named so that pytest collects it last: a run that stops at the first failure has run every
other test before this one.  It passes alone in a fresh process and after the other tests."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import assert_rows_close

pytestmark = pytest.mark.gpu

Q8_0, Q3_K, Q4_K = 8, 11, 12
SHAPES = [(Q8_0, 1536, 8960), (Q4_K, 4096, 1536), (Q3_K, 1536, 4096), (Q8_0, 16384, 64), (Q8_0, 1536, 151936)]


def _weights(ctx, ugb, kind, k, m, seed):
    import torch
    rb = ugb.row_bytes(kind, k)
    w = torch.empty(rb * m, dtype=torch.uint8, device="cuda")
    ctx.fill_synthetic(kind, w, k, m, seed)
    torch.cuda.synchronize()
    return w, rb


def _oracle_rows(orc, kind, w, rb, x, k, m):
    q, d, s, _ = orc.quant_act(x.reshape(1, k))
    return orc.matvec(kind, w.cpu().numpy(), rb, q, d, s, k, m, 1, mt=True)[0]


def _free_bytes(torch):
    torch.cuda.synchronize()
    return torch.cuda.mem_get_info()[0], torch.cuda.memory_allocated(), torch.cuda.memory_reserved()


def test_static_allocates_nothing(ugb, orc):
    """A fresh context whose only compute calls are ugb_linear_static."""
    import torch
    ctx = ugb.Context(0)
    try:
        kind, k, m = Q8_0, 1536, 8960
        w, rb = _weights(ctx, ugb, kind, k, m, seed=7)
        rng = np.random.default_rng(11)
        xs = [rng.standard_normal(k).astype(np.float32) for _ in range(3)]
        first = ctx.linear_static(kind, w, rb, xs[0], k, m)  # loads the kernels' code
        before = _free_bytes(torch)
        outs = [ctx.linear_static(kind, w, rb, x, k, m) for x in xs[1:]]
        after = _free_bytes(torch)
        assert after == before, f"device memory changed across ugb_linear_static calls: {before} -> {after}"
        for x, y in zip(xs, [first] + outs):
            assert_rows_close(y, _oracle_rows(orc, kind, w, rb, x, k, m))
    finally:
        ctx.close()
    # Positive control: the same measurement sees ugb_linear grow its workspace (a 16 MiB output
    # staging buffer; allocations of a page or less can come from memory the driver holds already).
    ctx = ugb.Context(0)
    try:
        m = 1 << 22
        w, rb = _weights(ctx, ugb, Q8_0, 32, m, seed=8)
        x = np.ones(32, np.float32)
        before = _free_bytes(torch)
        ctx.linear(Q8_0, w, rb, x, 32, m)
        after = _free_bytes(torch)
        assert after[0] < before[0], "the free-memory probe did not see ugb_linear's workspace"
    finally:
        ctx.close()


@pytest.mark.parametrize("kind,k,m", SHAPES)
def test_static_equals_linear_twice(ctx, ugb, orc, kind, k, m):
    w, rb = _weights(ctx, ugb, kind, k, m, seed=k + m)
    rng = np.random.default_rng(m)
    for call in range(2):
        x = rng.standard_normal(k).astype(np.float32)
        got = ctx.linear_static(kind, w, rb, x, k, m)
        want = ctx.linear(kind, w, rb, x, k, m)
        np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32),
                                      err_msg=f"call {call}: static and workspace forms differ")
        assert_rows_close(got, _oracle_rows(orc, kind, w, rb, x, k, m))
    assert ctx.status_read()[1] == 0


def test_static_rejects_sizes_beyond_scratch(ctx, ugb):
    k_big = ugb.LINEAR_STATIC_MAX_K + 32
    w, rb = _weights(ctx, ugb, Q8_0, k_big, 4, seed=1)
    with pytest.raises(ugb.UgbError) as e:
        ctx.linear_static(Q8_0, w, rb, np.ones(k_big, np.float32), k_big, 4)
    assert e.value.code == ugb.ESHAPE
    m_big = ugb.LINEAR_STATIC_MAX_M + 1
    w, rb = _weights(ctx, ugb, Q8_0, 32, m_big, seed=2)
    with pytest.raises(ugb.UgbError) as e:
        ctx.linear_static(Q8_0, w, rb, np.ones(32, np.float32), 32, m_big)
    assert e.value.code == ugb.ESHAPE
    # the context stays usable
    w, rb = _weights(ctx, ugb, Q8_0, 64, 8, seed=3)
    x = np.arange(64, dtype=np.float32) / 64
    np.testing.assert_array_equal(ctx.linear_static(Q8_0, w, rb, x, 64, 8).view(np.uint32),
                                  ctx.linear(Q8_0, w, rb, x, 64, 8).view(np.uint32))


def test_static_selects_its_device(ugb):
    """A context on device 1 called while device 0 is current runs on device 1 (two GPUs)."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    c1 = ugb.Context(1)
    try:
        with torch.cuda.device(1):
            rb = ugb.row_bytes(Q8_0, 1536)
            w = torch.empty(rb * 512, dtype=torch.uint8, device="cuda:1")
            c1.fill_synthetic(Q8_0, w, 1536, 512, 5, stream=torch.cuda.current_stream(1))
            torch.cuda.synchronize(1)
        x = np.linspace(-1, 1, 1536, dtype=np.float32)
        torch.cuda.set_device(0)
        s1 = torch.cuda.current_stream(1)
        got = c1.linear_static(Q8_0, w, rb, x, 1536, 512, stream=s1)
        torch.cuda.set_device(0)
        want = c1.linear(Q8_0, w, rb, x, 1536, 512, stream=s1)
        np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))
        assert torch.cuda.current_device() == 1  # the entry point made ctx's device current
    finally:
        torch.cuda.set_device(0)
        c1.close()
