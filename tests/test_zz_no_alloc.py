"""ugb_linear_static (fixed device scratch, no allocation) against ugb_linear (workspace grown
on demand): the same inputs give the same rows within the per-row tolerance, on two calls in
a row (the second reuses the scratch the first left behind), and out-of-range sizes are
refused.  Named to run last, after the other GPU tests have used the device."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import assert_rows_close

pytestmark = pytest.mark.gpu

Q8_0, Q3_K, Q4_K = 8, 11, 12


def _weights(ctx, ugb, kind, k, m, seed):
    import torch
    rb = ugb.row_bytes(kind, k)
    w = torch.empty(rb * m, dtype=torch.uint8, device="cuda")
    ctx.fill_synthetic(kind, w, k, m, seed)
    return w, rb


@pytest.mark.parametrize("kind,k,m", [(Q8_0, 1536, 8960), (Q4_K, 4096, 1536), (Q3_K, 1536, 4096),
                                      (Q8_0, 16384, 64), (Q8_0, 1536, 151936)])
def test_static_equals_linear_twice(ctx, ugb, kind, k, m):
    w, rb = _weights(ctx, ugb, kind, k, m, seed=k + m)
    rng = np.random.default_rng(m)
    for call in range(2):
        x = rng.standard_normal(k).astype(np.float32)
        want = ctx.linear(kind, w, rb, x, k, m)
        got = ctx.linear_static(kind, w, rb, x, k, m)
        assert_rows_close(got, want)
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
    assert_rows_close(ctx.linear_static(Q8_0, w, rb, x, 64, 8), ctx.linear(Q8_0, w, rb, x, 64, 8))
