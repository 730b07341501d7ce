"""CUDA-graph capture (ugb_graph_*) and programmatic dependent launch (ugb_set_pdl) give the
same bits as eager launches."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

Q8_0, Q4_K = 8, 12


@pytest.mark.parametrize("kind,k,m", [(Q8_0, 1536, 8960), (Q4_K, 3584, 512), (Q8_0, 8960, 1536)])
def test_graph_pdl_matches_eager(ctx, ugb, kind, k, m):
    import torch
    rb = ugb.row_bytes(kind, k)
    ws = [torch.empty(rb * m, dtype=torch.uint8, device="cuda") for _ in range(3)]
    for i, w in enumerate(ws):
        ctx.fill_synthetic(kind, w, k, m, seed=50 + i)
    xs = torch.randn((3, k), generator=torch.Generator().manual_seed(1)).cuda()
    xq = ugb.alloc_q8act(k, 1)
    eager = torch.empty((3, m), dtype=torch.float32, device="cuda")
    for i in range(3):
        ctx.quant_q8_1(xs[i], xq, k, 1)
        ctx.matvec(kind, ws[i], rb, xq, eager[i], k, m, 1)
    torch.cuda.synchronize()

    graphed = torch.full((3, m), float("nan"), dtype=torch.float32, device="cuda")
    ctx.set_pdl(True)
    try:
        def body():
            for i in range(3):
                ctx.quant_q8_1(xs[i], xq, k, 1)
                ctx.matvec(kind, ws[i], rb, xq, graphed[i], k, m, 1)
        g = ctx.capture(body, torch.cuda.Stream())
    finally:
        ctx.set_pdl(False)
    for _ in range(2):
        g.launch()
    torch.cuda.synchronize()
    assert np.array_equal(eager.cpu().numpy().view(np.uint32), graphed.cpu().numpy().view(np.uint32))
    code, bits = ctx.status_read()
    assert code == ugb.OK, bits
    g.close()
