"""The oracle's whole-prompt prefill (RefDecoder.prefill, the reference's prefill graph
gpu_prefill.rs:122-150) equals its token-by-token forward (RefDecoder.step, llm.rs:339-388)
exactly: the same per-row block dots, norms, rotations and attention, batched differently.
CPU only."""
from __future__ import annotations

import numpy as np
import pytest

Q8_0 = 8
CFG = dict(n_layer=2, n_embd=256, n_ff=512, n_head=4, n_head_kv=2, head_dim=128, n_vocab=300, n_ctx=64,
           rope_theta=1e6, norm_eps=1e-6, kind=Q8_0, head_kind=Q8_0)


def host_model(rng, c):
    def mat(k, m):
        nb = k // 32
        b = np.empty((m, nb, 34), dtype=np.uint8)
        b[:, :, 2:] = rng.integers(-127, 128, size=(m, nb, 32), dtype=np.int8).view(np.uint8)
        b[:, :, :2] = (0.002 * np.abs(rng.standard_normal((m, nb)))).astype(np.float16).view(np.uint8).reshape(m, nb, 2)
        return b.reshape(-1)

    def vec(n, center, amp):
        return (center + amp * rng.uniform(-1, 1, n)).astype(np.float32)

    q, kv, e, f = c["n_head"] * 128, c["n_head_kv"] * 128, c["n_embd"], c["n_ff"]
    w = {"tok_embd": mat(e, c["n_vocab"]), "output_norm": vec(e, 1.0, 0.1)}
    w["output"] = w["tok_embd"]
    w["layers"] = [dict(attn_norm=vec(e, 1, .1), ffn_norm=vec(e, 1, .1), bq=vec(q, 0, .02), bk=vec(kv, 0, .02),
                        bv=vec(kv, 0, .02), wq=mat(e, q), wk=mat(e, kv), wv=mat(e, kv), wo=mat(q, e),
                        w_gate=mat(e, f), w_up=mat(e, f), w_down=mat(f, e)) for _ in range(c["n_layer"])]
    return w


@pytest.mark.parametrize("kv_type", [0, 1])
def test_oracle_prefill_equals_steps(kv_type):
    from oracle.decode_ref import RefDecoder
    c = dict(CFG, kv_type=kv_type)
    w = host_model(np.random.default_rng(1), c)
    toks = np.random.default_rng(2).integers(0, c["n_vocab"], size=21)
    a, b = RefDecoder(c, w), RefDecoder(c, w)
    la, na = a.prefill(toks[:13], 0)
    la2, na2 = a.prefill(toks[13:], 13)  # a second prompt continuing the first
    for pos, t in enumerate(toks):
        lb, nb = b.step(int(t), pos)
        if pos == 12:
            np.testing.assert_array_equal(la, lb)
            assert na == nb
    np.testing.assert_array_equal(la2, lb)
    assert na2 == nb
    np.testing.assert_array_equal(a.kcache, b.kcache)
    np.testing.assert_array_equal(a.vcache, b.vcache)
