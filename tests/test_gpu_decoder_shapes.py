"""Layer-synchronised parity of the decoder step at the benchmarked shapes.

The decoder's trace (ugb_decoder_set_trace) records, for every layer, each quantiser's fp32
input and Q8_1 output and each matvec's output.  The CPU restatement (oracle/decode_ref.py,
oracle/ugb_oracle.c; reference: llm.rs:339-388, gpu_graph.rs:139-162) then checks the step one
stage at a time, each stage from the GPU's own inputs to it, so no Q8_1 rounding flip can
carry from one stage into the next:
  * every quantisation is bit-exact: quants, scales and block sums of quant_act(GPU's input);
  * every matvec output (Q/K/V, O, gate/up, down, head) within 1e-3 per row of the oracle's
    integer block dots scaled in fp32, with no statistical allowance;
  * the glue (RMSNorm, bias + RoPE + KV write, attention, SiLU * up) within fp32 summation-order
    tolerances written below, and the residual adds bit-exact;
  * the greedy token is the first maximum of the GPU's logits and of the oracle's.
Shapes: Qwen2.5-1.5B (hidden 1536, FFN 8960, 12/2 heads, vocab 151936, context 512, Q8_0, tied
head) and Qwen2.5-7B (hidden 3584, FFN 18944, 28/4 heads, vocab 152064, context 1024, Q4_K
layers, Q8_0 head), with 2 of their layers, so every row width, CTA split and head grouping of
the full models runs.  A seeded KV history fills the cache, and the steps are taken at positions
that cross every 64-position attention chunk boundary up to the end of the context.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import assert_rows_close
from test_gpu_decoder import CHAIN, TOKEN, build_model

pytestmark = pytest.mark.gpu

Q8_0, Q4_K = 8, 12
F32, F16 = 0, 1
C2 = dict(n_layer=2, n_embd=1536, n_ff=8960, n_head=12, n_head_kv=2, head_dim=128, n_vocab=151936, n_ctx=512,
          rope_theta=1e6, norm_eps=1e-6, kind=Q8_0, head_kind=Q8_0)
C4 = dict(n_layer=2, n_embd=3584, n_ff=18944, n_head=28, n_head_kv=4, head_dim=128, n_vocab=152064, n_ctx=1024,
          rope_theta=1e6, norm_eps=1e-6, kind=Q4_K, head_kind=Q8_0)
C2_POSITIONS = [0, 63, 64, 200, 447, 448, 511]
C4_POSITIONS = [0, 64, 575, 1023]

NORM_REL = 2e-5   # RMSNorm: the sum of squares in another order moves the scale by a few ulp
# attention: chunked log-sum-exp vs one softmax and dot products in another order; score errors of a
# few ulp of |score| (up to ~60 here) become relative errors of the probabilities (worst seen 3e-5)
ATT_REL = 1e-4
SILU_REL = 2e-6   # expf vs numpy's exp: an ulp or two
ROPE_REL = 2e-6   # the rotation with or without a fused multiply-add


def assert_close(gpu, ref, rel, what):
    """|gpu - ref| <= rel * max(|ref|, rms(ref)) elementwise."""
    gpu = np.asarray(gpu, np.float64)
    ref = np.asarray(ref, np.float64)
    assert np.all(np.isfinite(gpu)), f"{what}: non-finite GPU values"
    rms = np.sqrt(np.mean(ref * ref))
    err = np.abs(gpu - ref)
    bound = rel * np.maximum(np.abs(ref), rms)
    i = int(np.argmax(err - bound))
    assert err.flat[i] <= bound.flat[i], (f"{what}: worst index {i} gpu={gpu.flat[i]!r} ref={ref.flat[i]!r} "
                                          f"err={err.flat[i]:.3e} bound={bound.flat[i]:.3e}")


def assert_quant(orc, xq, pre, what):
    """The GPU's Q8_1 of every sequence equals quant_act of its own fp32 input, bit for bit."""
    q, d, s = xq
    q2, d2, s2, _ = orc.quant_act(pre)
    np.testing.assert_array_equal(q, q2, err_msg=f"{what}: quants")
    np.testing.assert_array_equal(d.view(np.uint32), d2.view(np.uint32), err_msg=f"{what}: scales")
    np.testing.assert_array_equal(s, s2, err_msg=f"{what}: block sums")


def matvec(orc, kind, w, xq, m):
    """The oracle's rows and, per row, the sum of its block terms' magnitudes: the GPU adds a
    row's blocks in another order (lane-strided units, K-split partials), which a row that
    cancels to near zero may show at the 2^-24 * terms level."""
    q, d, s = xq
    b, k = q.shape
    rb = orc.row_bytes(kind, k)
    return orc.matvec(kind, w, rb, q, d, s, k, m, b, mt=True), orc.matvec_terms(kind, w, rb, q, d, s, k, m, b)


def rows_close(gpu, want_terms):
    want, terms = want_terms
    assert_rows_close(gpu, want, terms=terms)


def seed_history(dec, cfg, rng):
    """Random rotated keys and values (N(0, 1), as the step's own rows roughly are after RoPE)
    at every position of every layer and sequence."""
    shape = (cfg["n_head_kv"], cfg["n_ctx"], cfg["head_dim"])
    for seq in range(cfg.get("batch", 1)):
        for layer in range(cfg["n_layer"]):
            dec.write_kv(layer, 0, rng.standard_normal(shape).astype(np.float32),
                         rng.standard_normal(shape).astype(np.float32), seq=seq)


def check_step(orc, ref, dec, host, cfg, toks, pos):
    """One traced step at `pos` with tokens `toks`, checked stage by stage."""
    B, hd, kind = len(toks), cfg["head_dim"], cfg["kind"]
    nh, nkv, E, F = cfg["n_head"], cfg["n_head_kv"], cfg["n_embd"], cfg["n_ff"]
    Q, KV = nh * hd, nkv * hd
    nxt = dec.tokens(list(toks), pos) if B > 1 else [dec.token(int(toks[0]), pos)]
    for li in range(cfg["n_layer"]):
        L = host["layers"][li]
        tr = {f: dec.trace(li, f) for f in ("X", "ATTN_NORM", "ATTN_XQ", "QKV", "ATT", "ATT_XQ", "O", "FFN_NORM",
                                          "FFN_XQ", "GATE_UP", "H", "H_XQ", "DOWN")}
        x = tr["X"]
        if li == 0:
            np.testing.assert_array_equal(x, np.stack([ref.embed(int(t)) for t in toks]))
        for b in range(B):
            assert_close(tr["ATTN_NORM"][b], ref.norm(x[b], L["attn_norm"]), NORM_REL, f"L{li} attn norm")
        assert_quant(orc, tr["ATTN_XQ"], tr["ATTN_NORM"], f"L{li} attn xq")
        parts = [matvec(orc, kind, L["wq"], tr["ATTN_XQ"], Q), matvec(orc, kind, L["wk"], tr["ATTN_XQ"], KV),
                 matvec(orc, kind, L["wv"], tr["ATTN_XQ"], KV)]
        rows_close(tr["QKV"], tuple(np.concatenate([p[i] for p in parts], axis=1) for i in range(2)))
        for b in range(B):
            qkv = tr["QKV"][b]
            q = ref.rotate((qkv[:Q] + L["bq"]).reshape(nh, hd), pos)
            k = ref.rotate((qkv[Q:Q + KV] + L["bk"]).reshape(nkv, hd), pos)
            v = (qkv[Q + KV:] + L["bv"]).reshape(nkv, hd)
            keys, vals = dec.read_kv(li, 0, pos + 1, seq=b)
            rel = 1e-3 if cfg.get("kv_type", F32) == F16 else ROPE_REL  # an fp16 rounding may flip with an ulp
            assert_close(keys[:, pos], ref.kv_round(k), rel, f"L{li} cached key")
            assert_close(vals[:, pos], ref.kv_round(v), 0.0, f"L{li} cached value")  # the same fp32 add and rounding
            assert_close(tr["ATT"][b], ref.attend(q, keys, vals).reshape(-1), ATT_REL, f"L{li} attention")
        assert_quant(orc, tr["ATT_XQ"], tr["ATT"], f"L{li} att xq")
        rows_close(tr["O"], matvec(orc, kind, L["wo"], tr["ATT_XQ"], E))
        mid = (x + tr["O"]).astype(np.float32)
        for b in range(B):
            assert_close(tr["FFN_NORM"][b], ref.norm(mid[b], L["ffn_norm"]), NORM_REL, f"L{li} ffn norm")
        assert_quant(orc, tr["FFN_XQ"], tr["FFN_NORM"], f"L{li} ffn xq")
        parts = [matvec(orc, kind, L["w_gate"], tr["FFN_XQ"], F), matvec(orc, kind, L["w_up"], tr["FFN_XQ"], F)]
        rows_close(tr["GATE_UP"], tuple(np.concatenate([p[i] for p in parts], axis=1) for i in range(2)))
        g, u = tr["GATE_UP"][:, :F], tr["GATE_UP"][:, F:]
        with np.errstate(over="ignore"):
            h = (g / (np.float32(1.0) + np.exp(-g)) * u).astype(np.float32)
        assert_close(tr["H"], h, SILU_REL, f"L{li} silu")
        assert_quant(orc, tr["H_XQ"], tr["H"], f"L{li} h xq")
        rows_close(tr["DOWN"], matvec(orc, kind, L["w_down"], tr["H_XQ"], E))
        x_next = dec.trace(li + 1, "X")
        np.testing.assert_array_equal(x_next, (mid + tr["DOWN"]).astype(np.float32), err_msg=f"L{li} residual")
    li = cfg["n_layer"]
    x, xn, xq = dec.trace(li, "X"), dec.trace(li, "ATTN_NORM"), dec.trace(li, "ATTN_XQ")
    for b in range(B):
        assert_close(xn[b], ref.norm(x[b], host["output_norm"]), NORM_REL, "output norm")
    assert_quant(orc, xq, xn, "head xq")
    logits = dec.logits().reshape(B, -1)
    want, terms = matvec(orc, cfg["head_kind"], host["output"], xq, cfg["n_vocab"])
    assert_rows_close(logits, want, terms=terms)
    for b in range(B):
        assert nxt[b] == int(np.argmax(logits[b])), "greedy token is not the first maximum of the logits"
        top = np.sort(want[b])[-2:]
        if top[1] - top[0] > 2e-3 * abs(top[1]):  # not a near tie within the row tolerance
            assert nxt[b] == int(np.argmax(want[b])), "greedy token differs from the oracle's"


def run_shape(ctx, ugb, orc, cfg, path, positions, seed):
    from oracle.decode_ref import RefDecoder
    dec, _, host = build_model_with(ctx, ugb, cfg, seed, path)
    ref = RefDecoder(cfg, host, mt=True)
    rng = np.random.default_rng(seed)
    seed_history(dec, cfg, rng)
    dec.set_trace(True)
    B = cfg.get("batch", 1)
    for pos in positions:
        toks = rng.integers(0, cfg["n_vocab"], size=B)
        check_step(orc, ref, dec, host, cfg, toks, pos)
    assert ctx.status_read()[1] == 0
    dec.set_trace(False)
    dec.close()


def build_model_with(ctx, ugb, cfg, seed, path):
    dev, host = build_model(ctx, ugb, cfg, seed)
    dec = ugb.Decoder(ctx, **cfg)
    dec.bind(dev["tok_embd"], dev["output_norm"], dev["output"], dev["layers"])
    assert dec.set_path(path) == path
    dec._dev = dev  # keep the weights alive as long as the decoder
    return dec, dev, host


@pytest.mark.parametrize("path", [CHAIN, TOKEN], ids=["chain", "token"])
@pytest.mark.parametrize("kv_type", [F32, F16], ids=["kv32", "kv16"])
def test_c2_shape_layer_synced(ctx, ugb, orc, path, kv_type):
    run_shape(ctx, ugb, orc, dict(C2, kv_type=kv_type), path, C2_POSITIONS, seed=101 + kv_type)


@pytest.mark.parametrize("path,kv_type", [(CHAIN, F16), (TOKEN, F16), (TOKEN, F32)],
                         ids=["chain-kv16", "token-kv16", "token-kv32"])
def test_c4_shape_layer_synced(ctx, ugb, orc, path, kv_type):
    run_shape(ctx, ugb, orc, dict(C4, kv_type=kv_type), path, C4_POSITIONS, seed=201 + kv_type)


def test_c4_shape_batch8_layer_synced(ctx, ugb, orc):
    """Eight sequences stepped together (the batched matvec kernels and batched glue)."""
    run_shape(ctx, ugb, orc, dict(C4, kv_type=F16, batch=8), CHAIN, [5, 640, 1023], seed=301)


def test_trace_is_off_by_default_and_bounded(ctx, ugb):
    """Reading a trace that is off is refused; record n_layer holds only X, ATTN_NORM, ATTN_XQ."""
    cfg = dict(C2, n_layer=1, n_vocab=1000)
    dec = ugb.Decoder(ctx, **cfg)
    dec.synthetic(3)
    with pytest.raises(ugb.UgbError):
        dec.trace(0, "X")
    dec.set_trace(True)
    dec.token(1, 0)
    dec.trace(1, "ATTN_XQ")
    with pytest.raises(ugb.UgbError):
        dec.trace(1, "QKV")
    with pytest.raises(ugb.UgbError):
        dec.trace(2, "X")
    dec.close()
