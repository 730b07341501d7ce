"""Whole-prompt prefill (ugb_decoder_prefill: gpu_prefill.rs:122-150, gpu_prefill.cu:10-101)
against the CPU restatement, layer by layer, through the prefill trace.

For every layer and every prompt token, from the GPU's own input to each stage: the RMSNorm,
the block-32 quantisation (the oracle re-quantises the GPU's fp32 input; the prefill quantiser is
bit-exact to it, test_gpu_prefill.py) followed by each INT8 GEMM -- Q/K/V, O, gate/up, down --
within 1e-3 per row, bias + RoPE into the KV cache, causal attention over the cache, SiLU * up,
and the residual adds bit-exact.  Then the last token's output norm, its Q8_1 (bit-exact), the
head within 1e-3 per row and the greedy choice; and the decode step that follows continues at
the next position.  Shapes: the benchmarked 1.5B widths with 2 layers and a 512-token prompt,
a prompt that ends inside a 128-token tile, a prefill that continues a cached history (pos0 > 0),
and the fp16 cache."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import assert_rows_close
from test_gpu_decoder import CHAIN, build_model
from test_gpu_decoder_shapes import ATT_REL, C2, F16, F32, NORM_REL, ROPE_REL, SILU_REL, assert_close, assert_quant

pytestmark = pytest.mark.gpu

Q8_0 = 8


def quant_matvec(orc, kind, w, x, m):
    """The oracle's matvec of its own quantisation of x [n, k], and the sums of the magnitudes of
    each row's block terms (the prefill's GEMMs may add a row's blocks in another order: split
    over K)."""
    q, d, s, _ = orc.quant_act(x)
    n, k = x.shape
    rb = orc.row_bytes(kind, k)
    return orc.matvec(kind, w, rb, q, d, s, k, m, n, mt=True), orc.matvec_terms(kind, w, rb, q, d, s, k, m, n)


def rows_close(gpu, want_terms):
    want, terms = want_terms
    assert_rows_close(gpu, want, terms=terms)


def check_prefill(orc, ref, dec, host, cfg, toks, pos0):
    n = len(toks)
    hd, kind = cfg["head_dim"], cfg["kind"]
    nh, nkv, E, F = cfg["n_head"], cfg["n_head_kv"], cfg["n_embd"], cfg["n_ff"]
    Q, KV = nh * hd, nkv * hd
    nxt = dec.prefill(list(toks), pos0)
    for li in range(cfg["n_layer"]):
        L = host["layers"][li]
        tr = {f: dec.prefill_trace(li, f, n) for f in ("X", "ATTN_NORM", "QKV", "ATT", "O", "FFN_NORM", "GATE_UP",
                                                      "H", "DOWN")}
        x = tr["X"]
        if li == 0:
            np.testing.assert_array_equal(x, np.stack([ref.embed(int(t)) for t in toks]))
        for t in range(n):
            assert_close(tr["ATTN_NORM"][t], ref.norm(x[t], L["attn_norm"]), NORM_REL, f"L{li} t{t} attn norm")
        parts = [quant_matvec(orc, kind, L[w], tr["ATTN_NORM"], rows) for w, rows in (("wq", Q), ("wk", KV), ("wv", KV))]
        rows_close(tr["QKV"], (np.concatenate([p[0] for p in parts], axis=1), np.concatenate([p[1] for p in parts], axis=1)))
        keys, vals = dec.read_kv(li, 0, pos0 + n)
        kv_rel = 1e-3 if cfg.get("kv_type", F32) == F16 else ROPE_REL
        for t in range(n):
            pos = pos0 + t
            qkv = tr["QKV"][t]
            q = ref.rotate((qkv[:Q] + L["bq"]).reshape(nh, hd), pos)
            k = ref.rotate((qkv[Q:Q + KV] + L["bk"]).reshape(nkv, hd), pos)
            v = (qkv[Q + KV:] + L["bv"]).reshape(nkv, hd)
            assert_close(keys[:, pos], ref.kv_round(k), kv_rel, f"L{li} t{t} cached key")
            assert_close(vals[:, pos], ref.kv_round(v), 0.0, f"L{li} t{t} cached value")
            assert_close(tr["ATT"][t], ref.attend(q, keys[:, :pos + 1], vals[:, :pos + 1]).reshape(-1), ATT_REL,
                         f"L{li} t{t} attention")
        rows_close(tr["O"], quant_matvec(orc, kind, L["wo"], tr["ATT"], E))
        mid = (x + tr["O"]).astype(np.float32)
        for t in range(n):
            assert_close(tr["FFN_NORM"][t], ref.norm(mid[t], L["ffn_norm"]), NORM_REL, f"L{li} t{t} ffn norm")
        g_, u_ = quant_matvec(orc, kind, L["w_gate"], tr["FFN_NORM"], F), quant_matvec(orc, kind, L["w_up"], tr["FFN_NORM"], F)
        rows_close(tr["GATE_UP"], (np.concatenate([g_[0], u_[0]], axis=1), np.concatenate([g_[1], u_[1]], axis=1)))
        g, u = tr["GATE_UP"][:, :F], tr["GATE_UP"][:, F:]
        with np.errstate(over="ignore"):
            h = (g / (np.float32(1.0) + np.exp(-g)) * u).astype(np.float32)
        assert_close(tr["H"], h, SILU_REL, f"L{li} silu")
        rows_close(tr["DOWN"], quant_matvec(orc, kind, L["w_down"], tr["H"], E))
        x_next = (mid + tr["DOWN"]).astype(np.float32)
        if li + 1 < cfg["n_layer"]:
            np.testing.assert_array_equal(dec.prefill_trace(li + 1, "X", n), x_next, err_msg=f"L{li} residual")
    li = cfg["n_layer"]
    x_last = dec.prefill_trace(li, "X", n)
    np.testing.assert_array_equal(x_last[0], x_next[-1], err_msg="last token's residual")
    xn = dec.prefill_trace(li, "ATTN_NORM", n)
    assert_close(xn[0], ref.norm(x_last[0], host["output_norm"]), NORM_REL, "output norm")
    xq = dec.prefill_trace(li, "ATTN_XQ", n)
    assert_quant(orc, xq, xn, "head xq")
    logits = dec.logits().reshape(1, -1)
    q8, d8, s8 = xq
    want = orc.matvec(cfg["head_kind"], host["output"], orc.row_bytes(cfg["head_kind"], E), q8, d8, s8, E,
                      cfg["n_vocab"], 1, mt=True)
    assert_rows_close(logits, want)
    assert nxt == int(np.argmax(logits[0]))
    return nxt


def make(ctx, ugb, cfg, seed, max_tokens):
    dev, host = build_model(ctx, ugb, cfg, seed)
    dec = ugb.Decoder(ctx, **cfg)
    dec.bind(dev["tok_embd"], dev["output_norm"], dev["output"], dev["layers"])
    dec._dev = dev
    dec.prefill_prepare(max_tokens)
    dec.set_trace(True)
    return dec, host


@pytest.mark.parametrize("n,kv_type", [(512, F32), (300, F16)], ids=["512-kv32", "300-kv16"])
def test_prefill_layer_synced(ctx, ugb, orc, n, kv_type):
    from oracle.decode_ref import RefDecoder
    cfg = dict(C2, kv_type=kv_type)
    dec, host = make(ctx, ugb, cfg, seed=401 + kv_type, max_tokens=512)
    ref = RefDecoder(cfg, host, mt=True)
    toks = np.random.default_rng(7).integers(0, cfg["n_vocab"], size=n)
    nxt = check_prefill(orc, ref, dec, host, cfg, toks, 0)
    assert ctx.status_read()[1] == 0
    # the decode step that follows continues at position n with the prefill's greedy token
    if n < cfg["n_ctx"]:
        dec.set_path(CHAIN)
        dec.step()
        tok, pos, _ = dec.get_state()
        assert (tok, pos) == (nxt, n)
    dec.close()


def test_prefill_continues_a_history(ctx, ugb, orc):
    """A second prefill from pos0 = 200 attends over the first one's cached positions."""
    from oracle.decode_ref import RefDecoder
    cfg = dict(C2, n_ctx=512)
    dec, host = make(ctx, ugb, cfg, seed=411, max_tokens=256)
    ref = RefDecoder(cfg, host, mt=True)
    rng = np.random.default_rng(8)
    dec.prefill(list(rng.integers(0, cfg["n_vocab"], size=200)), 0)
    check_prefill(orc, ref, dec, host, cfg, rng.integers(0, cfg["n_vocab"], size=77), 200)
    dec.close()


def test_prefill_matches_decode_steps(ctx, ugb):
    """Prefilling a prompt leaves the same KV cache as decoding it one token at a time (up to
    fp32 summation order: the GEMM and the matvec sum a row's blocks in different orders), and
    both pick the same next token."""
    cfg = dict(C2, n_layer=2, n_vocab=4096)
    dev, host = build_model(ctx, ugb, cfg, 421)
    pre = ugb.Decoder(ctx, **cfg)
    pre.bind(dev["tok_embd"], dev["output_norm"], dev["output"], dev["layers"])
    pre.prefill_prepare(64)
    step = ugb.Decoder(ctx, **cfg)
    step.bind(dev["tok_embd"], dev["output_norm"], dev["output"], dev["layers"])
    toks = list(np.random.default_rng(9).integers(0, cfg["n_vocab"], size=40))
    nxt = pre.prefill(toks, 0)
    for pos, t in enumerate(toks):
        last = step.token(int(t), pos)
    for layer in range(cfg["n_layer"]):
        k1, v1 = pre.read_kv(layer, 0, len(toks))
        k2, v2 = step.read_kv(layer, 0, len(toks))
        for a, b in ((k1, k2), (v1, v2)):
            err = np.abs(a - b).max() / np.abs(b).max()
            assert err <= 2e-2, err  # a Q8_1 flip in a deeper layer moves values by ~1e-2 at most
    assert nxt == last or np.sort(step.logits())[-2] > np.max(step.logits()) * (1 - 1e-2)
    pre.close()
    step.close()


def test_prefill_bad_arguments(ctx, ugb):
    cfg = dict(C2, n_layer=1, n_vocab=1000)
    dec = ugb.Decoder(ctx, **cfg)
    dec.synthetic(5)
    with pytest.raises(ugb.UgbError):  # not prepared
        dec.prefill([1, 2, 3], 0)
    dec.prefill_prepare(16)
    with pytest.raises(ugb.UgbError):  # more tokens than prepared
        dec.prefill(list(range(17)), 0)
    with pytest.raises(ugb.UgbError):  # past the context
        dec.prefill([1, 2], cfg["n_ctx"] - 1)
    with pytest.raises(ugb.UgbError):  # a token outside the vocabulary
        dec.prefill([1, 1000], 0)
    dec.close()
    moe = ugb.Decoder(ctx, **dict(cfg, n_ff=0, n_expert=4, top_k=2, n_ff_expert=256, expert_kind=11))
    moe.synthetic(5)
    with pytest.raises(ugb.UgbError):  # MoE layers have no prefill path
        moe.prefill_prepare(16)
    moe.close()
