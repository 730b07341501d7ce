"""CPU restatement of one decode token step of a Qwen2-style model.

TEST INFRASTRUCTURE ONLY: the checker for the decoder's GPU token step (tests/, the smoke check)
and the timed CPU leg of bench.py.  The product path never imports it.

It follows the reference's CPU forward (driver/src/llm.rs:339-388) with the numerics of the
reference's GPU decode graph (driver/src/gpu_graph.rs:139-162):
  * every linear layer takes a block-32 Q8_1 activation (quant_act, driver/kernels/gpu_dp4a.cu:23-31)
    and multiplies it by the weight's integer block dots (the C oracle's orc_matvec);
  * RMSNorm y = x * (1 / sqrt(sum(x^2)/n + eps)) * w (llm.rs:323-327);
  * Q/K/V biases added before RoPE; RoPE over the pairs (i, i + HD/2) with the table built from
    the f32 angle pos * powf(theta, -(2i)/HD) (gpu_graph.rs:132, llm.rs:328-337);
  * fp32 KV cache, scores q.k / sqrt(HD), exact exp softmax (gpu_attention.cu:1-26); with
    cfg["kv_type"] == 1 the cache holds fp16 instead: keys and values are rounded to nearest
    even as they are written, and attention reads them back (the current position included);
  * SiLU(gate) * up (llm.rs:374), residual adds, final norm, head, first-maximum greedy
    (llm.rs:383-385);
  * an MoE FFN when cfg["n_expert"] > 0 (Forward::ffn, frontier_forward.rs:164-199): router
    linear, softmax top-k with ties to the lower id and renormalised weights (the C oracle's
    orc_moe_route), per selected expert gate / up linears, SiLU(gate) * up, down linear, and
    out = sum of weight * value in rank order with a separate multiply and add.
"""
from __future__ import annotations

import numpy as np

from . import pyoracle as po

Q8_0 = po.Q8_0


def rope_table(n_ctx: int, head_dim: int, theta: float) -> np.ndarray:
    """[n_ctx][head_dim/2][2] (cos, sin) as float32 (gpu_graph.rs:132)."""
    i = np.arange(head_dim // 2)
    e = (-(2 * i).astype(np.float32) / np.float32(head_dim)).astype(np.float32)
    f = np.power(np.float64(np.float32(theta)), e.astype(np.float64)).astype(np.float32)
    ang = (np.arange(n_ctx, dtype=np.float32)[:, None] * f[None, :]).astype(np.float32)
    a64 = ang.astype(np.float64)
    return np.stack([np.cos(a64), np.sin(a64)], axis=-1).astype(np.float32)


class RefDecoder:
    """One sequence of decode steps on the CPU.

    cfg: dict with the fields of ugb_decoder_config.  weights: dict with tok_embd (Q8_0 bytes),
    output_norm (f32), output (head_kind bytes) and layers, a list of dicts with attn_norm,
    ffn_norm, bq, bk, bv (f32, biases may be None) and wq, wk, wv, wo, w_gate, w_up, w_down
    (raw GGUF row bytes of cfg["kind"])."""

    def __init__(self, cfg: dict, weights: dict, mt: bool = False):
        self.c = dict(cfg)
        self.w = weights
        self.mt = mt
        c = self.c
        self.hd = c["head_dim"]
        self.kcache = np.zeros((c["n_layer"], c["n_head_kv"], c["n_ctx"], self.hd), np.float32)
        self.vcache = np.zeros_like(self.kcache)
        self.rope = rope_table(c["n_ctx"], self.hd, c["rope_theta"])
        self.kv16 = c.get("kv_type", 0) == 1

    # ---- pieces ---------------------------------------------------------------------------

    def linear(self, kind: int, w: np.ndarray, x: np.ndarray, m: int) -> np.ndarray:
        k = x.size
        q, d, s, _ = po.quant_act(x.reshape(1, k))
        return self.linear_q8(kind, w, q[0], d[0], s[0], m)

    def linear_q8(self, kind: int, w: np.ndarray, q: np.ndarray, d: np.ndarray, s: np.ndarray, m: int) -> np.ndarray:
        """The matvec of an already quantised Q8_1 activation (q int8 [k], d f32 [k/32], s int32 [k/32])."""
        k = q.size
        return po.matvec(kind, w, po.row_bytes(kind, k), q.reshape(1, k), d.reshape(1, -1), s.reshape(1, -1), k, m,
                         1, mt=self.mt)[0]

    def kv_round(self, v: np.ndarray) -> np.ndarray:
        """The value the cache gives back for v (fp16 round to nearest even in an fp16 cache)."""
        return v.astype(np.float16).astype(np.float32) if self.kv16 else v.astype(np.float32)

    def attend(self, q: np.ndarray, keys: np.ndarray, vals: np.ndarray) -> np.ndarray:
        """q [n_head, HD] (rotated), keys / vals [n_kv, t, HD] -> attention output [n_head, HD]:
        scores q.k / sqrt(HD), exact exp softmax, probabilities times values (gpu_attention.cu:2-26)."""
        nh, nkv = q.shape[0], keys.shape[0]
        group = nh // nkv
        inv_sqrt = np.float32(1.0) / np.sqrt(np.float32(self.hd))
        att = np.empty((nh, self.hd), np.float32)
        for h in range(nh):
            kv = h // group
            sc = (keys[kv] @ q[h]).astype(np.float32) * inv_sqrt
            e = np.exp(sc - sc.max()).astype(np.float32)
            att[h] = (e @ vals[kv]).astype(np.float32) / np.float32(e.sum(dtype=np.float32))
        return att

    def norm(self, x: np.ndarray, w: np.ndarray) -> np.ndarray:
        n = x.size
        ss = np.float32(np.sum(x * x, dtype=np.float32))
        scale = np.float32(1.0) / np.sqrt(ss / np.float32(n) + np.float32(self.c["norm_eps"]))
        return (x * scale * w).astype(np.float32)

    def rotate(self, v: np.ndarray, pos: int) -> np.ndarray:
        """v [heads, HD] -> rotated copy."""
        h2 = self.hd // 2
        cs, sn = self.rope[pos, :, 0], self.rope[pos, :, 1]
        v0, v1 = v[:, :h2], v[:, h2:]
        return np.concatenate([v0 * cs - v1 * sn, v0 * sn + v1 * cs], axis=1).astype(np.float32)

    def embed(self, token: int) -> np.ndarray:
        n = self.c["n_embd"]
        rb = po.row_bytes(Q8_0, n)
        return po.dequantize(Q8_0, self.w["tok_embd"][token * rb:(token + 1) * rb], n)

    def moe_ffn(self, L: dict, xn: np.ndarray, experts: range | None = None) -> np.ndarray:
        """Routed SwiGLU experts of one layer; L holds router and the stacked expert tensors
        gate_exps / up_exps / down_exps (raw bytes, all n_expert experts).  With `experts`,
        only the selected experts in that range contribute (one expert-parallel shard's
        partial sum)."""
        c = self.c
        ek, ne, ff, d = c["expert_kind"], c["n_expert"], c["n_ff_expert"], c["n_embd"]
        scores = self.linear(c["kind"], L["router"], xn, ne)
        ids, weights = po.moe_route(scores, c["top_k"])
        rbi, rbf = po.row_bytes(ek, d), po.row_bytes(ek, ff)
        out = np.zeros(d, np.float32)
        for e, wgt in zip(ids, weights):
            if experts is not None and int(e) not in experts:
                continue
            g = self.linear(ek, L["gate_exps"][e * ff * rbi:(e + 1) * ff * rbi], xn, ff)
            u = self.linear(ek, L["up_exps"][e * ff * rbi:(e + 1) * ff * rbi], xn, ff)
            with np.errstate(over="ignore"):
                h = (g / (np.float32(1.0) + np.exp(-g)) * u).astype(np.float32)
            v = self.linear(ek, L["down_exps"][e * d * rbf:(e + 1) * d * rbf], h, d)
            out = (out + (np.float32(wgt) * v).astype(np.float32)).astype(np.float32)
        return out

    # ---- a whole prompt ------------------------------------------------------------------

    def prefill(self, tokens, pos0: int = 0):
        """The reference's prefill graph (gpu_prefill.rs:122-150, kernels gpu_prefill.cu:60-101):
        every layer over all prompt tokens at once -- per-token RMSNorm and block-32 quantisation,
        the linear layers as one batched matvec per matrix (the same integer block dots), bias + RoPE
        into the cache, causal attention of token t over positions [0, pos0 + t], SiLU * up -- then
        only the last token through the final norm and the head (gpu_prefill.rs:138-148).  Dense
        layers only.  Returns (last token's logits, greedy next token)."""
        c, hd = self.c, self.hd
        kind, nh, nkv = c["kind"], c["n_head"], c["n_head_kv"]
        qrows, kvrows, e = nh * hd, nkv * hd, c["n_embd"]
        n = len(tokens)
        x = np.stack([self.embed(int(t)) for t in tokens])

        def lin(w, xs, m):
            q, d, s, _ = po.quant_act(xs)
            k = xs.shape[1]
            return po.matvec(kind, w, po.row_bytes(kind, k), q, d, s, k, m, xs.shape[0], mt=self.mt)

        for li, L in enumerate(self.w["layers"]):
            xn = np.stack([self.norm(x[t], L["attn_norm"]) for t in range(n)])
            q, k, v = lin(L["wq"], xn, qrows), lin(L["wk"], xn, kvrows), lin(L["wv"], xn, kvrows)
            if L.get("bq") is not None:
                q, k, v = q + L["bq"], k + L["bk"], v + L["bv"]
            att = np.empty((n, qrows), np.float32)
            qr = np.empty((n, nh, hd), np.float32)
            for t in range(n):
                pos = pos0 + t
                qr[t] = self.rotate(q[t].reshape(nh, hd), pos)
                self.kcache[li, :, pos] = self.kv_round(self.rotate(k[t].reshape(nkv, hd), pos))
                self.vcache[li, :, pos] = self.kv_round(v[t].reshape(nkv, hd))
            for t in range(n):
                pos = pos0 + t
                att[t] = self.attend(qr[t], self.kcache[li, :, :pos + 1], self.vcache[li, :, :pos + 1]).reshape(-1)
            x = (x + lin(L["wo"], att, e)).astype(np.float32)
            xn = np.stack([self.norm(x[t], L["ffn_norm"]) for t in range(n)])
            g, u = lin(L["w_gate"], xn, c["n_ff"]), lin(L["w_up"], xn, c["n_ff"])
            with np.errstate(over="ignore"):
                h = (g / (np.float32(1.0) + np.exp(-g)) * u).astype(np.float32)
            x = (x + lin(L["w_down"], h, e)).astype(np.float32)
        xn = self.norm(x[-1], self.w["output_norm"])
        logits = self.linear(c["head_kind"], self.w["output"], xn, c["n_vocab"])
        return logits, int(np.argmax(logits))

    # ---- one token -----------------------------------------------------------------------

    def step(self, token: int, pos: int):
        """Returns (logits f32 [n_vocab], greedy next token)."""
        c, hd = self.c, self.hd
        kind = c["kind"]
        nh, nkv = c["n_head"], c["n_head_kv"]
        qrows, kvrows = nh * hd, nkv * hd
        x = self.embed(token)
        for li, L in enumerate(self.w["layers"]):
            xn = self.norm(x, L["attn_norm"])
            q = self.linear(kind, L["wq"], xn, qrows)
            k = self.linear(kind, L["wk"], xn, kvrows)
            v = self.linear(kind, L["wv"], xn, kvrows)
            if L.get("bq") is not None:
                q = q + L["bq"]
            if L.get("bk") is not None:
                k = k + L["bk"]
            if L.get("bv") is not None:
                v = v + L["bv"]
            q = self.rotate(q.reshape(nh, hd), pos)
            k = self.rotate(k.reshape(nkv, hd), pos)
            self.kcache[li, :, pos] = self.kv_round(k)
            self.vcache[li, :, pos] = self.kv_round(v.reshape(nkv, hd))
            att = self.attend(q, self.kcache[li, :, :pos + 1], self.vcache[li, :, :pos + 1])
            x = (x + self.linear(kind, L["wo"], att.reshape(-1), c["n_embd"])).astype(np.float32)
            xn = self.norm(x, L["ffn_norm"])
            if c.get("n_expert", 0):
                x = (x + self.moe_ffn(L, xn)).astype(np.float32)
                continue
            g = self.linear(kind, L["w_gate"], xn, c["n_ff"])
            u = self.linear(kind, L["w_up"], xn, c["n_ff"])
            with np.errstate(over="ignore"):  # exp(-g) = inf for very negative g gives -0, as expf
                h_act = (g / (np.float32(1.0) + np.exp(-g)) * u).astype(np.float32)
            x = (x + self.linear(kind, L["w_down"], h_act, c["n_embd"])).astype(np.float32)
        xn = self.norm(x, self.w["output_norm"])
        logits = self.linear(c["head_kind"], self.w["output"], xn, c["n_vocab"])
        return logits, int(np.argmax(logits))
