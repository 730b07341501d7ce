"""GGUF model files for the tests, written with the third-party `gguf` package (llama.cpp's
Python writer, 0.19.0 in this image): a Qwen2-style dense model or a Qwen3-MoE-style model from
host weight dicts (raw GGUF block bytes for matrices, fp32 norms and biases), with the
architecture metadata a loader reads.  Test infrastructure only."""
from __future__ import annotations

import numpy as np

KIND_BLOCK = {8: (32, 34), 11: (256, 110), 12: (256, 144), 0: (1, 4)}


def _rows(raw: np.ndarray, kind: int, k: int) -> np.ndarray:
    """Raw block bytes of a matrix with rows of k elements as a [rows, row_bytes] uint8 array."""
    blk, nb = KIND_BLOCK[kind]
    return np.ascontiguousarray(raw, dtype=np.uint8).reshape(-1, k // blk * nb)


def write_model(path: str, cfg: dict, host: dict, arch: str | None = None, tied: bool = True,
                split_max_tensors: int = 0, extra_meta: bool = True) -> list[str]:
    """Write host weights (the dict test_gpu_decoder.build_model returns) as GGUF; returns the
    file names written (several when split_max_tensors > 0)."""
    import gguf
    moe = cfg.get("n_expert", 0) > 0
    arch = arch or ("qwen3moe" if moe else "qwen2")
    w = gguf.GGUFWriter(path, arch, split_max_tensors=split_max_tensors)
    w.add_block_count(cfg["n_layer"])
    w.add_embedding_length(cfg["n_embd"])
    w.add_head_count(cfg["n_head"])
    w.add_head_count_kv(cfg["n_head_kv"])
    w.add_key_length(cfg["head_dim"])
    w.add_value_length(cfg["head_dim"])
    w.add_context_length(cfg["n_ctx"])
    w.add_rope_freq_base(float(cfg["rope_theta"]))
    w.add_layer_norm_rms_eps(float(cfg["norm_eps"]))
    if moe:
        w.add_expert_count(cfg["n_expert"])
        w.add_expert_used_count(cfg["top_k"])
        w.add_expert_feed_forward_length(cfg["n_ff_expert"])
    else:
        w.add_feed_forward_length(cfg["n_ff"])
    if extra_meta:
        w.add_array("tokenizer.ggml.tokens", [f"tok{i}" for i in range(16)])
        w.add_key_value("test.numbers", [3, 1, 4, 1, 5], gguf.GGUFValueType.ARRAY, sub_type=gguf.GGUFValueType.UINT32)
        w.add_array("test.signed", [-1, 2])  # int32 elements: not an unsigned value
        w.add_string("general.name", "synthetic ügb model")
    Q8, E = gguf.GGMLQuantizationType.Q8_0, cfg["n_embd"]
    qt = {8: gguf.GGMLQuantizationType.Q8_0, 11: gguf.GGMLQuantizationType.Q3_K, 12: gguf.GGMLQuantizationType.Q4_K}

    def mat(name, raw, kind, k):
        w.add_tensor(name, _rows(raw, kind, k), raw_dtype=qt[kind])

    def f32(name, v):
        w.add_tensor(name, np.ascontiguousarray(v, dtype=np.float32))

    mat("token_embd.weight", host["tok_embd"], 8, E)
    f32("output_norm.weight", host["output_norm"])
    if not tied:
        mat("output.weight", host["output"], cfg["head_kind"], E)
    kind, hd = cfg["kind"], cfg["head_dim"]
    q = cfg["n_head"] * hd
    for li, L in enumerate(host["layers"]):
        b = f"blk.{li}."
        f32(b + "attn_norm.weight", L["attn_norm"])
        f32(b + "ffn_norm.weight", L["ffn_norm"])
        mat(b + "attn_q.weight", L["wq"], kind, E)
        mat(b + "attn_k.weight", L["wk"], kind, E)
        mat(b + "attn_v.weight", L["wv"], kind, E)
        mat(b + "attn_output.weight", L["wo"], kind, q)
        for bias in ("bq", "bk", "bv"):
            if L.get(bias) is not None:
                f32(b + {"bq": "attn_q.bias", "bk": "attn_k.bias", "bv": "attn_v.bias"}[bias], L[bias])
        if moe:
            ek, ne, ff = cfg["expert_kind"], cfg["n_expert"], cfg["n_ff_expert"]
            mat(b + "ffn_gate_inp.weight", L["router"], kind, E)
            for name, raw, k, rows in (("ffn_gate_exps", L["gate_exps"], E, ff), ("ffn_up_exps", L["up_exps"], E, ff),
                                       ("ffn_down_exps", L["down_exps"], ff, E)):
                blk, nb = KIND_BLOCK[ek]
                arr = np.ascontiguousarray(raw, dtype=np.uint8).reshape(ne, rows, k // blk * nb)
                w.add_tensor(b + name + ".weight", arr, raw_dtype=qt[ek])
        else:
            mat(b + "ffn_gate.weight", L["w_gate"], kind, E)
            mat(b + "ffn_up.weight", L["w_up"], kind, E)
            mat(b + "ffn_down.weight", L["w_down"], kind, cfg["n_ff"])
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    if split_max_tensors:
        import glob
        import os
        stem = os.path.splitext(path)[0]
        return sorted(glob.glob(stem + "-*-of-*.gguf"))
    return [path]


def host_model(rng, c: dict) -> dict:
    """Seeded random weights in host memory: Q8_0 / K-quant matrices as raw block bytes (fp16
    scales |N(0,1)| * 0.002 where a format has them at the block start), fp32 norms and biases."""
    def mat(kind, k, m):
        blk, nb = KIND_BLOCK[kind]
        b = rng.integers(0, 256, size=(m, k // blk, nb), dtype=np.uint8)
        if kind == 8:
            b[:, :, :2] = (0.002 * np.abs(rng.standard_normal((m, k // blk)))).astype(np.float16).view(
                np.uint8).reshape(m, k // blk, 2)
        return b.reshape(-1)

    def vec(n, center, amp):
        return (center + amp * rng.uniform(-1, 1, n)).astype(np.float32)

    q, kv, e = c["n_head"] * c["head_dim"], c["n_head_kv"] * c["head_dim"], c["n_embd"]
    kind = c["kind"]
    w = {"tok_embd": mat(8, e, c["n_vocab"]), "output_norm": vec(e, 1.0, 0.1)}
    w["output"] = w["tok_embd"] if c["head_kind"] == 8 else mat(c["head_kind"], e, c["n_vocab"])
    moe = c.get("n_expert", 0) > 0
    w["layers"] = []
    for _ in range(c["n_layer"]):
        L = dict(attn_norm=vec(e, 1, .1), ffn_norm=vec(e, 1, .1), wq=mat(kind, e, q), wk=mat(kind, e, kv),
                 wv=mat(kind, e, kv), wo=mat(kind, q, e))
        if moe:
            ek, ne, ff = c["expert_kind"], c["n_expert"], c["n_ff_expert"]
            L.update(router=mat(kind, e, ne), gate_exps=mat(ek, e, ff * ne), up_exps=mat(ek, e, ff * ne),
                     down_exps=mat(ek, ff, e * ne))
        else:
            L.update(bq=vec(q, 0, .02), bk=vec(kv, 0, .02), bv=vec(kv, 0, .02), w_gate=mat(kind, e, c["n_ff"]),
                     w_up=mat(kind, e, c["n_ff"]), w_down=mat(kind, c["n_ff"], e))
        w["layers"].append(L)
    return w
