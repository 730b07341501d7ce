"""GGUF directory parsing and decoder binding (ugb_gguf_*), on the CPU.

The reference's parser is Shard::parse / Tensor::rows / Tensor::expert / ModelIndex
(frontier_gguf.rs:84-200).  Its own tests need header fixtures of a real model that are not in
this image, so the parser is pinned two ways:
* files written by the third-party `gguf` 0.19.0 package (llama.cpp's writer and reader): every
  tensor's name, dims, kind, absolute offset and size and every metadata value equal what
  gguf.GGUFReader reads, single files and split sets alike;
* the reference's own synthetic directories and corruptions (frontier_gguf.rs:238-262: overlap,
  alignment, offset and width overflow, partial blocks, truncation, version, limits) give the
  same error as its test expects.
Then ugb_gguf_decoder_config reads the shape back from the metadata and
ugb_gguf_model_weights points every tensor at base + (file offset - base offset)."""
from __future__ import annotations

import struct

import numpy as np
import pytest

import gguf_files as gf

Q8_0, Q3_K, Q4_K = 8, 11, 12
DENSE = dict(n_layer=2, n_embd=256, n_ff=512, n_head=4, n_head_kv=2, head_dim=128, n_vocab=300, n_ctx=64,
             rope_theta=1e6, norm_eps=1e-6, kind=Q8_0, head_kind=Q8_0)
MOE = dict(DENSE, n_ff=0, n_expert=8, top_k=2, n_ff_expert=256, expert_kind=Q3_K, n_layer=1)


@pytest.fixture(scope="module")
def dense_file(tmp_path_factory):
    path = str(tmp_path_factory.mktemp("gguf") / "dense.gguf")
    host = gf.host_model(np.random.default_rng(1), DENSE)
    return gf.write_model(path, DENSE, host)[0], host


def test_tensor_table_equals_gguf_reader(ugb, dense_file):
    import gguf
    path, _ = dense_file
    g = ugb.Gguf.open(path)
    r = gguf.GGUFReader(path)
    ours = g.tensors()
    assert len(ours) == len(r.tensors) == g.info()["n_tensors"] == g.info()["total_tensors"]
    for t, rt in zip(ours, r.tensors):
        assert t.name.decode() == rt.name
        assert [int(d) for d in t.dims[:t.rank]] == [int(d) for d in rt.shape]
        assert all(int(d) == 1 for d in t.dims[t.rank:])
        assert (t.kind, t.offset, t.bytes) == (int(rt.tensor_type), rt.data_offset, rt.n_bytes)
        assert t.bytes == t.row_bytes * int(np.prod([int(d) for d in rt.shape[1:]], dtype=np.int64))
        assert t.offset % 32 == 0
        f = g.tensor(t.name.decode())
        assert (f.offset, f.bytes) == (t.offset, t.bytes)
    with pytest.raises(ugb.GgufError) as e:
        g.tensor("blk.9.attn_q.weight")
    assert e.value.name == "missing"


def test_metadata_values(ugb, dense_file):
    path, _ = dense_file
    g = ugb.Gguf.open(path)
    assert g.meta("general.architecture") == "qwen2"
    assert g.meta("qwen2.block_count") == 2
    assert g.meta("qwen2.embedding_length") == 256
    assert g.meta("qwen2.rope.freq_base") == 1e6
    assert g.meta("qwen2.attention.layer_norm_rms_epsilon") == np.float32(1e-6)
    assert g.meta("general.name") == "synthetic ügb model"
    assert g.meta("test.numbers") == [3, 1, 4, 1, 5]
    assert g.meta("tokenizer.ggml.tokens") == [f"tok{i}" for i in range(16)]
    with pytest.raises(ugb.GgufError) as e:  # int32 elements are not unsigned (Value::unsigned)
        g.meta("test.signed")
    assert e.value.name == "type"
    with pytest.raises(ugb.GgufError) as e:
        g.meta("no.such.key")
    assert e.value.name == "missing"


def test_rows_and_experts(ugb, tmp_path):
    host = gf.host_model(np.random.default_rng(2), MOE)
    path = gf.write_model(str(tmp_path / "moe.gguf"), MOE, host)[0]
    g = ugb.Gguf.open(path)
    experts = 0
    for t in g.tensors():
        rows = t.bytes // t.row_bytes
        assert ugb.Gguf.rows(t, 0, rows) == (t.offset, t.bytes)
        with pytest.raises(ugb.GgufError) as e:
            ugb.Gguf.rows(t, rows, 1)
        assert e.value.name == "tensor_bounds"
        if t.rank == 3:
            experts += 1
            assert t.dims[2] == MOE["n_expert"]
            first, last = ugb.Gguf.expert(t, 0), ugb.Gguf.expert(t, MOE["n_expert"] - 1)
            assert first[0] == t.offset and last[0] + last[1] == t.offset + t.bytes
            with pytest.raises(ugb.GgufError) as e:
                ugb.Gguf.expert(t, MOE["n_expert"])
            assert e.value.name == "shape"
    assert experts == 3
    with pytest.raises(ugb.GgufError) as e:
        ugb.Gguf.expert(g.tensor("blk.0.attn_q.weight"), 0)
    assert e.value.name == "shape"


def synthetic(offsets, width):
    """frontier_gguf.rs:238-249: a directory of rank-2 Q8_0 tensors [width, 2] at the given offsets."""
    out = bytearray(b"GGUF") + struct.pack("<IQQ", 3, len(offsets), 0)
    for i, off in enumerate(offsets):
        name = f"tensor.{i}".encode()
        out += struct.pack("<Q", len(name)) + name + struct.pack("<IQQIQ", 2, width, 2, 8, off)
    return bytes(out)


@pytest.mark.parametrize("offsets,width,logical,want", [
    ([0, 32], 32, 10000, "overlap"),
    ([1], 32, 10000, "alignment"),
    ([2 ** 64 - 32], 32, 2 ** 64 - 1, "overflow"),
    ([0], 2 ** 64 - 32, 2 ** 64 - 1, "overflow"),
    ([0], 33, 10000, "shape"),
    ([0, 96], 32, 10000, "ok"),
])
def test_reference_malformed_ranges(ugb, offsets, width, logical, want):
    data = synthetic(offsets, width)
    if want == "ok":
        ugb.Gguf(data, logical)
    else:
        with pytest.raises(ugb.GgufError) as e:
            ugb.Gguf(data, logical)
        assert e.value.name == want


def test_reference_truncation_version_limits(ugb, dense_file):
    path, _ = dense_file
    raw = open(path, "rb").read()
    g = ugb.Gguf.open(path)
    hdr = raw[:g.info()["data_offset"]]
    for n in [0, 3, 4, 7, 8, 23, 24, 1024, len(hdr) - 64]:  # (the last 32 header bytes may be padding)
        with pytest.raises(ugb.GgufError):
            ugb.Gguf(hdr[:n], len(raw))
    with pytest.raises(ugb.GgufError) as e:  # the file is shorter than its tensors
        ugb.Gguf(hdr, len(raw) - 1)
    assert e.value.name == "tensor_bounds"
    bad = bytearray(hdr)
    bad[8:16] = struct.pack("<Q", 2 ** 64 - 1)
    with pytest.raises(ugb.GgufError) as e:
        ugb.Gguf(bytes(bad), len(raw))
    assert e.value.name == "limit"
    bad = bytearray(hdr)
    bad[4] = 2
    with pytest.raises(ugb.GgufError) as e:
        ugb.Gguf(bytes(bad), len(raw))
    assert e.value.name == "version"
    bad = bytearray(hdr)
    bad[0:4] = b"GGUG"
    with pytest.raises(ugb.GgufError) as e:
        ugb.Gguf(bytes(bad), len(raw))
    assert e.value.name == "magic"


def kv_directory(*items):
    """A directory with no tensors and the given (key, kind, value bytes) entries."""
    out = bytearray(b"GGUF") + struct.pack("<IQQ", 3, 0, len(items))
    for key, kind, payload in items:
        k = key.encode()
        out += struct.pack("<Q", len(k)) + k + struct.pack("<I", kind) + payload
    return bytes(out)


def test_metadata_errors(ugb):
    s = lambda t: struct.pack("<Q", len(t)) + t  # noqa: E731
    with pytest.raises(ugb.GgufError) as e:
        ugb.Gguf(kv_directory(("a", 4, b"\0" * 4), ("a", 4, b"\0" * 4)), 100)
    assert e.value.name == "duplicate"
    with pytest.raises(ugb.GgufError) as e:  # nested arrays
        ugb.Gguf(kv_directory(("a", 9, struct.pack("<IQ", 9, 1) + struct.pack("<IQ", 4, 0))), 100)
    assert e.value.name == "type"
    with pytest.raises(ugb.GgufError) as e:  # unknown value type
        ugb.Gguf(kv_directory(("a", 13, b"")), 100)
    assert e.value.name == "type"
    with pytest.raises(ugb.GgufError) as e:
        ugb.Gguf(kv_directory(("a", 8, s(b"\xff\xfe"))), 100)
    assert e.value.name == "utf8"
    with pytest.raises(ugb.GgufError) as e:
        ugb.Gguf(kv_directory(("a" * 257, 4, b"\0" * 4)), 1000)
    assert e.value.name == "limit"
    with pytest.raises(ugb.GgufError) as e:
        ugb.Gguf(kv_directory(("general.alignment", 4, struct.pack("<I", 48))), 100)
    assert e.value.name == "alignment"
    with pytest.raises(ugb.GgufError) as e:  # split.no must be below split.count
        ugb.Gguf(kv_directory(("split.no", 2, struct.pack("<H", 3)), ("split.count", 2, struct.pack("<H", 3))), 100)
    assert e.value.name == "split"
    g = ugb.Gguf(kv_directory(("split.no", 2, struct.pack("<H", 1)), ("split.count", 2, struct.pack("<H", 3)),
                              ("split.tensors.count", 5, struct.pack("<i", 7))), 1000)
    assert g.info()["split_no"] == 1 and g.info()["split_count"] == 3 and g.info()["total_tensors"] == 7


def test_split_model_index(ugb, tmp_path):
    host = gf.host_model(np.random.default_rng(3), DENSE)
    files = gf.write_model(str(tmp_path / "split.gguf"), DENSE, host, split_max_tensors=9)
    assert len(files) == 3
    shards = [ugb.Gguf.open(f) for f in files]
    ugb.gguf_check_index(shards)
    ugb.gguf_check_index(list(reversed(shards)))  # order of the list does not matter
    one = ugb.Gguf.open(gf.write_model(str(tmp_path / "one.gguf"), DENSE, host)[0])
    assert ugb.gguf_inventory(shards) == ugb.gguf_inventory([one])
    assert ugb.gguf_inventory(shards)[0] == sum(t.bytes for t in one.tensors())
    with pytest.raises(ugb.GgufError) as e:
        ugb.gguf_check_index(shards[:2])
    assert e.value.name == "split"
    with pytest.raises(ugb.GgufError) as e:
        ugb.gguf_check_index([shards[0], shards[1], shards[1]])
    assert e.value.name == "split"


def test_decoder_config_and_weights(ugb, dense_file, tmp_path):
    path, host = dense_file
    g = ugb.Gguf.open(path)
    cfg = ugb.gguf_decoder_config([g])
    for k in ("n_layer", "n_embd", "n_ff", "n_head", "n_head_kv", "head_dim", "n_vocab", "n_ctx", "kind",
              "head_kind"):
        assert cfg[k] == DENSE[k], k
    assert cfg["rope_theta"] == 1e6 and cfg["norm_eps"] == np.float32(1e-6) and cfg["batch"] == 1
    base, off = 0x7f0000000000, g.info()["data_offset"]
    size = __import__("os").path.getsize(path) - off
    w, layers = ugb.gguf_model_weights([g], [base], [off], [size], cfg)
    at = lambda name: base + g.tensor(name).offset - off  # noqa: E731
    assert w.tok_embd == at("token_embd.weight") and w.output == w.tok_embd  # tied head
    assert w.output_norm == at("output_norm.weight")
    for li in range(cfg["n_layer"]):
        L = layers[li]
        for field, name in (("wq", "attn_q.weight"), ("wk", "attn_k.weight"), ("wv", "attn_v.weight"),
                            ("wo", "attn_output.weight"), ("w_gate", "ffn_gate.weight"), ("w_up", "ffn_up.weight"),
                            ("w_down", "ffn_down.weight"), ("attn_norm", "attn_norm.weight"),
                            ("ffn_norm", "ffn_norm.weight"), ("bq", "attn_q.bias")):
            assert getattr(L, field) == at(f"blk.{li}.{name}"), (li, field)
        assert L.router is None and L.gate_exps is None
    # a vocabulary shard's head starts at its first row
    w2, _ = ugb.gguf_model_weights([g], [base], [off], [size], dict(cfg, vocab0=100, n_vocab_local=50))
    assert w2.output == w.tok_embd + 100 * g.tensor("token_embd.weight").row_bytes
    # a device copy that ends before a tensor is refused
    with pytest.raises(ugb.GgufError) as e:
        ugb.gguf_model_weights([g], [base], [off], [size - 1], cfg)
    assert e.value.name == "tensor_bounds"
    with pytest.raises(ugb.GgufError) as e:  # the wrong kind for the layers
        ugb.gguf_model_weights([g], [base], [off], [size], dict(cfg, kind=Q4_K))
    assert e.value.name == "type"


def test_moe_config_and_expert_shard(ugb, tmp_path):
    host = gf.host_model(np.random.default_rng(4), MOE)
    path = gf.write_model(str(tmp_path / "moe.gguf"), MOE, host)[0]
    g = ugb.Gguf.open(path)
    cfg = ugb.gguf_decoder_config([g])
    for k in ("n_expert", "top_k", "n_ff_expert", "expert_kind"):
        assert cfg[k] == MOE[k], k
    assert cfg["n_ff"] == 0
    base, off = 0x10000000, g.info()["data_offset"]
    size = __import__("os").path.getsize(path) - off
    _, layers = ugb.gguf_model_weights([g], [base], [off], [size], dict(cfg, expert0=4, n_expert_local=4))
    t = g.tensor("blk.0.ffn_down_exps.weight")
    assert layers[0].down_exps == base + ugb.Gguf.expert(t, 4)[0] - off
    assert layers[0].router == base + g.tensor("blk.0.ffn_gate_inp.weight").offset - off
