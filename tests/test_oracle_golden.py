"""Pin the CPU oracle before trusting it (CPU only).

* Decoders vs the gguf 0.19.0 golden vectors (llama.cpp's Python port of ggml's formats), and
  vs the reference's own operator fixture (frontier_gpu.rs:37-50).
* fp16 decode vs IEEE binary16 for all 65536 bit patterns (frontier_core.rs:60-65).
* Activation quantiser vs an independent numpy float32 statement (gpu_dp4a.cu:23-31).
* Integer block dots vs independent numpy integer decodes of the raw bytes.
* row_bytes and the descriptor ABI vs the reference's own unit tests
  (frontier_core.rs:129-134, frontier_dispatch.rs:33-71).
* The reference's other formats (Q6_K, IQ3_XXS, IQ4_NL, IQ4_XS, frontier_core.rs:80-101): the
  same three pins, and the IQ3_XXS grid compiled into libugb vs the gguf package's.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import golden

Q8_0, Q3_K, Q4_K = 8, 11, 12
Q6_K, IQ3_XXS, IQ4_NL, IQ4_XS = 14, 18, 20, 23
IQ4 = np.array([-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113], dtype=np.int64)


# ---- independent numpy integer decoders (restating gguf's reshape-based bit maps) ----------

def q8_0_ints(raw: np.ndarray):
    b = raw.reshape(-1, 34)
    d = b[:, :2].copy().view(np.float16).astype(np.float32).reshape(-1)
    q = b[:, 2:].view(np.int8).astype(np.int64)
    return d, q  # q [nblocks, 32]


def q4_k_ints(raw: np.ndarray):
    b = raw.reshape(-1, 144)
    n = b.shape[0]
    d = b[:, 0:2].copy().view(np.float16).astype(np.float32).reshape(-1)
    dmin = b[:, 2:4].copy().view(np.float16).astype(np.float32).reshape(-1)
    sc12 = b[:, 4:16].reshape(n, 3, 4)
    dd, mm, md = sc12[:, 0], sc12[:, 1], sc12[:, 2]
    sc = np.concatenate([dd & 0x3F, (md & 0x0F) | ((dd >> 2) & 0x30)], axis=1).astype(np.int64)
    mn = np.concatenate([mm & 0x3F, (md >> 4) | ((mm >> 2) & 0x30)], axis=1).astype(np.int64)
    qs = b[:, 16:].reshape(n, 4, 1, 32) >> np.array([0, 4], dtype=np.uint8).reshape(1, 1, 2, 1)
    q = (qs & 0x0F).reshape(n, 8, 32).astype(np.int64)
    return d, dmin, sc, mn, q  # q [n, 8 sub-blocks, 32]


def q3_k_ints(raw: np.ndarray):
    b = raw.reshape(-1, 110)
    n = b.shape[0]
    hm = b[:, 0:32]
    qs = b[:, 32:96]
    s = b[:, 96:108]
    d = b[:, 108:110].copy().view(np.float16).astype(np.float32).reshape(-1)
    lo4 = np.concatenate([s[:, :8] & 15, s[:, :8] >> 4], axis=1)
    hi2 = (s[:, 8:12].reshape(n, 1, 4) >> np.array([0, 2, 4, 6], dtype=np.uint8).reshape(1, 4, 1)) & 3
    sc = (lo4 | (hi2.reshape(n, 16) << 4)).astype(np.int64) - 32
    lo = (qs.reshape(n, 2, 1, 32) >> np.array([0, 2, 4, 6], dtype=np.uint8).reshape(1, 1, 4, 1)) & 3
    lo = lo.reshape(n, 256).astype(np.int64)
    h = (hm.reshape(n, 1, 32) >> np.arange(8, dtype=np.uint8).reshape(1, 8, 1)) & 1
    h = h.reshape(n, 256).astype(np.int64)
    q = lo - 4 * (1 - h)
    return d, sc, q  # q [n, 256], sc [n, 16]


def _f16(b: np.ndarray) -> np.ndarray:
    return b.copy().view(np.float16).astype(np.float32).reshape(-1)


def q6_k_ints(raw: np.ndarray):
    """q [n, 256] in [-32, 31] and the int8 scale of each element's 16-group."""
    b = raw.reshape(-1, 210)
    n = b.shape[0]
    ql, qh = b[:, :128].astype(np.int64), b[:, 128:192].astype(np.int64)
    sc = b[:, 192:208].view(np.int8).astype(np.int64)
    d = _f16(b[:, 208:210])
    q = np.empty((n, 256), np.int64)
    s = np.empty((n, 256), np.int64)
    for h in range(2):
        for g in range(4):
            low = (ql[:, 64 * h + 32 * (g % 2): 64 * h + 32 * (g % 2) + 32] >> (4 * (g // 2))) & 15
            high = (qh[:, 32 * h: 32 * h + 32] >> (2 * g)) & 3
            q[:, 128 * h + 32 * g: 128 * h + 32 * g + 32] = (low | (high << 4)) - 32
            s[:, 128 * h + 32 * g: 128 * h + 32 * g + 16] = sc[:, 8 * h + 2 * g, None]
            s[:, 128 * h + 32 * g + 16: 128 * h + 32 * g + 32] = sc[:, 8 * h + 2 * g + 1, None]
    return d, s, q


def iq4_nl_ints(raw: np.ndarray):
    b = raw.reshape(-1, 18)
    qs = b[:, 2:].astype(np.int64)
    idx = np.concatenate([qs & 15, qs >> 4], axis=1)
    return _f16(b[:, :2]), IQ4[idx]  # values [n, 32]


def iq4_xs_ints(raw: np.ndarray):
    b = raw.reshape(-1, 136)
    n = b.shape[0]
    d = _f16(b[:, :2])
    sh = (b[:, 2].astype(np.int64) | (b[:, 3].astype(np.int64) << 8))
    sl = b[:, 4:8].astype(np.int64)
    sc = np.stack([((sl[:, j // 2] >> (4 * (j % 2))) & 15) | (((sh >> (2 * j)) & 3) << 4) for j in range(8)], axis=1)
    qs = b[:, 8:].reshape(n, 8, 16).astype(np.int64)
    idx = np.concatenate([qs & 15, qs >> 4], axis=2)  # [n, 8, 32]
    return d, sc - 32, IQ4[idx]


def iq3_xxs_ints(raw: np.ndarray, grid_words: np.ndarray):
    b = raw.reshape(-1, 98)
    n = b.shape[0]
    d = _f16(b[:, :2])
    idx = b[:, 2:66].astype(np.int64).reshape(n, 8, 8)
    aux = b[:, 66:98].copy().view(np.uint32).astype(np.int64).reshape(n, 8)
    mag = (grid_words[idx][..., None] >> (8 * np.arange(4))) & 255  # [n, 8, 8, 4]
    mag = mag.reshape(n, 8, 32)
    signs = np.empty((n, 8, 32), np.int64)
    for g in range(4):
        s7 = (aux >> (7 * g)) & 127
        par = np.array([bin(int(v)).count("1") & 1 for v in s7.reshape(-1)], np.int64).reshape(n, 8)
        s8 = s7 | (par << 7)
        for e in range(8):
            signs[:, :, 8 * g + e] = np.where((s8 >> e) & 1, -1, 1)
    scale = d[:, None] * (np.float32(0.5) + (aux >> 28).astype(np.float32)) * np.float32(0.5)
    return scale.astype(np.float32), mag * signs  # values [n, 8, 32]


# ---- decoders vs gguf --------------------------------------------------------------------

@pytest.mark.parametrize("name,kind", [("q8_0", Q8_0), ("q4_k", Q4_K), ("q3_k", Q3_K), ("q6_k", Q6_K),
                                       ("iq3_xxs", IQ3_XXS), ("iq4_nl", IQ4_NL), ("iq4_xs", IQ4_XS)])
def test_dequant_matches_gguf_bit_exact(orc, name, kind):
    g = golden(f"dequant_{name}.npz")
    raw, values = g["raw"], g["values"]
    out = orc.dequantize(kind, raw, values.size)
    np.testing.assert_array_equal(out.view(np.uint32), values.view(np.uint32))


def test_reference_fixture_q8_0(orc):
    """frontier_gpu.rs:37-50 operator fixture: xorshift bytes, cycling fp16 scales."""
    g = golden("fixture_q8_0.npz")
    n, m = int(g["n"]), int(g["m"])
    out = orc.dequantize(Q8_0, g["raw"], n * m)
    np.testing.assert_array_equal(out.view(np.uint32), g["values"].view(np.uint32))
    # the scales cycle through the reference's four fp16 patterns
    blocks = g["raw"].reshape(-1, 34)
    h = blocks[:, 0].astype(np.uint16) | (blocks[:, 1].astype(np.uint16) << 8)
    assert list(h[:4]) == [0x2000, 0x2800, 0x3000, 0xB000]


def test_half_all_patterns(orc):
    bits = np.arange(65536, dtype=np.uint32)
    want = bits.astype(np.uint16).view(np.float16).astype(np.float32)
    lib = orc.lib()
    got = np.array([lib.orc_half(int(b)) for b in bits], dtype=np.float32)
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(got), nan)
    np.testing.assert_array_equal(got[~nan].view(np.uint32), want[~nan].view(np.uint32))


def test_quant_act_matches_numpy_golden(orc):
    g = golden("quant_act.npz")
    q, d, s, bad = orc.quant_act(g["x"])
    assert bad == 0
    np.testing.assert_array_equal(q, g["q"])
    np.testing.assert_array_equal(d.view(np.uint32), g["d"].view(np.uint32))
    np.testing.assert_array_equal(s, g["s"])
    # ties round to even: block 0 has a = 127, inv = 1
    assert list(q[1:8]) == [0, 2, 2, 0, -2, -2, 4]


def test_quant_act_nonfinite_flagged(orc):
    x = np.ones(64, dtype=np.float32)
    x[3] = np.nan
    x[40] = np.inf
    q, d, s, bad = orc.quant_act(x)
    assert bad == 1
    assert q[3] == 0 and q[40] == 0
    assert np.isfinite(d).all()


# ---- integer block dots -------------------------------------------------------------------

def _rand_act(rng, k):
    return rng.integers(-127, 128, size=k, dtype=np.int64).astype(np.int8)


def test_block_dots_q8_0(orc):
    g = golden("dequant_q8_0.npz")
    raw = g["raw"]
    k = raw.size // 34 * 32
    x = _rand_act(np.random.default_rng(1), k)
    d, q = q8_0_ints(raw)
    want = (q * x.reshape(-1, 32).astype(np.int64)).sum(axis=1)
    np.testing.assert_array_equal(orc.block_dots(Q8_0, raw, x), want)
    # the integer view reproduces the gguf values exactly
    vals = (d[:, None] * q.astype(np.float32)).reshape(-1)
    np.testing.assert_array_equal(vals.view(np.uint32), g["values"].view(np.uint32))


def test_block_dots_q4_k(orc):
    g = golden("dequant_q4_k.npz")
    raw = g["raw"]
    k = raw.size // 144 * 256
    x = _rand_act(np.random.default_rng(2), k)
    d, dmin, sc, mn, q = q4_k_ints(raw)
    want = (q.reshape(-1, 32) * x.reshape(-1, 32).astype(np.int64)).sum(axis=1)
    np.testing.assert_array_equal(orc.block_dots(Q4_K, raw, x), want)
    dl = (d[:, None] * sc.astype(np.float32))[:, :, None]
    ml = (dmin[:, None] * mn.astype(np.float32))[:, :, None]
    vals = (dl * q.astype(np.float32) - ml).reshape(-1).astype(np.float32)
    np.testing.assert_array_equal(vals.view(np.uint32), g["values"].view(np.uint32))


def test_block_dots_q3_k(orc):
    g = golden("dequant_q3_k.npz")
    raw = g["raw"]
    k = raw.size // 110 * 256
    x = _rand_act(np.random.default_rng(3), k)
    d, sc, q = q3_k_ints(raw)
    xs = x.astype(np.int64).reshape(-1, 16)
    halves = (q.reshape(-1, 16) * xs).sum(axis=1) * sc.reshape(-1)
    want = halves.reshape(-1, 2).sum(axis=1)
    np.testing.assert_array_equal(orc.block_dots(Q3_K, raw, x), want)
    vals = ((d[:, None] * sc.astype(np.float32)).repeat(16, axis=1) * q.astype(np.float32))
    np.testing.assert_array_equal(vals.reshape(-1).astype(np.float32).view(np.uint32),
                                  g["values"].view(np.uint32))


def test_block_dots_q6_k(orc):
    g = golden("dequant_q6_k.npz")
    raw = g["raw"]
    x = _rand_act(np.random.default_rng(6), raw.size // 210 * 256)
    d, s, q = q6_k_ints(raw)
    halves = (q.reshape(-1, 16) * x.astype(np.int64).reshape(-1, 16)).sum(axis=1) * s.reshape(-1, 16)[:, 0]
    np.testing.assert_array_equal(orc.block_dots(Q6_K, raw, x), halves.reshape(-1, 2).sum(axis=1))
    vals = ((d[:, None] * s.astype(np.float32)) * q.astype(np.float32)).reshape(-1)
    np.testing.assert_array_equal(vals.view(np.uint32), g["values"].view(np.uint32))


def test_block_dots_iq4_nl(orc):
    g = golden("dequant_iq4_nl.npz")
    raw = g["raw"]
    x = _rand_act(np.random.default_rng(7), raw.size // 18 * 32)
    d, v = iq4_nl_ints(raw)
    np.testing.assert_array_equal(orc.block_dots(IQ4_NL, raw, x), (v * x.astype(np.int64).reshape(-1, 32)).sum(axis=1))
    vals = (d[:, None] * v.astype(np.float32)).reshape(-1)
    np.testing.assert_array_equal(vals.view(np.uint32), g["values"].view(np.uint32))


def test_block_dots_iq4_xs(orc):
    g = golden("dequant_iq4_xs.npz")
    raw = g["raw"]
    x = _rand_act(np.random.default_rng(8), raw.size // 136 * 256)
    d, sc, v = iq4_xs_ints(raw)
    np.testing.assert_array_equal(orc.block_dots(IQ4_XS, raw, x),
                                  (v.reshape(-1, 32) * x.astype(np.int64).reshape(-1, 32)).sum(axis=1))
    vals = ((d[:, None] * sc.astype(np.float32))[:, :, None] * v.astype(np.float32)).reshape(-1)
    np.testing.assert_array_equal(vals.view(np.uint32), g["values"].view(np.uint32))


def test_block_dots_iq3_xxs(orc):
    g = golden("dequant_iq3_xxs.npz")
    raw = g["raw"]
    x = _rand_act(np.random.default_rng(9), raw.size // 98 * 256)
    scale, v = iq3_xxs_ints(raw, orc.iq3_grid().astype(np.int64))
    np.testing.assert_array_equal(orc.block_dots(IQ3_XXS, raw, x),
                                  (v.reshape(-1, 32) * x.astype(np.int64).reshape(-1, 32)).sum(axis=1))
    vals = (scale[:, :, None] * np.abs(v).astype(np.float32)) * np.where(v < 0, -1, 1).astype(np.float32)
    np.testing.assert_array_equal(vals.reshape(-1).view(np.uint32), g["values"].view(np.uint32))


def test_iq3_grid_compiled_equals_gguf(orc):
    """The grid compiled into libugb (csrc/iq3_grid.inc, generated by csrc/gen_iq3_grid.py) is the
    one the gguf package decodes; its first entries are the reference's IQ3_GRID values."""
    import os
    import re
    inc = os.path.join(os.path.dirname(__file__), "..", "uefi-gpu_b200", "csrc", "iq3_grid.inc")
    words = np.array([int(w, 16) for w in re.findall(r"0x([0-9a-f]{8})u", open(inc).read())], np.uint32)
    np.testing.assert_array_equal(words, orc.iq3_grid())
    assert list(words[:4]) == [0x04040404, 0x04040414, 0x04040424, 0x04040C0C]


# ---- scaled matvec ---------------------------------------------------------------------------

@pytest.mark.parametrize("name,kind,elems,bsz", [("q8_0", Q8_0, 32, 34), ("q4_k", Q4_K, 256, 144),
                                                 ("q3_k", Q3_K, 256, 110), ("q6_k", Q6_K, 256, 210),
                                                 ("iq3_xxs", IQ3_XXS, 256, 98), ("iq4_nl", IQ4_NL, 32, 18),
                                                 ("iq4_xs", IQ4_XS, 256, 136)])
def test_matvec_vs_float64(orc, name, kind, elems, bsz):
    """The oracle's fp32 block-order sum vs an fp64 sum of dequantised weight x dequantised
    activation: the only difference is fp32 rounding."""
    g = golden(f"dequant_{name}.npz")
    raw = g["raw"]
    nblk = raw.size // bsz
    m = 4 if elems == 32 else 3
    k = nblk * elems // m
    k -= k % elems
    rb = k // elems * bsz
    w = raw[: m * rb]
    rng = np.random.default_rng(4)
    xf = rng.standard_normal(k).astype(np.float32)
    q, d, s, _ = orc.quant_act(xf)
    y = orc.matvec(kind, w, rb, q, d, s, k, m)[0]
    wdq = g["values"][: m * k].reshape(m, k).astype(np.float64)
    xdq = (q.astype(np.float64).reshape(-1, 32) * d.astype(np.float64)[:, None]).reshape(-1)
    ref = wdq @ xdq
    l1 = np.abs(wdq) @ np.abs(xdq)
    assert np.all(np.abs(y - ref) <= 1e-5 * l1 + 1e-30)


def test_matvec_mt_identical(orc):
    rng = np.random.default_rng(5)
    k, m = 1536, 37
    raw = rng.integers(0, 256, size=m * k // 32 * 34, dtype=np.uint8)
    raw.reshape(-1, 34)[:, 1] = 0x20  # finite fp16 scales
    q, d, s, _ = orc.quant_act(rng.standard_normal((2, k)).astype(np.float32))
    a = orc.matvec(Q8_0, raw, k // 32 * 34, q, d, s, k, m, 2)
    b = orc.matvec(Q8_0, raw, k // 32 * 34, q, d, s, k, m, 2, mt=True)
    np.testing.assert_array_equal(a.view(np.uint32), b.view(np.uint32))


# ---- reference unit-test known answers -------------------------------------------------------

def test_row_bytes_reference_cases(orc):
    # frontier_core.rs:129-134 rejects_bad_quant
    assert orc.row_bytes(23, 640) == -2  # Err(Shape)
    assert orc.row_bytes(20, 160) == 90
    assert orc.row_bytes(18, 2560) == 980
    assert orc.row_bytes(99, 256) == -1  # Err(QuantType)
    assert orc.row_bytes(Q8_0, 1536) == 1632
    assert orc.row_bytes(Q4_K, 3584) == 14 * 144
    assert orc.row_bytes(Q3_K, 4096) == 16 * 110


def _job(m, offset):
    # frontier_dispatch.rs:44-45
    return (0x400000000, 0x100010000, 0xE0000000 + offset, 18, 2560, m, 980)


@pytest.mark.parametrize("count", [1, 2, 3, 4, 11, 23, 32])
def test_dispatch_abi_and_padded_rows(orc, count):
    """frontier_dispatch.rs:46-67 abi_and_padded_row_mapping."""
    jobs, offset = [], 0
    for i in range(count):
        m = [1, 3, 640, 2560][i % 4]
        jobs.append(_job(m, offset))
        offset += m * 4
    packed = orc.dispatch_pack(jobs)
    assert packed is not None
    data, grid = packed
    assert len(data) == count * 48
    prefix = 0
    starts = []
    for i in range(count):
        rec = data[i * 48:(i + 1) * 48]
        assert int.from_bytes(rec[0:8], "little") == jobs[i][0]
        assert int.from_bytes(rec[8:16], "little") == jobs[i][1]
        assert int.from_bytes(rec[16:24], "little") == jobs[i][2]
        assert int.from_bytes(rec[40:44], "little") == prefix
        assert rec[44:48] == b"\0\0\0\0"
        starts.append(prefix)
        prefix += (jobs[i][5] + 3) & ~3
    seen = 0
    for row in range(grid * 4):
        lo, hi = 0, count
        while lo + 1 < hi:
            mid = (lo + hi) // 2
            if starts[mid] <= row:
                lo = mid
            else:
                hi = mid
        assert row // 4 * 4 >= starts[lo]
        if row - starts[lo] < jobs[lo][5]:
            seen += 1
    assert seen == sum(j[5] for j in jobs)


def test_dispatch_rejects(orc):
    """frontier_dispatch.rs:68-70 reject_aliases_overflows (minus the platform window)."""
    assert orc.dispatch_pack([]) is None
    assert orc.dispatch_pack([_job(1, 0)] * 33) is None
    assert orc.dispatch_pack([_job(640, 0), _job(640, 4)]) is None
    assert orc.dispatch_pack([_job(0, 0)]) is None
    assert orc.dispatch_pack([_job(0xFFFFFFFF, 0)]) is None
    j = list(_job(1, 0))
    j[0] = 2**64 - 1
    assert orc.dispatch_pack([tuple(j)]) is None
    j = list(_job(1, 0))
    j[1] = 2**64 - 1
    assert orc.dispatch_pack([tuple(j)]) is None


# ---- routing ------------------------------------------------------------------------------------

def test_moe_route_ties_and_weights(orc):
    logits = np.array([1.0, 3.0, 3.0, -2.0, 0.5, 3.0], dtype=np.float32)
    ids, w = orc.moe_route(logits, 3)
    assert list(ids) == [1, 2, 5]  # equal scores: lower id first (frontier_forward.rs:167)
    np.testing.assert_allclose(w, [1 / 3] * 3, rtol=1e-6)
    ids, w = orc.moe_route(logits, 4)
    assert list(ids) == [1, 2, 5, 0]
    assert abs(float(w.sum()) - 1.0) < 1e-6
    bad = logits.copy()
    bad[2] = np.nan
    assert orc.moe_route(bad, 2) is None


def test_prefill_repack_lossless(orc):
    rng = np.random.default_rng(6)
    n, k, n_pad = 20, 256, 128
    raw = rng.integers(0, 256, size=n * k // 32 * 34, dtype=np.uint8)
    qa, sa = orc.prefill_repack_q8_0(raw, n, k, n_pad)
    d, q = q8_0_ints(raw)
    np.testing.assert_array_equal(qa[:n].astype(np.int64), q.reshape(n, k))
    assert not qa[n:].any() and not sa[:, n:].any()
    np.testing.assert_array_equal(sa[:, :n].T.reshape(-1).view(np.uint32),
                                  d.astype(np.float32).view(np.uint32))
