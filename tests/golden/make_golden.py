"""Generate the committed golden vectors in tests/golden/.

Run in the build container (it needs the third-party ``gguf`` 0.19.0 package, llama.cpp's
Python port of ggml's block formats, which is not available on the GPU box):

    python tests/golden/make_golden.py

Outputs (all small .npz files):

* ``dequant_<kind>.npz``: seeded random raw blocks of Q8_0 / Q4_K / Q3_K, and of the reference's
  other formats Q6_K / IQ3_XXS / IQ4_NL / IQ4_XS, and the values ``gguf.quants.dequantize``
  decodes them to.  The oracle's decoders (oracle/ugb_oracle.c)
  and the CUDA block decoders are checked against these.  fp16 scales are drawn from a set
  that includes zero, subnormal, negative and large values.
* ``fixture_q8_0.npz``: the reference's own xorshift operator fixture
  (frontier_gpu.rs:37-50, kind 8, n=2560 x m=2) and its gguf dequantisation.
* ``quant_act.npz``: activation vectors with hand-made edge cases (exact .5 ties, zero
  blocks, a single non-zero, negative maxima, tiny and huge magnitudes) and their block-32
  quantisation computed here in numpy float32 exactly as gpu_dp4a.cu:23-31 /
  gpu_prefill.rs:105-106 state it (d = a/127, q = rint(x * (127/a)), clamp +-127, round
  half to even).  This is an implementation independent of the C oracle.
"""
from __future__ import annotations

import os

import numpy as np
import gguf
from gguf.constants import GGMLQuantizationType as T

HERE = os.path.dirname(os.path.abspath(__file__))

# fp16 bit patterns: zero, smallest subnormal, a subnormal, typical weight scales, negative,
# and large values.
SCALE_BITS = np.array([0x0000, 0x0001, 0x0210, 0x1419, 0x2000, 0x2800, 0x3000, 0xB000,
                       0x3C00, 0x4D00, 0x8000, 0x9C41, 0x1A0F, 0x2E66], dtype=np.uint16)


def _xorshift_bytes(count: int, seed: int = 0x13243546) -> np.ndarray:
    """frontier_gpu.rs:38-39: state ^= state<<13; state ^= state>>17; state ^= state<<5."""
    out = np.empty(count, dtype=np.uint8)
    state = seed
    for i in range(count):
        state ^= (state << 13) & 0xFFFFFFFF
        state ^= state >> 17
        state ^= (state << 5) & 0xFFFFFFFF
        out[i] = state & 0xFF
    return out


def reference_fixture_q8_0(n: int, m: int) -> np.ndarray:
    """frontier_gpu.rs:37-50 fixture(kind=8, n*m): xorshift bytes with the fp16 scale of
    block b overwritten by [0x2000, 0x2800, 0x3000, 0xb000][b % 4]."""
    total = n * m
    raw = _xorshift_bytes(total // 32 * 34)
    blocks = raw.reshape(-1, 34)
    halves = np.array([0x2000, 0x2800, 0x3000, 0xB000], dtype=np.uint16)
    for b in range(blocks.shape[0]):
        h = int(halves[b % 4])
        blocks[b, 0] = h & 0xFF
        blocks[b, 1] = h >> 8
    return blocks.reshape(-1)


def random_blocks(kind: T, nblocks: int, rng: np.random.Generator) -> np.ndarray:
    bsize = {T.Q8_0: 34, T.Q4_K: 144, T.Q3_K: 110, T.Q6_K: 210, T.IQ3_XXS: 98, T.IQ4_NL: 18, T.IQ4_XS: 136}[kind]
    raw = rng.integers(0, 256, size=(nblocks, bsize), dtype=np.uint8)
    scale_offsets = {T.Q8_0: [0], T.Q4_K: [0, 2], T.Q3_K: [108], T.Q6_K: [208], T.IQ3_XXS: [0],
                     T.IQ4_NL: [0], T.IQ4_XS: [0]}[kind]
    for b in range(nblocks):
        for off in scale_offsets:
            h = int(SCALE_BITS[rng.integers(0, len(SCALE_BITS))])
            raw[b, off] = h & 0xFF
            raw[b, off + 1] = h >> 8
    return raw


def quant_act_numpy(x: np.ndarray):
    x = x.astype(np.float32).reshape(-1, 32)
    a = np.max(np.abs(x), axis=1).astype(np.float32)
    d = (a / np.float32(127.0)).astype(np.float32)
    with np.errstate(divide="ignore"):
        inv = np.where(a > 0, np.float32(127.0) / a, np.float32(0.0)).astype(np.float32)
    prod = (x * inv[:, None]).astype(np.float32)
    q = np.clip(np.rint(prod), -127, 127).astype(np.int8)
    s = q.astype(np.int32).sum(axis=1).astype(np.int32)
    return q.reshape(-1), d, s


def activation_cases(rng: np.random.Generator) -> np.ndarray:
    blocks = []
    # Exact ties: a = 127 so inv = 1 and x*inv keeps the .5 fractions.
    tie = np.array([127.0, 0.5, 1.5, 2.5, -0.5, -1.5, -2.5, 3.5] + [0.0] * 24, dtype=np.float32)
    blocks.append(tie)
    blocks.append(np.zeros(32, dtype=np.float32))
    one = np.zeros(32, dtype=np.float32)
    one[7] = -3.25
    blocks.append(one)
    neg = rng.standard_normal(32).astype(np.float32)
    neg[5] = -40.0
    blocks.append(neg)
    blocks.append((rng.standard_normal(32) * 1e-30).astype(np.float32))
    blocks.append((rng.standard_normal(32) * 1e30).astype(np.float32))
    blocks.append(np.full(32, 7.0, dtype=np.float32))
    for _ in range(57):
        blocks.append(rng.standard_normal(32).astype(np.float32))
    return np.concatenate(blocks)


def main() -> None:
    rng = np.random.default_rng(20261201)
    for kind, name, nblocks in [(T.Q8_0, "q8_0", 96), (T.Q4_K, "q4_k", 12), (T.Q3_K, "q3_k", 12)]:
        raw = random_blocks(kind, nblocks, rng)
        values = gguf.quants.dequantize(raw.reshape(-1), kind).astype(np.float32).reshape(-1)
        np.savez_compressed(os.path.join(HERE, f"dequant_{name}.npz"), raw=raw.reshape(-1),
                            values=values, kind=np.int32(int(kind)))

    n, m = 2560, 2
    fixture = reference_fixture_q8_0(n, m)
    values = gguf.quants.dequantize(fixture, T.Q8_0).astype(np.float32).reshape(-1)
    np.savez_compressed(os.path.join(HERE, "fixture_q8_0.npz"), raw=fixture, values=values,
                        n=np.int32(n), m=np.int32(m))

    x = activation_cases(rng)
    q, d, s = quant_act_numpy(x)
    np.savez_compressed(os.path.join(HERE, "quant_act.npz"), x=x, q=q, d=d, s=s)

    # the reference's other formats, from a generator of their own so the files above keep
    # their bytes
    rng2 = np.random.default_rng(20261202)
    for kind, name, nblocks in [(T.Q6_K, "q6_k", 12), (T.IQ3_XXS, "iq3_xxs", 12), (T.IQ4_NL, "iq4_nl", 96),
                                (T.IQ4_XS, "iq4_xs", 12)]:
        raw = random_blocks(kind, nblocks, rng2)
        values = gguf.quants.dequantize(raw.reshape(-1), kind).astype(np.float32).reshape(-1)
        np.savez_compressed(os.path.join(HERE, f"dequant_{name}.npz"), raw=raw.reshape(-1),
                            values=values, kind=np.int32(int(kind)))
    print("golden vectors written to", HERE, "gguf", gguf.__file__)


if __name__ == "__main__":
    main()
