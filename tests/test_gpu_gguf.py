"""Decoders loaded from GGUF files (ugb_gguf_* + ugb_decoder_bind, the reference's
frontier_gguf.rs:145-200 directory and its tensors in place) decode exactly as decoders bound
to the same weights directly, dense and MoE, tied and untied heads, one file or a split set;
and a loaded model's step passes the layer-synchronised oracle check."""
from __future__ import annotations

import os

import numpy as np
import pytest

import gguf_files as gf
from test_gpu_decoder import MOE, SMALL, build_model
from test_gpu_decoder_shapes import check_step

pytestmark = pytest.mark.gpu

Q8_0, Q3_K, Q4_K = 8, 11, 12


@pytest.mark.parametrize("cfg,tied", [(SMALL, True), (dict(SMALL, kind=Q4_K, head_kind=Q4_K), False),
                                      (MOE, True)], ids=["dense-q8", "dense-q4k-untied", "moe-q3k"])
def test_loaded_equals_bound(ctx, ugb, tmp_path, cfg, tied):
    dev, host = build_model(ctx, ugb, cfg, seed=501)
    path = gf.write_model(str(tmp_path / "m.gguf"), cfg, host, tied=tied)[0]
    direct = ugb.Decoder(ctx, **cfg)
    direct.bind(dev["tok_embd"], dev["output_norm"], dev["output"], dev["layers"])
    loaded = ugb.load_gguf_decoder(ctx, path, n_ctx=cfg["n_ctx"])
    for pos, tok in enumerate([3, 77, 500, 999, 1]):
        a = direct.token(tok, pos)
        b = loaded.token(tok, pos)
        assert a == b
        np.testing.assert_array_equal(direct.logits().view(np.uint32), loaded.logits().view(np.uint32))
    assert ctx.status_read()[1] == 0
    direct.close()
    loaded.close()


def test_split_files_bind(ctx, ugb, tmp_path):
    """A model split over three files, each copied to its own device buffer."""
    import torch
    dev, host = build_model(ctx, ugb, SMALL, seed=502)
    files = gf.write_model(str(tmp_path / "s.gguf"), SMALL, host, split_max_tensors=9)
    shards = [ugb.Gguf.open(f) for f in files]
    cfg = ugb.gguf_decoder_config(shards)
    bufs, bases, offs, sizes = [], [], [], []
    for f, g in zip(files, shards):
        off = g.info()["data_offset"]
        data = np.fromfile(f, dtype=np.uint8, offset=off)
        t = torch.from_numpy(data).cuda()
        bufs.append(t)
        bases.append(t.data_ptr())
        offs.append(off)
        sizes.append(t.numel())
    w, layers = ugb.gguf_model_weights(shards, bases, offs, sizes, cfg)
    loaded = ugb.Decoder(ctx, **cfg)
    assert ugb.lib().ugb_decoder_bind(loaded.handle, __import__("ctypes").byref(w)) == 0
    direct = ugb.Decoder(ctx, **SMALL)
    direct.bind(dev["tok_embd"], dev["output_norm"], dev["output"], dev["layers"])
    for pos, tok in enumerate([5, 6, 7]):
        assert loaded.token(tok, pos) == direct.token(tok, pos)
        np.testing.assert_array_equal(loaded.logits(), direct.logits())
    loaded.close()
    direct.close()


def test_loaded_model_layer_synced(ctx, ugb, orc, tmp_path):
    """The 1.5B widths (one layer, full vocabulary) from a GGUF file, checked stage by stage."""
    from oracle.decode_ref import RefDecoder
    cfg = dict(n_layer=1, n_embd=1536, n_ff=8960, n_head=12, n_head_kv=2, head_dim=128, n_vocab=151936,
               n_ctx=512, rope_theta=1e6, norm_eps=1e-6, kind=Q8_0, head_kind=Q8_0)
    _, host = build_model(ctx, ugb, cfg, seed=503)
    path = gf.write_model(str(tmp_path / "c2.gguf"), cfg, host)[0]
    dec = ugb.load_gguf_decoder(ctx, path, n_ctx=512)
    dec.set_trace(True)
    ref = RefDecoder(cfg, host, mt=True)
    for pos in (0, 1, 2):  # attention is checked over the GPU's own cache
        check_step(orc, ref, dec, host, cfg, np.array([11 + pos]), pos)
    dec.close()
