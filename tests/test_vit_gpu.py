"""SAM 3 image encoder (ViT + SimpleFPN neck) on the B200 engine against the
numpy oracle, through the C ABI (s3b_load_model / s3b_encode_* /
s3b_output_copy), on seeded synthetic .ggml models.

Tolerances: the engine rounds GEMM and attention operands to f16 (as ggml's
CPU path does for f16 weights); outputs must reach cosine >= 0.9999 against
the oracle's exact-f32 forward, with mean-abs <= 1% and max-abs <= 5% of the
reference's mean / max magnitude. The reference's own bar for this stage is
cos > 0.999 and mean < 0.05 (tests/test_phase3.cpp:516-577)."""
import os

import numpy as np
import pytest

from oracle import quant as oq
from oracle import vit as ov
from parity import assert_close

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def tiny_cfg(synth):
    return synth.Sam3Config(img_size=336, patch=14, embed=256, depth=3, heads=4, mlp_ratio_x1000=4625, window=8,
                            global_idx=(1,), neck_dim=64, neck_mid=128, visual_only=1)


@pytest.mark.parametrize("qtype", [None, 2, 8])
def test_vit_tiny_vs_oracle(engine, s3b, tmp_path, qtype):
    from sam3_b200 import synth
    cfg = tiny_cfg(synth)
    path = str(tmp_path / "tiny.ggml")
    T = synth.write_sam3(path, cfg, seed=3, ftype=1, qtype=qtype, quantize=s3b.quantize_rows, ln_random=True)
    W = synth.stored_values(T, 1, qtype, oq.quantize, oq.dequantize)
    engine.load_model(path)
    frames = synth.frames_u8(2, cfg.img_size, base_seed=1000)
    engine.encode_u8(frames)
    engine.sync()
    chw = ov.preprocess_u8(frames)
    x, _ = ov.backbone(W, chw, cfg)
    necks = ov.neck(W, x)
    for f in range(2):
        got = engine.output("vit_output", f)
        assert got.shape == x[f].shape
        assert_close(got, x[f], 0.9999, 0.01, 0.05, f"vit_output[{f}]")
        for i in range(4):
            gi = engine.output(f"neck_trk_{i}", f)
            assert gi.shape == necks[i][f].shape, (gi.shape, necks[i][f].shape)
            assert_close(gi, necks[i][f], 0.9999, 0.01, 0.05, f"neck_trk_{i}[{f}]")


def test_vit_tiny_chw_entry_matches_u8(engine, s3b, tmp_path):
    """sam3_encode_image_from_preprocessed path == uint8 path on the same frames."""
    from sam3_b200 import synth
    cfg = tiny_cfg(synth)
    path = str(tmp_path / "tiny.ggml")
    synth.write_sam3(path, cfg, seed=5, ftype=1)
    engine.load_model(path)
    frames = synth.frames_u8(1, cfg.img_size, base_seed=7)
    engine.encode_u8(frames)
    a = engine.output("neck_trk_2", 0)
    engine.encode_chw(ov.preprocess_u8(frames))
    b = engine.output("neck_trk_2", 0)
    assert np.array_equal(a, b)
    d = torch.from_numpy(ov.preprocess_u8(frames)).cuda()
    engine.encode_chw(d)
    c = engine.output("neck_trk_2", 0)
    assert np.array_equal(a, c)
