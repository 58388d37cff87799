"""SAM 2 / 2.1 Hiera encoder: oracle checks on CPU and the B200 engine against
the oracle on GPU (through the C ABI).

The SAM 2 reference dump (tests/dump_sam2_reference.py) needs the external
sam2 package, so the Hiera oracle is pinned component-wise: its bicubic PE
resampling against PyTorch's bicubic (the op the reference's C++ bicubic
reproduces, sam3.cpp:4070-4109), and through the shared building blocks that
the ViT / memory-attention fixtures pin."""
import numpy as np
import pytest

from oracle import hiera as oh
from oracle import quant as oq
from parity import assert_close


def test_oracle_bicubic_matches_torch():
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(0)
    src = rng.standard_normal((16, 7, 7)).astype(np.float32)
    for H, W in ((256, 256), (64, 64), (37, 50)):
        ref = torch.nn.functional.interpolate(torch.from_numpy(src)[None], size=(H, W), mode="bicubic",
                                              align_corners=False)[0].numpy()
        np.testing.assert_allclose(oh.bicubic(src, H, W), ref, rtol=1e-5, atol=1e-5)


def test_oracle_window_path_matches_reference():
    """The oracle's padded window partition / unpartition and the Hiera q-stride path (partition at ws, 2x2 max
    pool per window, unpartition at ws // 2 onto the halved padded grid, crop) against the reference's own
    window_partition / window_unpartition (tests/dump_vit_reference.py:64-86; fixture by
    tests/golden/make_golden.py). Pure data movement and max: bit-exact."""
    import json
    import os
    from oracle import nn
    g = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "window_golden.npz"))
    meta = json.loads(str(g["meta"]))
    rng = np.random.default_rng(meta["seed"])
    for c, (shape, ws) in enumerate(meta["cases"]):
        x = rng.standard_normal(tuple(shape)).astype(np.float32)
        win, pad_hw = nn.window_partition(x, ws)
        assert tuple(pad_hw) == tuple(g[f"case{c}_pad_hw"]), c
        assert np.array_equal(win, g[f"case{c}_windows"]), c
        assert np.array_equal(nn.window_unpartition(win, ws, pad_hw, tuple(shape[1:3])), x), c
        key = f"case{c}_qpool_unpartition"
        if key in g:
            B, H, W, C = shape
            ws2, th, tw = ws // 2, H // 2, W // 2
            pad2 = (th + (ws2 - th % ws2) % ws2, tw + (ws2 - tw % ws2) % ws2)
            got = nn.window_unpartition(nn.maxpool2(win), ws2, pad2, (th, tw))
            assert np.array_equal(got, g[key]), c


def test_hiera_block_metadata(s3b):
    """Per-block dims / heads / windows / q-stride of Hiera-T (sam3.cpp:1676-1742)."""
    from sam3_b200 import synth
    b = synth.HIERA_T.blocks()
    assert [x[3] for x in b] == [8, 8, 4, 4, 14, 0, 14, 0, 14, 0, 14, 7]
    assert [i for i, x in enumerate(b) if x[4]] == [1, 3, 10]
    assert [x[1] for x in b] == [96, 192, 192, 384, 384, 384, 384, 384, 384, 384, 768, 768]


def small_cfgs(synth):
    return {
        # hd 96, padded windows at stage 2 (16 -> 28), q-stride with padded unpartition at block 5, one global block
        "t": synth.Sam2Config(img_size=256, embed=96, heads=1, stages=(1, 2, 2, 1), global_idx=(4,),
                              window_spec=(8, 4, 14, 7)),
        # Hiera-L-like head dim 72
        "l": synth.Sam2Config(img_size=256, embed=144, heads=2, stages=(1, 2, 2, 1), global_idx=(3,),
                              window_spec=(8, 4, 16, 8)),
    }


@pytest.mark.gpu
@pytest.mark.parametrize("name,qtype", [("t", None), ("t", 2), ("l", 8)])
def test_hiera_small_vs_oracle(engine, s3b, tmp_path, name, qtype):
    from sam3_b200 import synth
    cfg = small_cfgs(synth)[name]
    path = str(tmp_path / "h.ggml")
    T = synth.write_sam2(path, cfg, seed=4, ftype=1, qtype=qtype, quantize=s3b.quantize_rows, ln_random=True)
    W = synth.stored_values(T, 1, qtype, oq.quantize, oq.dequantize)
    engine.load_model(path)
    frames = synth.frames_u8(2, cfg.img_size, base_seed=31)
    chw = oh.preprocess_u8(frames)
    stages = oh.backbone(W, chw, cfg)
    fpn = oh.fpn(W, stages, cfg)
    engine.encode_u8(frames)
    for f in range(2):
        for i in range(3):
            got = engine.output(f"neck_trk_{i}", f)
            assert got.shape == fpn[i][f].shape, (got.shape, fpn[i][f].shape)
            assert_close(got, fpn[i][f], 0.9999, 0.01, 0.05, f"{name} fpn {i} frame {f}")
    # backbone state after every block (stage runner)
    ends = np.cumsum(cfg.stages) - 1
    for nb in range(1, sum(cfg.stages) + 1):
        if nb - 1 not in ends:
            continue
        engine.set_option("stop_after_blocks", nb)
        try:
            engine.encode_u8(frames[:1])
            got = engine.output("backbone", 0)
        finally:
            engine.set_option("stop_after_blocks", -1)
        ref = stages[list(ends).index(nb - 1)][0]
        assert_close(got, ref, 0.9999, 0.01, 0.05, f"{name} stage after block {nb - 1}")


@pytest.mark.gpu
def test_hiera_u8_entry_matches_chw(engine, s3b, tmp_path):
    """The uint8 path normalises the frames inside the patch-column kernel; it gives the bits of the f32
    CHW path fed with the same normalisation (the oracle's, f32 (p / 255 - mean) / std), from host and
    device memory, for frames of the model size and for frames the device resize brings to it."""
    import torch
    from sam3_b200 import synth
    cfg = small_cfgs(synth)["t"]
    path = str(tmp_path / "h_u8.ggml")
    synth.write_sam2(path, cfg, seed=8, ftype=1)
    engine.load_model(path)
    frames = synth.frames_u8(3, cfg.img_size, base_seed=77)
    engine.encode_chw(oh.preprocess_u8(frames))
    ref = [[engine.output(f"neck_trk_{i}", f) for i in range(3)] for f in range(3)]
    engine.encode_u8(frames)
    host = [[engine.output(f"neck_trk_{i}", f) for i in range(3)] for f in range(3)]
    engine.encode_u8(torch.from_numpy(frames).cuda())
    dev = [[engine.output(f"neck_trk_{i}", f) for i in range(3)] for f in range(3)]
    engine.encode_image_u8(frames)  # the model size: no resize, the fused path
    img = [[engine.output(f"neck_trk_{i}", f) for i in range(3)] for f in range(3)]
    for f in range(3):
        for i in range(3):
            assert np.array_equal(host[f][i], ref[f][i]), (f, i)
            assert np.array_equal(dev[f][i], ref[f][i]), (f, i)
            assert np.array_equal(img[f][i], ref[f][i]), (f, i)


@pytest.mark.gpu
def test_hiera_t_full_vs_oracle(engine, s3b, tmp_path):
    """SAM 2.1 Hiera-Tiny at 1024^2 (BASELINE configs[0] shape), f16 weights, one frame."""
    from sam3_b200 import synth
    cfg = synth.HIERA_T
    path = str(tmp_path / "hiera_t.ggml")
    T = synth.write_sam2(path, cfg, seed=0, ftype=1, ln_random=True)
    W = synth.stored_values(T, 1, None)
    engine.load_model(path)
    frames = synth.frames_u8(1, 1024, base_seed=1000)
    engine.encode_u8(frames)
    fpn = oh.fpn(W, oh.backbone(W, oh.preprocess_u8(frames), cfg), cfg)
    for i in range(3):
        got = engine.output(f"neck_trk_{i}", 0)
        assert got.shape == (256 >> i, 256 >> i, 256)
        print(assert_close(got, fpn[i][0], 0.9999, 0.01, 0.05, f"hiera-t fpn {i}"))
