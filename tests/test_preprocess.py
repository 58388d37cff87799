"""Frame preprocessing at any input size: the reference's uint8 bilinear resize
(sam3_resize_bilinear, sam3.cpp:3441-3481) followed by the SAM 3 / SAM 2
normalisation (3486-3544).

The oracle's resize is pinned against PyTorch's bilinear interpolation
(align_corners=False), which the reference's comment names as the op it
matches: equal everywhere except at exact half-way values, where torch rounds
half to even and the reference adds 0.5 and truncates. The engine must equal
the oracle bit for bit."""
import numpy as np
import pytest

from oracle import hiera as oh
from oracle import nn

SIZES = [((480, 640), (1008, 1008)), ((1500, 1200), (1024, 1024)), ((1, 1), (7, 5)), ((37, 91), (64, 48)),
         ((2000, 3000), (1008, 1008)), ((256, 256), (256, 256)), ((300, 17), (29, 301))]


def test_oracle_resize_matches_torch():
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(0)
    for (h, w), (dh, dw) in SIZES[:5]:
        img = rng.integers(0, 256, (h, w, 3), dtype=np.uint8)
        got = nn.resize_bilinear_u8(img, dw, dh)
        x = torch.from_numpy(img).permute(2, 0, 1)[None].double()
        v = torch.nn.functional.interpolate(x, size=(dh, dw), mode="bilinear", align_corners=False)
        v = v[0].permute(1, 2, 0).numpy()
        ref = np.clip(np.round(v), 0, 255).astype(np.uint8)
        tie = np.abs(v - np.floor(v) - 0.5) < 1e-9
        assert np.array_equal(got[~tie], ref[~tie]), (h, w, dh, dw)
        # at a tie either neighbour, depending on the last bit of each side's f64 sum
        lo = np.floor(v[tie]).astype(np.int64)
        assert np.all((got[tie] == lo) | (got[tie] == lo + 1)), (h, w, dh, dw)
        assert tie.mean() < 1e-2


def test_oracle_resize_identity_and_constant():
    rng = np.random.default_rng(1)
    img = rng.integers(0, 256, (33, 47, 3), dtype=np.uint8)
    assert np.array_equal(nn.resize_bilinear_u8(img, 47, 33), img)
    c = np.full((5, 9, 3), 200, np.uint8)
    assert np.all(nn.resize_bilinear_u8(c, 1008, 1008) == 200)


@pytest.mark.gpu
def test_resize_bilinear_u8_bit_exact(engine):
    import torch
    rng = np.random.default_rng(2)
    for (h, w), (dh, dw) in SIZES:
        img = rng.integers(0, 256, (2, h, w, 3), dtype=np.uint8)
        src = torch.from_numpy(img).cuda()
        out = torch.empty((2, dh, dw, 3), dtype=torch.uint8, device="cuda")
        engine.resize_bilinear_u8(src, out)
        engine.sync()
        got = out.cpu().numpy()
        for f in range(2):
            ref = nn.resize_bilinear_u8(img[f], dw, dh)
            assert np.array_equal(got[f], ref), ((h, w), (dh, dw), f, int(np.count_nonzero(got[f] != ref)))


@pytest.mark.gpu
def test_encode_image_any_size(engine, s3b, tmp_path):
    """Frames of another size are resized on the device: the encoder outputs equal those of
    the oracle-resized frames given at the model size; a native-size frame skips the resize."""
    import torch
    from sam3_b200 import synth
    cfg = synth.Sam2Config(img_size=256, embed=96, heads=1, stages=(1, 2, 2, 1), global_idx=(4,),
                           window_spec=(8, 4, 14, 7))
    path = str(tmp_path / "h.ggml")
    synth.write_sam2(path, cfg, seed=4, ftype=1)
    engine.load_model(path)
    rng = np.random.default_rng(3)
    for h, w in ((480, 640), (200, 131), (256, 256)):
        frames = rng.integers(0, 256, (2, h, w, 3), dtype=np.uint8)
        resized = np.stack([nn.resize_bilinear_u8(f, 256, 256) for f in frames])
        engine.encode_u8(resized)
        want = [[engine.output(f"neck_trk_{i}", f) for i in range(3)] for f in range(2)]
        engine.encode_image_u8(frames)
        got_host = [[engine.output(f"neck_trk_{i}", f) for i in range(3)] for f in range(2)]
        engine.encode_image_u8(torch.from_numpy(frames).cuda())
        got_dev = [[engine.output(f"neck_trk_{i}", f) for i in range(3)] for f in range(2)]
        for f in range(2):
            for i in range(3):
                assert np.array_equal(got_host[f][i], want[f][i]), (h, w, f, i)
                assert np.array_equal(got_dev[f][i], want[f][i]), (h, w, f, i)
    # the preprocessed frame itself: backbone input = oracle normalisation of the oracle resize
    assert np.array_equal(oh.preprocess_u8(resized)[0].shape, (3, 256, 256))
