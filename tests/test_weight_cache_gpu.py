"""Persistent device-weight cache (s3b_load_model_cached).

A load through the cache builds the model from the file and writes the cache; the next load copies the
cached device form back with no conversion. The two models must give the same bits on the encoder and
the tracker, for SAM 3 (q4_0 in block form) and SAM 2 (q8_0 dequantised at load); a changed source file,
another weights_quantised option or a damaged cache must fall back to the file (and rewrite the cache)."""
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _write(tmp_path, s3b, sam2):
    from sam3_b200 import ggml_io, synth
    if sam2:
        cfg = synth.Sam2Config(img_size=256, embed=96, heads=1, stages=(1, 2, 2, 1), global_idx=(4,),
                               window_spec=(8, 4, 14, 7), with_mem_attn=True, with_sam_dec=True)
        T = synth.sam2_tensors(cfg, seed=13, ln_random=True)
        magic, ver, q = ggml_io.MAGIC_SAM2, 1, 8
    else:
        cfg = synth.Sam3Config(img_size=224, patch=14, embed=128, depth=2, heads=2, window=8, global_idx=(1,),
                               neck_dim=256, neck_mid=128, with_mem_attn=True, with_sam_dec=True)
        T = synth.sam3_tensors(cfg, seed=13, ln_random=True)
        magic, ver, q = ggml_io.MAGIC_SAM3, 3, 2
    T.update(synth.mem_enc_tensors(14))
    path = str(tmp_path / f"cache_src_{int(sam2)}.ggml")
    synth.write_model(path, T, cfg.hparams(), magic, ver, 1, q, s3b.quantize_rows)
    return cfg, path


def _run(e, cfg, frames):
    e.encode_u8(frames)
    outs = {n: e.output(n, 0) for n in ("neck_trk_0", "neck_trk_1", "neck_trk_2")}
    H = int(round(outs["neck_trk_2"].size / 256) ** 0.5)
    t = [torch.from_numpy(outs[n].reshape(-1, 256)).cuda() for n in ("neck_trk_0", "neck_trk_1", "neck_trk_2")]
    g = torch.Generator(device="cuda").manual_seed(3)
    bank = [torch.randn(H * H, 64, device="cuda", generator=g) for _ in range(2)]
    ptrs = torch.randn(2, 256, device="cuda", generator=g)
    step = e.track_step(H, t[0], t[1], t[2], bank, [0, 1], ptrs, [1, 2])
    e.sync()
    outs.update({k: v.cpu().numpy() for k, v in step.items()})
    return outs


@pytest.mark.parametrize("sam2,wq", [(False, 1), (True, 0)], ids=["sam3_q4_0_blockform", "sam2_q8_0_f16"])
def test_cached_model_equals_file_model(tmp_path, s3b, sam2, wq):
    from sam3_b200 import synth
    cfg, path = _write(tmp_path, s3b, sam2)
    cache = str(tmp_path / "weights.s3bc")
    frames = synth.frames_u8(1, cfg.img_size, base_seed=77)
    engines = []
    try:
        for expect_hit in (False, True):
            e = s3b.Engine(0)
            engines.append(e)
            e.set_option("weights_quantised", wq)
            assert e.load_model_cached(path, cache) is expect_hit
            assert os.path.exists(cache)
        a, b = (_run(e, cfg, frames) for e in engines)
        assert engines[0].model_info() == engines[1].model_info()
        for k in a:
            assert np.array_equal(a[k], b[k]), k
    finally:
        for e in engines:
            e.close()


def test_cache_invalidation(tmp_path, s3b):
    cfg, path = _write(tmp_path, s3b, False)
    cache = str(tmp_path / "weights.s3bc")
    e = s3b.Engine(0)
    try:
        assert e.load_model_cached(path, cache) is False
        assert e.load_model_cached(path, cache) is True
        # another weights_quantised option shapes another device form
        e.set_option("weights_quantised", 1)
        assert e.load_model_cached(path, cache) is False
        assert e.load_model_cached(path, cache) is True
        # the source file changed (modification time)
        st = os.stat(path)
        os.utime(path, ns=(st.st_atime_ns, st.st_mtime_ns + 1_000_000_000))
        assert e.load_model_cached(path, cache) is False
        assert e.load_model_cached(path, cache) is True
        # a damaged (truncated) cache falls back to the file and is rewritten
        with open(cache, "r+b") as f:
            f.truncate(os.path.getsize(cache) // 2)
        assert e.load_model_cached(path, cache) is False
        assert e.load_model_cached(path, cache) is True
        # a missing model file is an error
        with pytest.raises(s3b.S3BError):
            e.load_model_cached(str(tmp_path / "missing.ggml"), cache)
    finally:
        e.close()
