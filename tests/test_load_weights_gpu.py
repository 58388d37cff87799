"""s3b_load_weights: the weights handed over as the caller's host tensors (the tensors sam3.cpp holds after
sam3_load_tensors, sam3.cpp:3091-3194) instead of a second parse of the .ggml file. It must give the same
device model as s3b_load_model on the file: identical encoder outputs (bit for bit), for SAM 3 with q4_0
weights and SAM 2 with f16 weights, and reject malformed descriptors."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _file_tensors(path, n_hparams):
    from sam3_b200 import ggml_io
    magic, version, ftype, hp, recs = ggml_io.read(path, n_hparams)
    tensors = [(r.name, r.dtype, r.shape, r.data) for r in recs.values()]
    return magic == ggml_io.MAGIC_SAM2, hp, ftype, tensors


@pytest.mark.parametrize("kind", ["sam3_q4_0", "sam2_f16"])
def test_load_weights_equals_load_model(s3b, tmp_path, kind):
    from sam3_b200 import synth
    if kind == "sam3_q4_0":
        cfg = synth.Sam3Config(img_size=336, patch=14, embed=256, depth=2, heads=4, window=8, global_idx=(1,),
                               neck_dim=64, neck_mid=128, with_mem_attn=True)
        path = str(tmp_path / "w.ggml")
        synth.write_sam3(path, cfg, seed=5, ftype=1, qtype=2, quantize=s3b.quantize_rows)
        names = ["vit_output"] + [f"neck_trk_{i}" for i in range(4)]
    else:
        cfg = synth.Sam2Config(img_size=256, embed=96, heads=1, stages=(1, 2, 2, 1), global_idx=(4,),
                               window_spec=(8, 4, 14, 7))
        path = str(tmp_path / "w.ggml")
        synth.write_sam2(path, cfg, seed=6, ftype=1)
        names = [f"neck_trk_{i}" for i in range(3)]
    is_sam2, hp, ftype, tensors = _file_tensors(path, len(cfg.hparams()))
    frames = synth.frames_u8(2, cfg.img_size, base_seed=40)
    outs = []
    for mode in ("file", "descs"):
        eng = s3b.Engine(0)
        try:
            if mode == "file":
                eng.load_model(path)
            else:
                eng.load_weights(int(is_sam2), hp, ftype, tensors)
            info = eng.model_info()
            eng.encode_u8(frames)
            eng.sync()
            outs.append(({(n, f): eng.output(n, f) for n in names for f in range(2)}, info))
        finally:
            eng.close()
    (a, ia), (b, ib) = outs
    assert ia == ib
    for k in a:
        assert np.array_equal(a[k], b[k]), k


def test_load_weights_rejects_bad_descriptors(s3b, tmp_path, engine):
    from sam3_b200 import synth
    cfg = synth.Sam3Config(img_size=336, patch=14, embed=256, depth=1, heads=4, window=8, global_idx=(),
                           neck_dim=64, neck_mid=128)
    path = str(tmp_path / "w.ggml")
    synth.write_sam3(path, cfg, seed=5, ftype=1)
    is_sam2, hp, ftype, tensors = _file_tensors(path, len(cfg.hparams()))
    with pytest.raises(s3b.S3BError):
        engine.load_weights(0, hp[:-3], ftype, tensors)  # truncated hparams
    with pytest.raises(s3b.S3BError):
        engine.load_weights(0, hp + [0], ftype, tensors)  # one value too many
    bad = list(tensors)
    name, dtype, shape, data = bad[0]
    bad[0] = (name, 7, shape, data)  # unknown dtype
    with pytest.raises(s3b.S3BError):
        engine.load_weights(0, hp, ftype, bad)
