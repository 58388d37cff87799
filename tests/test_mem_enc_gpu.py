"""Memory encoder and object pointer on the GPU (s3b_mem_encode / s3b_obj_ptr).

The engine follows sam3.cpp's graph (GELU-tanh as ggml_gelu, convolution inputs rounded to f16 as
ggml's im2col does), so it is compared with the oracle in that form (oracle/mem_enc.py, gelu="tanh",
f16_inputs=True): cosine >= 0.9999 and max |err| <= 1e-2 of the largest value. Against the reference's
Python dump (erf GELU, f32 convolutions: tests/golden/mem_enc_golden.npz) the bound is the distance
between the two GELU forms, 1e-2 of the largest value. The object pointer is an f32 MLP (atol 1e-4).
Host and device entry points give the same bits.
"""
import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
import make_golden as mg  # noqa: E402

from oracle import mem_enc as me  # noqa: E402

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

GOLDEN = np.load(os.path.join(HERE, "golden", "mem_enc_golden.npz"))


def _cos(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-30))


def _sam3_file(tmp_path, seed):
    from sam3_b200 import ggml_io, synth
    cfg = synth.Sam3Config(img_size=1008, patch=14, embed=128, depth=1, heads=2, window=8, global_idx=(),
                           neck_dim=256, neck_mid=128)
    T = synth.sam3_tensors(cfg, seed=5)
    T.update(synth.mem_enc_tensors(seed))
    path = str(tmp_path / f"menc3_{seed}.ggml")
    synth.write_model(path, T, cfg.hparams(), ggml_io.MAGIC_SAM3, 3, 1)
    return path, synth.stored_values(synth.mem_enc_tensors(seed), 1, None)


@pytest.mark.parametrize("name,score", [("present", 2.5), ("absent", -1.5)])
def test_memory_encoder_full_size(tmp_path, engine, name, score):
    path, W = _sam3_file(tmp_path, mg.MEMENC_SEED)
    engine.load_model(path)
    pix, logits, token = mg.mem_enc_inputs()
    dev_score = torch.tensor([score], device="cuda")
    out = engine.mem_encode(72, torch.from_numpy(pix.reshape(-1, 256)).cuda(), torch.from_numpy(logits).cuda(),
                            dev_score)
    ptr = engine.obj_ptr(torch.from_numpy(token).cuda(), dev_score)
    engine.sync()
    got = out.cpu().numpy().reshape(72, 72, 64)
    ref = me.encode(W, pix, logits, score, 1008, gelu="tanh", f16_inputs=True)
    assert _cos(got, ref) >= 0.9999, _cos(got, ref)
    assert np.abs(got - ref).max() <= 1e-2 * np.abs(ref).max()
    # the reference's own (erf-GELU, f32) encoder: within the GELU forms' distance
    idx, gv = GOLDEN[f"{name}_output__idx"], GOLDEN[f"{name}_output__val"]
    assert np.abs(got.reshape(-1)[idx] - gv).max() <= 1e-2 * np.abs(gv).max()
    np.testing.assert_allclose(ptr.cpu().numpy(), GOLDEN[f"{name}_obj_ptr"], rtol=0, atol=1e-4)
    # host entry points: same bits
    host = engine.mem_encode(72, pix.reshape(-1, 256), logits, np.float32(score))
    assert np.array_equal(host, out.cpu().numpy())
    assert np.array_equal(engine.obj_ptr(token, np.float32(score)), ptr.cpu().numpy())


def test_memory_encoder_sam2_size(tmp_path, engine):
    # SAM 2.1 tracker size: 64^2 features, 256^2 mask logits, input 1024 (the second resize is 1024 -> 1024)
    # and sigmoid scale / bias from the file's hparams
    from sam3_b200 import ggml_io, synth
    cfg = synth.Sam2Config(img_size=1024, embed=96, heads=1, stages=(1, 2, 2, 1), global_idx=(4,),
                           window_spec=(8, 4, 14, 7))
    T = synth.sam2_tensors(cfg, seed=3)
    T.update(synth.mem_enc_tensors(8))
    hp = cfg.hparams()
    hp[-17], hp[-16] = 1500, -500  # sigmoid scale 15, bias -5
    path = str(tmp_path / "menc2.ggml")
    synth.write_model(path, T, hp, ggml_io.MAGIC_SAM2, 1, 1)
    engine.load_model(path)
    W = synth.stored_values(synth.mem_enc_tensors(8), 1, None)
    rng = np.random.default_rng(4)
    pix = rng.standard_normal((64, 64, 256), dtype=np.float32)
    logits = (rng.standard_normal((256, 256), dtype=np.float32) * 3).astype(np.float32)
    got = engine.mem_encode(64, pix.reshape(-1, 256), logits, None).reshape(64, 64, 64)
    ref = me.encode(W, pix, logits, 1.0, 1024, gelu="tanh", f16_inputs=True, scale=15.0, bias=-5.0)
    assert _cos(got, ref) >= 0.9999, _cos(got, ref)
    assert np.abs(got - ref).max() <= 1e-2 * np.abs(ref).max()


def test_obj_ptr_without_score_is_the_mlp(tmp_path, engine):
    path, W = _sam3_file(tmp_path, 12)
    engine.load_model(path)
    tok = np.random.default_rng(5).standard_normal(256).astype(np.float32)
    got = engine.obj_ptr(tok, None)
    np.testing.assert_allclose(got, me.obj_ptr(W, tok, 1.0), rtol=0, atol=1e-4)
    np.testing.assert_array_equal(engine.obj_ptr(tok, np.float32(0.0)), W["no_obj_ptr"].reshape(-1))
