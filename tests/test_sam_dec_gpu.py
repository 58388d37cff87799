"""SAM mask decoder on the GPU (s3b_sam_decode) against the reference and the oracle.

- At the SAM 3 size (72^2 image tokens, 288^2 masks) the engine's masks, IoU, object score and SAM
  token are compared with the outputs of the reference's own PyTorch decoder (dump_case() of
  tests/dump_phase6_reference.py, committed as tests/golden/sam_dec_golden.npz) on the same seeded
  weights, features and prompts, with the prompt tokens built by s3b_sam_prompt_tokens.
- At other sizes (the Hiera tracker's 64^2, a small 16^2) and in the tracker's form (memory-attention
  output as the image features, the single not_a_point token) it is compared with the oracle.
- Host and device entry points give the same bits; the dense PE matches the oracle.

Tolerances: the image-side projections take f16 operands (the reference's ggml CPU mul_mat rounds its
activations to f16 too), so the checks are cosine >= 0.9999 and max |err| <= 2e-2 of the largest
reference value for the masks, 2e-3 absolute for IoU / object score, cosine >= 0.9999 for tokens.
"""
import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
import make_golden as mg  # noqa: E402

from oracle import mask_decoder as md  # noqa: E402

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

GOLDEN = np.load(os.path.join(HERE, "golden", "sam_dec_golden.npz"))


def _cos(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-30))


def _model_file(tmp_path, dec_seed=mg.SAMDEC_SEED, qtype=None, s3b=None):
    """A small SAM 3 encoder file carrying the seeded decoder tensors (the decoder does not depend on
    the encoder's size)."""
    from sam3_b200 import ggml_io, synth
    cfg = synth.Sam3Config(img_size=1008 if dec_seed == mg.SAMDEC_SEED else 336, patch=14, embed=128, depth=1,
                           heads=2, window=8, global_idx=(), neck_dim=256, neck_mid=128)
    T = synth.sam3_tensors(cfg, seed=5)
    T.update(synth.sam_dec_tensors(dec_seed))
    path = str(tmp_path / f"dec_{dec_seed}_{qtype}.ggml")
    synth.write_model(path, T, cfg.hparams(), ggml_io.MAGIC_SAM3, 3, 1, qtype, s3b.quantize_rows if qtype else None)
    W = synth.stored_values({k: v for k, v in T.items() if k.startswith(("sam_", "no_mem"))}, 1, qtype,
                            s3b.quantize_rows if qtype else None, s3b.dequantize_rows if qtype else None)
    return path, W


@pytest.fixture(scope="module")
def golden_setup(tmp_path_factory, s3b):
    import torch
    e = s3b.Engine(0)
    e.set_stream(torch.cuda.current_stream().cuda_stream)
    path, W = _model_file(tmp_path_factory.mktemp("dec"), s3b=s3b)
    e.load_model(path)
    feats = [torch.from_numpy(f.reshape(-1, 256)).cuda() for f in mg.sam_dec_features()]
    yield e, W, feats
    e.set_stream(None)
    e.close()


@pytest.mark.parametrize("case", mg.SAMDEC_CASES, ids=[c[0] for c in mg.SAMDEC_CASES])
def test_decoder_matches_reference_at_sam3_size(golden_setup, case):
    e, W, (f0, f1, f2) = golden_setup
    name, pos, neg, box = case
    sparse = e.sam_prompt_tokens(box=box, pos_points=pos, neg_points=neg, orig_size=(1008, 1008))
    np.testing.assert_allclose(sparse, GOLDEN[f"{name}_sparse"], rtol=0, atol=2e-6)
    masks, iou, obj, toks = e.sam_decode(72, f2, f0, f1, torch.from_numpy(sparse).cuda(), add_no_mem=True)
    torch.cuda.synchronize()
    m = masks.cpu().numpy().reshape(-1)
    idx, ref = GOLDEN[f"{name}_masks__idx"], GOLDEN[f"{name}_masks__val"]
    got = m[idx]
    assert _cos(got, ref) >= 0.9999, _cos(got, ref)
    assert np.abs(got - ref).max() <= 2e-2 * np.abs(ref).max()
    st = GOLDEN[f"{name}_masks__stats"]
    assert abs(m.mean() - st[0]) <= 1e-3 * st[2] + 1e-6
    np.testing.assert_allclose(iou.cpu().numpy(), GOLDEN[f"{name}_iou"], rtol=0, atol=2e-3)
    np.testing.assert_allclose(obj.cpu().numpy(), GOLDEN[f"{name}_obj_score"], rtol=0, atol=2e-3)
    assert _cos(toks.cpu().numpy()[0], GOLDEN[f"{name}_sam_token"]) >= 0.9999
    assert _cos(toks.cpu().numpy(), GOLDEN[f"{name}_mask_tokens"]) >= 0.9999


@pytest.mark.parametrize("H,prompt", [(16, "points"), (64, "tracker"), (32, "box")])
def test_decoder_matches_oracle(tmp_path, s3b, engine, H, prompt):
    path, W = _model_file(tmp_path, dec_seed=17 + H, s3b=s3b)
    engine.load_model(path)
    rng = np.random.default_rng(H)
    f0, f1, f2 = (rng.standard_normal((s * s, 256), dtype=np.float32) for s in (4 * H, 2 * H, H))
    sparse = None
    add_no_mem = prompt != "tracker"
    if prompt == "points":
        sparse = engine.sam_prompt_tokens(pos_points=[(100.0, 120.0), (10.0, 300.0)], neg_points=[(200.0, 50.0)],
                                          orig_size=(480, 640))
        coords, labs = md.prompt_points([(100.0, 120.0), (10.0, 300.0)], [(200.0, 50.0)])
        ref_sparse = md.sparse_embeddings(W, coords, labs, input_size=336, orig_w=480, orig_h=640)
        np.testing.assert_allclose(sparse, ref_sparse, rtol=0, atol=2e-6)
    elif prompt == "box":
        sparse = engine.sam_prompt_tokens(box=(20.0, 30.0, 200.0, 310.0), pos_points=[(50.0, 60.0)])
        coords, labs = md.prompt_points([(50.0, 60.0)], [], (20.0, 30.0, 200.0, 310.0))
        ref_sparse = md.sparse_embeddings(W, coords, labs, input_size=336)
        np.testing.assert_allclose(sparse, ref_sparse, rtol=0, atol=2e-6)
    ref_in = sparse if sparse is not None else W["sam_pe.not_a_point_embed.weight"].reshape(1, 256)
    rm, ri, ro, rt = md.decode(W, f2.reshape(H, H, 256), f0.reshape(4 * H, 4 * H, 256), f1.reshape(2 * H, 2 * H, 256),
                               ref_in, add_no_mem=add_no_mem)
    dev = [torch.from_numpy(x).cuda() for x in (f2, f0, f1)]
    sp = None if sparse is None else torch.from_numpy(sparse).cuda()
    masks, iou, obj, toks = engine.sam_decode(H, dev[0], dev[1], dev[2], sp, add_no_mem=add_no_mem)
    engine.sync()
    got = masks.cpu().numpy()
    assert got.shape == rm.shape
    assert _cos(got, rm) >= 0.9999, _cos(got, rm)
    assert np.abs(got - rm).max() <= 2e-2 * np.abs(rm).max()
    np.testing.assert_allclose(iou.cpu().numpy(), ri, rtol=0, atol=2e-3)
    np.testing.assert_allclose(obj.cpu().numpy(), ro, rtol=0, atol=2e-3)
    assert _cos(toks.cpu().numpy()[0], rt) >= 0.9999
    # the host entry point gives the same bits as the device one
    hm, hi, ho, ht = engine.sam_decode(H, f2, f0, f1, sparse, add_no_mem=add_no_mem)
    assert np.array_equal(hm, got)
    assert np.array_equal(hi, iou.cpu().numpy()) and np.array_equal(ho, obj.cpu().numpy())
    assert np.array_equal(ht, toks.cpu().numpy())


def test_dense_pe_matches_oracle(tmp_path, s3b, engine):
    path, W = _model_file(tmp_path, dec_seed=3, s3b=s3b)
    engine.load_model(path)
    for H in (16, 72):
        got = engine.sam_dense_pe(H)
        ref = md.dense_pe(W, H).reshape(H * H, 256)
        np.testing.assert_allclose(got, ref, rtol=0, atol=2e-5)


def test_decoder_rejects_bad_arguments(tmp_path, s3b, engine):
    path, W = _model_file(tmp_path, dec_seed=4, s3b=s3b)
    engine.load_model(path)
    H = 8
    f = [torch.zeros(s * s, 256, device="cuda") for s in (4 * H, 2 * H, H)]
    too_many = torch.zeros(27, 256, device="cuda")
    with pytest.raises(s3b.S3BError):
        engine.sam_decode(H, f[2], f[0], f[1], too_many)
    # the context stays usable
    engine.sam_decode(H, f[2], f[0], f[1], None)
    engine.sync()
