"""Pins the CPU oracle to the reference's own PyTorch forward (fixtures made by
tests/golden/make_golden.py from the reference's tests/dump_vit_reference.py
and tests/dump_phase7_reference.py on seeded synthetic weights)."""
import json
import os

import numpy as np
import pytest

from oracle import mem_attn as om
from oracle import vit as ov

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = os.path.join(HERE, "golden")


def gold(name):
    return np.load(os.path.join(GOLD, name))


def check_samples(arr, g, key, rtol_mean, rtol_max, cos_min=0.99999):
    shape = tuple(g[key + "__shape"])
    assert tuple(arr.shape) == shape, (arr.shape, shape)
    got = np.ascontiguousarray(arr, np.float32).ravel()[g[key + "__idx"]]
    ref = g[key + "__val"]
    d = np.abs(got.astype(np.float64) - ref)
    cos = float(np.dot(got, ref) / (np.linalg.norm(got) * np.linalg.norm(ref)))
    msg = f"{key}: max {d.max():.3e} mean {d.mean():.3e} ref mean {np.abs(ref).mean():.3e} cos {cos:.7f}"
    assert cos >= cos_min, msg
    assert d.mean() <= rtol_mean * np.abs(ref).mean(), msg
    assert d.max() <= rtol_max * np.abs(ref).max(), msg
    return msg


def test_oracle_preprocess_matches_reference(s3b):
    from sam3_b200 import synth
    g = gold("vit_golden.npz")
    meta = json.loads(str(g["meta"]))
    frame = synth.frames_u8(1, 1008, base_seed=meta["frame_seed"])
    check_samples(ov.preprocess_u8(frame)[0], g, "preprocessed", 1e-7, 1e-6, 0.9999999)


def test_oracle_vit_block0_matches_reference(s3b):
    """prefix (patch embed, tiled pos, ln_pre) + windowed block 0 vs the reference's PyTorch dump."""
    from sam3_b200 import synth
    g = gold("vit_golden.npz")
    meta = json.loads(str(g["meta"]))
    cfg = synth.Sam3Config(depth=1, global_idx=())  # same RNG stream for prefix + block 0
    W = synth.stored_values(synth.sam3_tensors(cfg, seed=meta["weights_seed"], ln_random=True), 1, None)
    chw = ov.preprocess_u8(synth.frames_u8(1, 1008, base_seed=meta["frame_seed"]))
    x = ov.prefix(W, chw, cfg)
    print(check_samples(x[0], g, "after_ln_pre", 1e-5, 1e-4))
    x = ov.block(W, x, 0, cfg)
    print(check_samples(x[0], g, "block_0_out", 1e-5, 1e-4))


@pytest.mark.skipif(os.environ.get("S3B_SLOW_TESTS") != "1", reason="full-size oracle forward (~4 min); S3B_SLOW_TESTS=1")
def test_oracle_full_vit_and_neck_match_reference(s3b):
    from sam3_b200 import synth
    g = gold("vit_golden.npz")
    meta = json.loads(str(g["meta"]))
    cfg = synth.SAM3_VIT_L
    W = synth.stored_values(synth.sam3_tensors(cfg, seed=meta["weights_seed"], ln_random=True), 1, None)
    chw = ov.preprocess_u8(synth.frames_u8(1, 1008, base_seed=meta["frame_seed"]))
    x, taps = ov.backbone(W, chw, cfg, taps=(0, 7))
    print(check_samples(taps[7][0], g, "block_7_out", 1e-4, 1e-3))
    print(check_samples(x[0], g, "vit_final", 1e-4, 1e-3))
    outs = ov.neck(W, x)
    for i in range(4):
        print(check_samples(outs[i][0], g, f"neck_det_{i}", 1e-4, 1e-3))


def test_oracle_mem_attn_matches_reference(s3b):
    """The oracle's memory attention vs run_memory_attention() of the reference's phase-7 dump code."""
    from sam3_b200 import synth
    g = gold("mem_attn_golden.npz")
    meta = json.loads(str(g["meta"]))
    cfg = synth.Sam3Config(depth=1, global_idx=(), with_mem_attn=True)
    T = synth.sam3_tensors(cfg, seed=meta["weights_seed"], ln_random=True)
    W = synth.stored_values({k: v for k, v in T.items() if k.startswith("mem_attn.")}, 1, None)
    curr, prompt, prompt_pos, n_ptr = om.golden_inputs(meta)
    taps = {}
    out = om.mem_attn(W, curr, om.src_pos(meta["feat"]), meta["feat"], prompt, prompt_pos, n_ptr, taps=taps)
    print(check_samples(taps["input"], g, "input", 1e-6, 1e-5))
    print(check_samples(taps["layer0_after_sa"], g, "layer0_after_sa", 1e-5, 1e-4))
    print(check_samples(taps["layer0_after_ca"], g, "layer0_after_ca", 1e-5, 1e-4))
    print(check_samples(taps["layer0_after_ffn"], g, "layer0_after_ffn", 1e-5, 1e-4))
    print(check_samples(out, g, "output", 1e-5, 1e-4))
