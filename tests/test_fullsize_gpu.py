"""The engine at the configurations' full sizes against the oracle, through the C ABI.

- SAM 3 ViT-L + tracker neck with q4_0 weights, 8 frames in one encoder pass, weights in block
  form in HBM (the bench's default, weights_quantised = 1); frames 0 and 7 of the pass against the oracle.
- SAM 2.1 Hiera-L + FPN neck with q8_0 weights at 1024^2, 2 frames in one pass; every
  neck_trk_i against the oracle.

The oracle needs minutes per frame at these sizes, so its outputs come from committed fixtures
(tests/golden/make_oracle_fixtures.py: deterministic samples + statistics of every output). Tolerances as
the reference-pinned tests: cosine >= 0.999 on the samples, mean-abs <= 2% of the mean |value|, max-abs
<= 20% of the max |value| (the engine rounds GEMM / attention operands to f16 like ggml's CPU path)."""
import json
import os

import numpy as np
import pytest

from test_golden import check_samples, gold

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _fixture(name):
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", name)
    if not os.path.exists(path):
        pytest.skip(f"{name} not generated (tests/golden/make_oracle_fixtures.py)")
    g = gold(name)
    return g, json.loads(str(g["meta"]))


def test_vit_l_q4_0_batch8_vs_oracle(s3b, tmp_path):
    from sam3_b200 import synth
    g, meta = _fixture("fullsize_vit_l_q4_0.npz")
    path = str(tmp_path / "vit_l_q4_0.ggml")
    synth.write_sam3(path, synth.SAM3_VIT_L, seed=meta["weights_seed"], ftype=1, qtype=2,
                     quantize=s3b.quantize_rows)
    eng = s3b.Engine(0)
    try:
        eng.set_option("weights_quantised", 1)
        eng.set_option("frames_per_pass", 8)
        eng.load_model(path)
        frames = torch.from_numpy(synth.frames_u8(meta["frames_in_pass"], 1008, base_seed=meta["frame_seed"])).cuda()
        eng.encode_u8(frames)
        eng.sync()
        for f in meta["frames"]:
            print(check_samples(eng.output("vit_output", f), g, f"frame{f}_vit_output", 0.02, 0.2, 0.999))
            for i in range(4):
                print(check_samples(eng.output(f"neck_trk_{i}", f), g, f"frame{f}_neck_trk_{i}", 0.02, 0.2, 0.999))
    finally:
        eng.close()


def test_hiera_l_q8_0_fullsize_vs_oracle(s3b, tmp_path):
    from sam3_b200 import synth
    g, meta = _fixture("fullsize_hiera_l_q8_0.npz")
    path = str(tmp_path / "hiera_l_q8_0.ggml")
    synth.write_sam2(path, synth.HIERA_L, seed=meta["weights_seed"], ftype=1, qtype=8, quantize=s3b.quantize_rows)
    eng = s3b.Engine(0)
    try:
        eng.set_option("weights_quantised", 1)
        eng.load_model(path)
        frames = torch.from_numpy(synth.frames_u8(2, 1024, base_seed=meta["frame_seed"])).cuda()
        eng.encode_u8(frames)
        eng.sync()
        for f in meta["frames"]:
            for i in range(3):
                print(check_samples(eng.output(f"neck_trk_{i}", f), g, f"frame{f}_neck_trk_{i}", 0.02, 0.2, 0.999))
    finally:
        eng.close()
