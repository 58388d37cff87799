"""Memory encoder + object-pointer MLP: the oracle (oracle/mem_enc.py) against the reference's own PyTorch
code (run_memory_encoder() / run_obj_ptr() of tests/dump_phase7_reference.py, committed as
tests/golden/mem_enc_golden.npz), with the oracle in the Python reference's form (erf GELU, f32 conv
inputs); plus the mask resize restated from sam3_bilinear_interpolate against torch's bilinear
interpolation (align_corners=False), which it follows."""
import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
import make_golden as mg  # noqa: E402

from oracle import mem_enc as me  # noqa: E402

GOLDEN = np.load(os.path.join(HERE, "golden", "mem_enc_golden.npz"))


@pytest.fixture(scope="module")
def inputs():
    return mg.mem_enc_weights(), mg.mem_enc_inputs()


@pytest.mark.parametrize("name,score", [("present", 2.5), ("absent", -1.5)])
def test_oracle_memory_encoder_matches_reference(inputs, name, score):
    W, (pix, logits, token) = inputs
    taps = {}
    taps["output"] = me.encode(W, pix, logits, score, 1008, gelu="erf", f16_inputs=False, taps=taps)
    for key in ("mask_downsampled", "fuser0", "fuser1", "output"):
        idx, ref = GOLDEN[f"{name}_{key}__idx"], GOLDEN[f"{name}_{key}__val"]
        got = taps[key].reshape(-1)[idx]
        assert np.abs(got - ref).max() <= 3e-4 * np.abs(ref).max(), key
    np.testing.assert_allclose(me.obj_ptr(W, token, score), GOLDEN[f"{name}_obj_ptr"], rtol=0, atol=2e-6)


def test_bilinear_follows_torch():
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(3)
    src = rng.standard_normal((37, 53)).astype(np.float32)
    for dh, dw in ((101, 80), (20, 30), (37, 53)):
        got = me.bilinear(src, dw, dh)
        ref = torch.nn.functional.interpolate(torch.from_numpy(src)[None, None], size=(dh, dw), mode="bilinear",
                                              align_corners=False)[0, 0].numpy()
        np.testing.assert_allclose(got, ref, rtol=0, atol=3e-5)
