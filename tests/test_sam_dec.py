"""SAM prompt encoder + mask decoder: the oracle (oracle/mask_decoder.py) against the reference's own
PyTorch decoder (dump_case() of tests/dump_phase6_reference.py, whose outputs are the committed fixture
tests/golden/sam_dec_golden.npz), and the host-side pieces of the C ABI that need no GPU (mask choice)."""
import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
import make_golden as mg  # noqa: E402  (seeded weights / features, no reference access)

from oracle import mask_decoder as md  # noqa: E402

GOLDEN = np.load(os.path.join(HERE, "golden", "sam_dec_golden.npz"))


@pytest.fixture(scope="module")
def inputs():
    return mg.sam_dec_weights(), mg.sam_dec_features()


@pytest.mark.parametrize("case", mg.SAMDEC_CASES, ids=[c[0] for c in mg.SAMDEC_CASES])
def test_oracle_decoder_matches_reference(inputs, case):
    W, (f0, f1, f2) = inputs
    name, pos, neg, box = case
    coords, labs = md.prompt_points(pos, neg, box)
    sparse = md.sparse_embeddings(W, coords, labs)
    np.testing.assert_allclose(sparse, GOLDEN[f"{name}_sparse"], rtol=0, atol=2e-6)
    taps = {}
    masks, iou, obj, tok = md.decode(W, f2, f0, f1, sparse, add_no_mem=True, taps=taps)
    np.testing.assert_allclose(iou, GOLDEN[f"{name}_iou"], rtol=0, atol=1e-6)
    np.testing.assert_allclose(obj, GOLDEN[f"{name}_obj_score"], rtol=0, atol=1e-6)
    np.testing.assert_allclose(tok, GOLDEN[f"{name}_sam_token"], rtol=0, atol=2e-5)
    np.testing.assert_allclose(taps["final_queries"], GOLDEN[f"{name}_final_queries"], rtol=0, atol=2e-5)
    for key, arr in (("masks", masks), ("upscaled", taps["upscaled"]), ("block1_keys", taps["block1_keys"])):
        idx, ref = GOLDEN[f"{name}_{key}__idx"], GOLDEN[f"{name}_{key}__val"]
        assert arr.size == int(np.prod(GOLDEN[f"{name}_{key}__shape"]))
        got = arr.reshape(-1)[idx]
        assert np.abs(got - ref).max() <= 1e-5 * max(1.0, np.abs(ref).max())


def test_best_mask_rule(s3b):
    # sam3_propagate_single: no multimask -> mask 0; multimask -> best IoU among 1..3, first on ties
    assert s3b.sam_best_mask([0.9, 0.1, 0.2, 0.3], multimask=False) == 0
    assert s3b.sam_best_mask([0.9, 0.1, 0.2, 0.3], multimask=True) == 3
    assert s3b.sam_best_mask([0.9, 0.5, 0.5, 0.1], multimask=True) == 1
    assert s3b.sam_best_mask([0.0, 0.2, 0.7, 0.7], multimask=True) == 2
