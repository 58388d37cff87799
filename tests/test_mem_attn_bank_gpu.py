"""Memory attention from a device-resident memory bank (s3b_mem_attn_bank / s3b_op_build_prompt).

The device prompt build must give the arrays of sam3_build_prompt_and_pos (sam3.cpp:9123-9209) bit for bit:
slot features, slot PE + temporal PE row (maskmem_tpos_enc[num_maskmem - tpos - 1] for 0 <= tpos <
num_maskmem), then each kept object pointer split into 4 tokens of 64 with the 256 -> 64 projection of the
1-D sine PE of distance / 15 (pointers with a negative distance skipped). Memory attention run from the bank
must then EQUAL s3b_mem_attn on those arrays, and at the configs[4] shape (feat 64, 7 slots + 16 pointers,
M = 28,736 memory tokens) it must agree with the oracle's memory attention.
"""
import numpy as np
import pytest

from oracle import mem_attn as om
from oracle import nn
from parity import assert_close

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _model(s3b, tmp_path, seed=9):
    from sam3_b200 import synth
    cfg = synth.Sam3Config(img_size=336, patch=14, embed=128, depth=1, heads=2, window=8, global_idx=(),
                           neck_dim=256, neck_mid=128, with_mem_attn=True)
    path = str(tmp_path / f"mem_bank_{seed}.ggml")
    T = synth.write_sam3(path, cfg, seed=seed, ftype=1, ln_random=True)
    W = synth.stored_values(T, 1, None)
    return cfg, path, W


def _bank(feat, n_slots, n_ptrs, seed, with_pes):
    g = torch.Generator(device="cuda").manual_seed(seed)
    N = feat * feat
    feats = [torch.randn(N, 64, device="cuda", generator=g) for _ in range(n_slots)]
    pes = [torch.randn(N, 64, device="cuda", generator=g) * 0.5 for _ in range(n_slots)] if with_pes else None
    ptrs = torch.randn(n_ptrs, 256, device="cuda", generator=g) if n_ptrs else None
    return feats, pes, ptrs


def _oracle_prompt(W, cfg, feat, feats, pes, slot_tpos, ptrs, ptr_tpos):
    pe_default = nn.sine_pe_2d(feat, feat, 64).reshape(feat * feat, 64)
    slot_pes = [p.cpu().numpy() for p in pes] if pes is not None else [pe_default] * len(feats)
    return om.build_prompt([f.cpu().numpy() for f in feats], slot_pes, slot_tpos,
                           W["mem_enc.tpos_enc"].reshape(cfg.num_maskmem, 64),
                           [] if ptrs is None else list(ptrs.cpu().numpy()), list(ptr_tpos),
                           W["obj_ptr_tpos_proj.weight"], W["obj_ptr_tpos_proj.bias"], cfg.num_maskmem)


# (feat, slots, spatial tpos, pointer distances, slot PEs given): conditioning frame (tpos 0), the usual
# n_sel - s positions, a tpos beyond the table (no temporal row), skipped pointers, no pointers, no slots
CASES = [
    (16, [0, 3, 2, 1], [1, 2, 3, 5, 16], True),
    (8, [7, 6, 5, 4, 3, 2, 1], [1, -1, 4, 2, -3, 15, 40, 1, 9, 10, 11, 12, 13, 14, 15, 16], False),
    (12, [9, 1], [], True),
    (16, [], [3, 1, 2], False),
]


@pytest.mark.parametrize("feat,slot_tpos,ptr_tpos,with_pes", CASES)
def test_build_prompt_bit_exact(engine, s3b, tmp_path, feat, slot_tpos, ptr_tpos, with_pes):
    cfg, path, W = _model(s3b, tmp_path)
    engine.load_model(path)
    feats, pes, ptrs = _bank(feat, len(slot_tpos), len(ptr_tpos), feat + len(ptr_tpos), with_pes)
    prompt, pos, n_ptr = engine.build_prompt(feat, feats, slot_tpos, ptrs, ptr_tpos, slot_pes=pes)
    engine.sync()
    ref_p, ref_pos, ref_n = _oracle_prompt(W, cfg, feat, feats, pes, slot_tpos, ptrs, ptr_tpos)
    assert n_ptr == ref_n
    assert prompt.shape == ref_p.shape
    assert np.array_equal(prompt.cpu().numpy(), ref_p)
    assert np.array_equal(pos.cpu().numpy(), ref_pos)


def test_mem_attn_bank_equals_host_prompt_path(engine, s3b, tmp_path):
    cfg, path, W = _model(s3b, tmp_path, seed=10)
    engine.load_model(path)
    feat, slot_tpos, ptr_tpos = 16, [0, 2, 1], [1, 2, -1, 7]
    feats, pes, ptrs = _bank(feat, 3, 4, 77, with_pes=False)
    g = torch.Generator(device="cuda").manual_seed(78)
    curr = torch.randn(feat * feat, 256, device="cuda", generator=g)
    src_pos = torch.from_numpy(nn.sine_pe_2d(feat, feat, 256).reshape(-1, 256)).cuda()
    ref_p, ref_pos, n_ptr = _oracle_prompt(W, cfg, feat, feats, None, slot_tpos, ptrs, ptr_tpos)
    want = engine.mem_attn(curr, src_pos, feat, torch.from_numpy(ref_p).cuda(), torch.from_numpy(ref_pos).cuda(),
                           n_ptr)
    # src_pos given, then NULL (the engine's own cached sine PE): both equal the host-prompt path; the third
    # call replays the layers' CUDA graph
    for sp in (src_pos, None, None):
        got = engine.mem_attn_bank(curr, feat, feats, slot_tpos, ptrs, ptr_tpos, src_pos=sp)
        engine.sync()
        assert torch.equal(got, want)


def test_mem_attn_bank_rejects_bad_banks(engine, s3b, tmp_path):
    cfg, path, W = _model(s3b, tmp_path, seed=11)
    engine.load_model(path)
    feats, _, ptrs = _bank(8, 17, 2, 5, False)
    curr = torch.zeros(64, 256, device="cuda")
    with pytest.raises(s3b.S3BError):
        engine.mem_attn_bank(curr, 8, feats, list(range(17)))  # 17 slots > 16
    with pytest.raises(s3b.S3BError):
        engine.mem_attn_bank(curr, 8, [], [], ptrs, [-1, -2])  # every pointer skipped and no slot: no memory


def test_mem_attn_bank_configs4_shape_vs_oracle(engine, s3b, tmp_path):
    """configs[4]'s memory attention shape: 64 x 64 current tokens, 7 memory slots of 64 x 64 tokens and 16
    object pointers (M = 7 * 4096 + 64 = 28,736), 4 layers, d = 256, against the oracle."""
    from sam3_b200 import synth
    cfg = synth.Sam3Config(img_size=336, patch=14, embed=128, depth=1, heads=2, window=8, global_idx=(),
                           neck_dim=256, neck_mid=128, with_mem_attn=True)
    path = str(tmp_path / "mem_c4.ggml")
    T = synth.write_sam3(path, cfg, seed=21, ftype=1, qtype=8, quantize=s3b.quantize_rows, ln_random=True)
    from oracle import quant as oq
    W = synth.stored_values(T, 1, 8, oq.quantize, oq.dequantize)
    engine.load_model(path)
    feat = 64
    slot_tpos = [7 - s for s in range(7)]
    ptr_tpos = list(range(1, 17))
    feats, _, ptrs = _bank(feat, 7, 16, 404, with_pes=False)
    g = torch.Generator(device="cuda").manual_seed(405)
    curr = torch.randn(feat * feat, 256, device="cuda", generator=g)
    got = engine.mem_attn_bank(curr, feat, feats, slot_tpos, ptrs, ptr_tpos)
    engine.sync()
    prompt, ppos, n_ptr = _oracle_prompt(W, cfg, feat, feats, None, slot_tpos, ptrs, ptr_tpos)
    assert prompt.shape[0] == 28736 and n_ptr == 64
    ref = om.mem_attn(W, curr.cpu().numpy(), om.src_pos(feat), feat, prompt, ppos, n_ptr)
    assert_close(got.cpu().numpy(), ref, 0.9999, 0.01, 0.05, "mem_attn configs[4] shape")
