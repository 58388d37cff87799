"""GEMMs on weights kept in q4_0 / q8_0 block form in device memory (option
"weights_quantised", s3b_op_gemm_q). Mode 2 (and s3b_op_gemm_q): the GEMM
dequantises each weight tile in shared memory; mode 1: one kernel dequantises
the layer's weight into an f16 staging buffer right before the f16 GEMM. The
dequantised values equal the load-time f16 dequantisation bit for bit and the
tensor-core work is the same, so outputs must EQUAL those of the f16 path on
the dequantised weights (same tile shapes: SM pairs), and stay within the
GEMM tolerance of an fp32 reference.

The quantised weights stand in for ggml_mul_mat on q4_0 / q8_0 tensors
(sam3.cpp:3738, 3792-3795, 4345, 4447-4450, 9250-9324)."""
import numpy as np
import pytest

from oracle import quant as oq
from oracle import vit as ov
from parity import assert_close

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _blocks(qtype, N, K, seed):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((N, K)) * 0.05).astype(np.float32)
    raw = oq.quantize(qtype, w)
    deq = oq.dequantize(qtype, raw, K)  # exact f32 values of the blocks
    return torch.from_numpy(raw).cuda(), torch.from_numpy(deq).cuda().half()


# (M, N, K, f32 in-place residual, act): QKV-like and fc1-like (16 epilogue warps), fc2-like (long K, 8 warps),
# K = 96 (half a 64-column stage, Hiera-T stage 0), N below one 256-column tile, M below one pair tile
CASES = [(5184 + 130, 3072, 1024, False, 0), (1000, 4736, 1024, False, 1), (777, 1024, 4736, True, 0),
         (300, 96, 96, True, 0), (4097, 288, 96, False, 2), (100, 256, 64, False, 3), (257, 512, 2048, True, 0)]


@pytest.mark.parametrize("qtype", [2, 8])
@pytest.mark.parametrize("M,N,K,resid,act", CASES)
def test_gemm_q_equals_f16_path(engine, qtype, M, N, K, resid, act):
    g = torch.Generator(device="cuda").manual_seed(M + N + K + qtype)
    A = (torch.randn(M, K, device="cuda", generator=g) * 0.5).half()
    raw, Bh = _blocks(qtype, N, K, M + K)
    bias = torch.randn(N, device="cuda", generator=g) * 0.1
    if resid:
        r0 = torch.randn(M, N, device="cuda", generator=g)
        got, want = r0.clone(), r0.clone()
    else:
        got = torch.empty(M, N, device="cuda", dtype=torch.float16)
        want = torch.empty_like(got)
    engine.set_option("gemm_pairs", 2)  # the quantised GEMM always runs 256-row tiles on SM pairs
    try:
        engine.gemm(A, Bh, want, bias=bias, act=act, resid=want if resid else None)
        engine.gemm_q(A, raw, qtype, N, got, bias=bias, act=act, resid=got if resid else None)
        engine.sync()
    finally:
        engine.set_option("gemm_pairs", 2)  # the default
    assert torch.equal(got, want), (got.float() - want.float()).abs().max().item()
    ref = A.float() @ Bh.float().T + bias
    if act == 1:
        ref = torch.nn.functional.gelu(ref)
    elif act == 2:
        ref = torch.nn.functional.gelu(ref, approximate="tanh")
    elif act == 3:
        ref = torch.relu(ref)
    if resid:
        ref = ref + r0
    err = (got.float() - ref).abs().max().item()
    assert err < 2e-3 * max(1.0, ref.abs().max().item()) + 1e-4 * K ** 0.5 + (0 if resid else 1e-2), err


def test_gemm_q_rejects_bad_shapes(engine, s3b):
    A = torch.zeros(128, 80, device="cuda", dtype=torch.float16)
    raw = torch.zeros(64 * 60, device="cuda", dtype=torch.uint8)
    out = torch.zeros(128, 64, device="cuda", dtype=torch.float32)
    with pytest.raises(s3b.S3BError):
        engine.gemm_q(A, raw, 2, 64, out)  # K = 80 is not a multiple of 32
    A = torch.zeros(128, 64, device="cuda", dtype=torch.float16)
    with pytest.raises(s3b.S3BError):
        engine.gemm_q(A, raw, 3, 64, out)  # q4_1 is dequantised at load, not in the GEMM


def _encode_both(engine, path, frames, names, modes=(0, 1, 2)):
    outs = []
    for wq in modes:
        engine.set_option("weights_quantised", wq)
        try:
            engine.load_model(path)
            info = engine.model_info()
            engine.encode_u8(frames)
            engine.sync()
            outs.append(({(n, f): engine.output(n, f) for n in names for f in range(len(frames))}, info))
        finally:
            engine.set_option("weights_quantised", 0)
    return outs


@pytest.mark.parametrize("qtype", [2, 8])
def test_vit_weights_quantised_equal_and_vs_oracle(engine, s3b, tmp_path, qtype):
    """SAM 3 ViT + SimpleFPN with block-form weights: identical outputs to the load-time dequantisation,
    less device memory, and the oracle's cosine bar."""
    from sam3_b200 import synth
    cfg = synth.Sam3Config(img_size=336, patch=14, embed=256, depth=3, heads=4, mlp_ratio_x1000=4625, window=8,
                           global_idx=(1,), neck_dim=64, neck_mid=128, visual_only=1)
    path = str(tmp_path / "tiny_q.ggml")
    T = synth.write_sam3(path, cfg, seed=3, ftype=1, qtype=qtype, quantize=s3b.quantize_rows, ln_random=True)
    frames = synth.frames_u8(2, cfg.img_size, base_seed=1000)
    names = ["vit_output"] + [f"neck_trk_{i}" for i in range(4)]
    (f16_out, f16_info), (q_out, q_info), (q2_out, q2_info) = _encode_both(engine, path, frames, names)
    for key in f16_out:
        assert np.array_equal(f16_out[key], q_out[key]), key
        assert np.array_equal(f16_out[key], q2_out[key]), key
    assert q_info["weights_mib"] < f16_info["weights_mib"], (q_info, f16_info)
    assert q2_info["weights_mib"] == q_info["weights_mib"]
    W = synth.stored_values(T, 1, qtype, oq.quantize, oq.dequantize)
    x, _ = ov.backbone(W, ov.preprocess_u8(frames), cfg)
    assert_close(q_out[("vit_output", 1)], x[1], 0.9999, 0.01, 0.05, "vit_output[1]")


@pytest.mark.parametrize("qtype", [2, 8])
def test_hiera_weights_quantised_equal(engine, s3b, tmp_path, qtype):
    """SAM 2.1 Hiera-T-like (K = 96 stage-0 GEMMs, half a stage of K) with block-form weights."""
    from sam3_b200 import synth
    cfg = synth.Sam2Config(img_size=256, embed=96, heads=1, stages=(1, 2, 3, 1), global_idx=(4,),
                           window_spec=(8, 4, 14, 7))
    path = str(tmp_path / "h_q.ggml")
    synth.write_sam2(path, cfg, seed=4, ftype=1, qtype=qtype, quantize=s3b.quantize_rows, ln_random=True)
    frames = synth.frames_u8(2, cfg.img_size, base_seed=31)
    names = [f"neck_trk_{i}" for i in range(3)]
    (f16_out, _), (q_out, _), (q2_out, _) = _encode_both(engine, path, frames, names)
    for key in f16_out:
        assert np.array_equal(f16_out[key], q_out[key]), key
        assert np.array_equal(f16_out[key], q2_out[key]), key


@pytest.mark.parametrize("qtype", [2, 8])
def test_mem_attn_weights_quantised_equal(engine, s3b, tmp_path, qtype):
    """Memory attention (self-attention q / k / v rows concatenated in block form) with block-form weights."""
    from sam3_b200 import synth
    from oracle import mem_attn as om
    cfg = synth.Sam3Config(img_size=336, patch=14, embed=128, depth=1, heads=2, window=8, global_idx=(),
                           neck_dim=256, neck_mid=128, with_mem_attn=True)
    path = str(tmp_path / "mem_q.ggml")
    synth.write_sam3(path, cfg, seed=9, ftype=1, qtype=qtype, quantize=s3b.quantize_rows, ln_random=True)
    rng = np.random.default_rng(5)
    feat, slots, ptrs = 16, 2, 4
    N = feat * feat
    curr = rng.standard_normal((N, 256), dtype=np.float32)
    M = slots * N + 4 * ptrs
    prompt = rng.standard_normal((M, 64), dtype=np.float32)
    ppos = rng.standard_normal((M, 64), dtype=np.float32)
    pos = om.src_pos(feat)
    outs = []
    for wq in (0, 1, 2):
        engine.set_option("weights_quantised", wq)
        try:
            engine.load_model(path)
            outs.append(engine.mem_attn(curr, pos, feat, prompt, ppos, 4 * ptrs).copy())
            # the second and third calls replay the captured graph (staging launches included)
            outs.append(engine.mem_attn(curr, pos, feat, prompt, ppos, 4 * ptrs).copy())
            outs.append(engine.mem_attn(curr, pos, feat, prompt, ppos, 4 * ptrs).copy())
        finally:
            engine.set_option("weights_quantised", 0)
    for o in outs[1:]:
        assert np.array_equal(outs[0], o)
