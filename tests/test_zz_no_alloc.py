"""s3b_conv3x3_noalloc: the 3x3 convolution entry point for callers that
cannot allocate device memory (their GPU memory is pre-sized and owned by
another allocator, their CUDA context forbids cudaMalloc, or they run on a
real-time thread where cudaMalloc would synchronise the device).

It must give the same result as s3b_op_conv3x3 (which takes its workspace
from an s3b_ctx) on two calls in a row — the second call reuses the shared
static scratch left over by the first — and reject sizes beyond its fixed
scratch. This file is collected last on purpose."""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

SCRATCH_BYTES = 32 * 1024 * 1024


def _noalloc(s3b, x, w, bias, out, stream=None):
    B, H, W, C = x.shape
    Cout = w.shape[0]
    stream = (stream or torch.cuda.current_stream()).cuda_stream
    return s3b.lib().s3b_conv3x3_noalloc(x.data_ptr(), B, H, W, C, w.data_ptr(),
                                         bias.data_ptr() if bias is not None else None, out.data_ptr(), Cout,
                                         ctypes.c_void_p(stream))


def _case(shape, cout, seed, device="cuda"):
    g = torch.Generator(device=device).manual_seed(seed)
    B, H, W, C = shape
    x = torch.randn(B, H, W, C, device=device, generator=g).half()
    w = (torch.randn(cout, 3, 3, C, device=device, generator=g) * 0.05).half()
    bias = torch.randn(cout, device=device, generator=g) * 0.1
    return x, w, bias


def _status(s3b):
    code = ctypes.c_int(-12345)
    rc = s3b.lib().s3b_conv3x3_noalloc_status(ctypes.byref(code))
    return rc, code.value


def _check(got, ref):
    assert torch.isfinite(got).all()
    err = (got - ref).abs().max().item()
    assert err <= 2e-3 * max(1.0, ref.abs().max().item()), err


def test_noalloc_matches_ctx_entry_point_twice(engine, s3b):
    # two calls in a row with different shapes; both fit in the 32 MiB scratch
    cases = [((1, 72, 72, 256), 256, 1), ((2, 36, 36, 256), 128, 2)]
    for shape, cout, seed in cases:
        x, w, bias = _case(shape, cout, seed)
        B, H, W, _ = shape
        ref = torch.empty(B, H, W, cout, device="cuda", dtype=torch.float32)
        engine.conv3x3(x, w, bias, ref)
        engine.sync()
        got = torch.full((B, H, W, cout), float("nan"), device="cuda", dtype=torch.float32)
        rc = _noalloc(s3b, x, w, bias, got)
        assert rc == 0
        torch.cuda.synchronize()
        _check(got, ref)
        # every bounded wait of the call finished: the status word reads 0
        assert _status(s3b) == (0, 0)


def test_noalloc_rejects_sizes_beyond_scratch(engine, s3b):
    # 1 x 80 x 80 x 256 needs 80*80*9*256*2 = 29.5 MB (fits); 1 x 96 x 96 x 256 needs 42.5 MB (rejected)
    x, w, bias = _case((1, 96, 96, 256), 256, 3)
    out = torch.zeros(1, 96, 96, 256, device="cuda", dtype=torch.float32)
    assert 96 * 96 * 9 * 256 * 2 > SCRATCH_BYTES
    rc = _noalloc(s3b, x, w, bias, out)
    assert rc == -1  # S3B_ERR_ARG
    torch.cuda.synchronize()
    assert out.abs().max().item() == 0.0


def test_noalloc_ragged_k_on_user_stream_after_larger_call(engine, s3b):
    # C = 72: K = 648 is not a multiple of the GEMM's 64-wide k-block (a partial last k tile), run on a
    # stream the caller created, right after a call that filled more of the scratch (so the im2col region
    # must be rewritten, not read from the earlier call)
    big = _case((1, 64, 64, 256), 64, 4)
    out_big = torch.empty(1, 64, 64, 64, device="cuda", dtype=torch.float32)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    assert _noalloc(s3b, *big, out_big, stream=side) == 0
    x, w, bias = _case((2, 20, 24, 72), 40, 5)
    ref = torch.empty(2, 20, 24, 40, device="cuda", dtype=torch.float32)
    engine.set_option("conv_implicit", 0)
    try:
        engine.conv3x3(x, w, bias, ref)
        engine.sync()
    finally:
        engine.set_option("conv_implicit", 1)
    got = torch.full((2, 20, 24, 40), float("nan"), device="cuda", dtype=torch.float32)
    assert _noalloc(s3b, x, w, bias, got, stream=side) == 0
    side.synchronize()
    _check(got, ref)
    assert _status(s3b) == (0, 0)
    # and the earlier, larger call on the same stream was right too
    ref_big = torch.empty_like(out_big)
    engine.conv3x3(*big, ref_big)
    engine.sync()
    _check(out_big, ref_big)


def test_noalloc_and_ctx_ops_on_a_second_gpu(s3b):
    # kernel attributes (the dynamic shared-memory opt-in) are per device: the first use of a kernel on
    # cuda:1, after cuda:0 in the same process, must set them up there too
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    for dev in (0, 1):
        with torch.cuda.device(dev):
            e = s3b.Engine(dev)
            try:
                e.set_stream(torch.cuda.current_stream(dev).cuda_stream)
                x, w, bias = _case((1, 32, 32, 128), 64, 6 + dev, device=f"cuda:{dev}")
                ref = torch.empty(1, 32, 32, 64, device=f"cuda:{dev}", dtype=torch.float32)
                e.conv3x3(x, w, bias, ref)
                e.sync()
                got = torch.full_like(ref, float("nan"))
                assert _noalloc(s3b, x, w, bias, got) == 0
                torch.cuda.synchronize(dev)
                _check(got, ref)
                assert _status(s3b) == (0, 0)
                e.set_stream(None)
            finally:
                e.close()
