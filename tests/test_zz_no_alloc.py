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


def _noalloc(s3b, x, w, bias, out):
    B, H, W, C = x.shape
    Cout = w.shape[0]
    stream = torch.cuda.current_stream().cuda_stream
    return s3b.lib().s3b_conv3x3_noalloc(x.data_ptr(), B, H, W, C, w.data_ptr(),
                                         bias.data_ptr() if bias is not None else None, out.data_ptr(), Cout,
                                         ctypes.c_void_p(stream))


def _case(shape, cout, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    B, H, W, C = shape
    x = torch.randn(B, H, W, C, device="cuda", generator=g).half()
    w = (torch.randn(cout, 3, 3, C, device="cuda", generator=g) * 0.05).half()
    bias = torch.randn(cout, device="cuda", generator=g) * 0.1
    return x, w, bias


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
        assert torch.isfinite(got).all()
        err = (got - ref).abs().max().item()
        assert err <= 2e-3 * max(1.0, ref.abs().max().item()), err


def test_noalloc_rejects_sizes_beyond_scratch(engine, s3b):
    # 1 x 80 x 80 x 256 needs 80*80*9*256*2 = 29.5 MB (fits); 1 x 96 x 96 x 256 needs 42.5 MB (rejected)
    x, w, bias = _case((1, 96, 96, 256), 256, 3)
    out = torch.zeros(1, 96, 96, 256, device="cuda", dtype=torch.float32)
    assert 96 * 96 * 9 * 256 * 2 > SCRATCH_BYTES
    rc = _noalloc(s3b, x, w, bias, out)
    assert rc == -1  # S3B_ERR_ARG
    torch.cuda.synchronize()
    assert out.abs().max().item() == 0.0
