"""Failure detection on the device, tested without faulting or hanging the GPU.

Every wait of the engine's kernels (a TMA stage, an accumulator, a peer CTA) is bounded: a wait that runs
out records a code in the context's device error word and the kernel returns, so the host sees an error
instead of a hung GPU. s3b_test_wait_timeout runs one kernel whose barrier wait uses that same bounded wait
with a short limit; withholding the barrier's only arrive makes the wait run out (a flag that nothing sets).
The next s3b_sync must report S3B_ERR_DEVICE, clear the word, and the context must stay usable."""
import ctypes
import time

import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

S3B_OK, S3B_ERR_ARG, S3B_ERR_DEVICE = 0, -1, -7


def test_bounded_wait_runs_out_into_an_error_and_the_context_survives(s3b):
    eng = s3b.Engine(0)
    L = s3b.lib()
    try:
        # the arrive is made: the wait completes, no error
        assert L.s3b_test_wait_timeout(eng.h, 50_000_000, 0) == S3B_OK
        assert L.s3b_sync(eng.h) == S3B_OK
        # the arrive is withheld: the wait gives up after its 50 ms limit
        t0 = time.perf_counter()
        assert L.s3b_test_wait_timeout(eng.h, 50_000_000, 1) == S3B_OK
        rc = L.s3b_sync(eng.h)
        elapsed = time.perf_counter() - t0
        assert rc == S3B_ERR_DEVICE, rc
        assert b"timed out" in L.s3b_last_error(eng.h)
        assert 0.04 <= elapsed < 5.0, elapsed
        # the word was cleared and the context still computes correctly
        assert L.s3b_sync(eng.h) == S3B_OK
        g = torch.Generator(device="cuda").manual_seed(1)
        A = torch.randn(256, 128, device="cuda", generator=g).half()
        B = torch.randn(64, 128, device="cuda", generator=g).half()
        out = torch.empty(256, 64, device="cuda", dtype=torch.float32)
        eng.set_stream(torch.cuda.current_stream().cuda_stream)
        eng.gemm(A, B, out)
        eng.sync()
        ref = A.float() @ B.float().T
        assert (out - ref).abs().max().item() < 2e-2
        eng.set_stream(None)
        # limits outside (0, 2 s] are refused before anything is launched
        assert L.s3b_test_wait_timeout(eng.h, 0, 1) == S3B_ERR_ARG
        assert L.s3b_test_wait_timeout(eng.h, 3_000_000_000, 1) == S3B_ERR_ARG
        assert L.s3b_sync(eng.h) == S3B_OK
    finally:
        eng.close()
