"""Failure detection without a GPU fault. Every wait of the persistent kernels
is an mbarrier wait with a cycle budget; when it runs out the kernel sets the
timeout bit of the device status word and returns, and the call reports
RNS8_BACKEND_FAILURE. rns8_cuda_wait_probe runs that wait in isolation: with
nothing arriving on the barrier (a flag that nothing sets) it must give up
within its budget, report the failure, and leave the context usable."""

from __future__ import annotations

import ctypes as C
import time

import numpy as np
import pytest

OK, INVALID, BACKEND_FAILURE = 0, 1, 8


@pytest.fixture(scope="module")
def lib():
    import rns8_b200

    return rns8_b200.lib()


def test_probe_rejects_bad_arguments(lib):
    fake = C.c_void_p(256)  # never dereferenced: validation comes first
    assert lib.rns8_cuda_wait_probe(0, 0, 1000, None, None) == INVALID
    assert lib.rns8_cuda_wait_probe(0, 2, 1000, fake, None) == INVALID
    assert lib.rns8_cuda_wait_probe(0, 0, 0, fake, None) == INVALID
    assert lib.rns8_cuda_wait_probe(0, 0, 4_000_000_001, fake, None) == INVALID


@pytest.mark.gpu
def test_wait_runs_out_and_context_stays_usable(lib):
    torch = pytest.importorskip("torch")
    import rns8_b200 as r8

    status = torch.zeros(4, dtype=torch.int32, device="cuda")
    s = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert lib.rns8_cuda_wait_probe(0, 1, 1_000_000, status.data_ptr(), s) == OK  # the barrier completes
    assert int(status[0].item()) == 0
    t0 = time.perf_counter()
    assert lib.rns8_cuda_wait_probe(0, 0, 20_000_000, status.data_ptr(), s) == BACKEND_FAILURE  # ~10 ms budget
    elapsed = time.perf_counter() - t0
    assert int(status[0].item()) & 0x100  # kDevWaitTimeout
    assert elapsed < 2.0
    # The device and a context on it still work: a bounded one-shot GEMM.
    ctx = r8.Context(0)
    rng = np.random.default_rng(3)
    A = rng.integers(-(2**20), 2**20, (64, 48), dtype=np.int64, endpoint=True)
    B = rng.integers(-(2**20), 2**20, (48, 32), dtype=np.int64, endpoint=True)
    desc = r8.gemm_desc(r8.Semantics.BOUNDED_I64, r8.BoundKind.GLOBAL_MAX_ABS, 64, 32, 48, bound=48 * 2**40)
    np.testing.assert_array_equal(r8.gemm_i64_oneshot(ctx, desc, A, B), A @ B)
    # And the probe passes again once something arrives.
    assert lib.rns8_cuda_wait_probe(0, 1, 1_000_000, status.data_ptr(), s) == OK
    ctx.close()
