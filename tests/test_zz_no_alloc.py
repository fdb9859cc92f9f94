"""The allocation-free plane GEMM (rns8_cuda_gemm_rns_device_no_alloc).

It exists for callers that cannot allocate device memory — a host whose
device memory belongs to a fixed-budget allocator, a foreign-language caller
that holds only its input and output buffers, a loop where cudaMalloc would
synchronise the device — and takes its scratch from a file-scope device array
instead. Its output must equal the allocating entry point's bit for bit (the
tolerance for this integer work is zero), on two calls in a row so that the
shared array's leftover split-K sums cannot leak into the next result. This
file is collected last and also passes alone in a fresh process.
"""

import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

LADDER = [256, 255, 253, 251, 247, 239, 233, 229, 227, 223, 217, 211, 199, 197, 193, 191, 181, 179, 173, 167]
INVALID_ARGUMENT = 1
WORKSPACE_TOO_SMALL = 7


@pytest.fixture(scope="module")
def lib(rns8):
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    h = rns8.lib()
    fn = h.rns8_cuda_gemm_rns_device_no_alloc
    fn.restype = C.c_uint32
    fn.argtypes = [C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_int64, C.c_int64, C.c_uint32,
                   C.c_void_p]
    return h


def residues(rng, planes, rows, cols):
    out = np.empty((planes, rows, cols), np.int8)
    for p in range(planes):
        m = LADDER[p]
        lo, hi = (-128, 127) if m == 256 else (-(m // 2), m // 2)
        out[p] = rng.integers(lo, hi + 1, (rows, cols)).astype(np.int8)
    return torch.from_numpy(out).cuda()


@pytest.mark.parametrize("m,n,k,prefix", [
    (256, 256, 8192, 8),   # few output tiles: K is split, the array holds the int32 sums
    (1024, 1024, 512, 9),  # 288 tiles, no split: only the status word is used
    (130, 272, 2048, 3),   # ragged tails with a split
    (130, 272, 1000, 3),   # K % 16 != 0: zero-padded plane copies fit in the array
    (512, 512, 1000, 9),   # K % 16 != 0 and the padded copies exceed 8 MiB: CUDA-core kernels on the array
])
def test_no_alloc_matches_allocating_entry_point(lib, m, n, k, prefix):
    rng = np.random.default_rng(m + n + k + prefix)
    a = residues(rng, prefix, m, k)
    b = residues(rng, prefix, k, n)
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    want = torch.empty((prefix, m, n), dtype=torch.int8, device="cuda")
    status = torch.zeros(4, dtype=torch.int32, device="cuda")
    sb = lib.rns8_cuda_gemm_rns_scratch_bytes(0, m, n, k, prefix)
    scratch = torch.empty(max(sb, 1), dtype=torch.uint8, device="cuda")
    assert lib.rns8_cuda_gemm_rns_device(0, a.data_ptr(), b.data_ptr(), want.data_ptr(), m, n, k, prefix, 0,
                                         scratch.data_ptr(), sb, status.data_ptr(), stream) == 0
    torch.cuda.synchronize()
    assert int(status[0].item()) == 0
    for call in range(2):
        got = torch.full((prefix, m, n), 77, dtype=torch.int8, device="cuda")
        assert lib.rns8_cuda_gemm_rns_device_no_alloc(0, a.data_ptr(), b.data_ptr(), got.data_ptr(), m, n, k,
                                                      prefix, stream) == 0
        torch.cuda.synchronize()
        assert torch.equal(got, want), f"call {call}"


def test_no_alloc_rejects_problems_beyond_the_array(lib):
    # 512 x 512 with 9 planes gives 72 tiles, so K is split and the sums need
    # 9 * 512 * 512 * 4 bytes = 9 MiB > 8 MiB: rejected before any launch.
    m = n = 512
    k, prefix = 1024, 9
    a = torch.zeros((prefix, m, k), dtype=torch.int8, device="cuda")
    b = torch.zeros((prefix, k, n), dtype=torch.int8, device="cuda")
    c = torch.full((prefix, m, n), 5, dtype=torch.int8, device="cuda")
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert lib.rns8_cuda_gemm_rns_scratch_bytes(0, m, n, k, prefix) > 8 << 20
    assert lib.rns8_cuda_gemm_rns_device_no_alloc(0, a.data_ptr(), b.data_ptr(), c.data_ptr(), m, n, k, prefix,
                                                  stream) == WORKSPACE_TOO_SMALL
    torch.cuda.synchronize()
    assert bool((c == 5).all())


def test_no_alloc_device_id_and_current_device(lib):
    # A device id the process cannot see is the caller's mistake, and the call
    # leaves the caller's current device as it found it.
    m = n = k = 64
    a = torch.zeros((1, m, k), dtype=torch.int8, device="cuda")
    b = torch.zeros((1, k, n), dtype=torch.int8, device="cuda")
    c = torch.full((1, m, n), 5, dtype=torch.int8, device="cuda")
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    count = torch.cuda.device_count()
    for bad in (-1, count, count + 7):
        assert lib.rns8_cuda_gemm_rns_device_no_alloc(bad, a.data_ptr(), b.data_ptr(), c.data_ptr(), m, n, k, 1,
                                                      stream) == INVALID_ARGUMENT
    torch.cuda.synchronize()
    assert bool((c == 5).all())
    before = torch.cuda.current_device()
    assert lib.rns8_cuda_gemm_rns_device_no_alloc(0, a.data_ptr(), b.data_ptr(), c.data_ptr(), m, n, k, 1,
                                                  stream) == 0
    assert torch.cuda.current_device() == before
    torch.cuda.synchronize()
    assert bool((c == 0).all())
