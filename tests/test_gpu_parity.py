"""GPU parity: every kernel of the hot path against the CPU oracle, bit for bit.

Calls go through librns8.so's C ABI only: the device-pointer seam
(include/rns8/rns8_cuda.h) for the individual kernels and the public
rns8.h entry points for the whole path. torch is used only to hold device
memory. Sizes are ones the oracle finishes in seconds; the full-size
configurations are checked through size-independent properties (exact
products recomputed with limb-split fp64 GEMMs).
"""

import ctypes as C
import json
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

OK, RANGE = 0, 5
KATS = json.loads((Path(__file__).resolve().parent / "golden" / "reference_kats.json").read_text())
LADDER = [256, 255, 253, 251, 247, 239, 233, 229, 227, 223, 217, 211, 199, 197, 193, 191, 181, 179, 173, 167]


def dev(a: np.ndarray):
    if a.dtype == np.uint64:
        a = a.view(np.int64)
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t, dtype=None):
    a = t.cpu().numpy()
    return a.view(dtype) if dtype is not None else a


def stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def random_residues(rng, planes, rows, cols):
    out = np.empty((planes, rows, cols), np.int8)
    for p in range(planes):
        m = LADDER[p]
        lo = -(m // 2) if m % 2 else -128
        hi = m // 2 if m % 2 else 127
        out[p] = rng.integers(lo, hi + 1, (rows, cols), dtype=np.int64).astype(np.int8)
    return out


@pytest.fixture(scope="module")
def lib(rns8):
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return rns8.lib()


# ---- pack -------------------------------------------------------------------------
@pytest.mark.parametrize("prefix", [1, 7, 9, 18, 20])
@pytest.mark.parametrize("shape,ld", [((64, 256), 256), ((7, 13), 15), ((33, 40), 48)])
def test_pack_i64_u64_match_oracle(lib, oracle, prefix, shape, ld):
    rng = np.random.default_rng(prefix * 1000 + shape[0])
    rows, cols = shape
    full = rng.integers(-(2**63), 2**63 - 1, (rows, ld), dtype=np.int64, endpoint=True)
    full[0, : min(cols, 6)] = [-(2**63), 2**63 - 1, -1, 0, 1, -(2**62)][: min(cols, 6)]
    for signed in (True, False):
        src = full if signed else full.view(np.uint64)
        want = oracle.pack(src[:, :cols], prefix)
        d_src = dev(src)
        d_out = torch.empty((prefix, rows, cols), dtype=torch.int8, device="cuda")
        fn = lib.rns8_cuda_pack_i64_device if signed else lib.rns8_cuda_pack_u64_device
        assert fn(0, d_src.data_ptr(), rows, cols, ld, prefix, d_out.data_ptr(), stream()) == OK
        torch.cuda.synchronize()
        np.testing.assert_array_equal(host(d_out), want)


U8_MODULI = [2, 97, 127, 128, 129, 170, 171, 172, 251, 255, 256]  # per-byte modulo, one subtraction, one compare, identity
U8_SHAPES = [((32, 64), 64),    # contiguous: 16-byte groups over the flattened matrix
             ((16, 48), 64),    # strided rows, 16-byte groups per row
             ((5, 9), 11)]      # ragged: one byte per thread


@pytest.mark.parametrize("modulus", U8_MODULI)
@pytest.mark.parametrize("shape,ld", U8_SHAPES)
def test_pack_finite_u8_matches_oracle(lib, oracle, modulus, shape, ld):
    rng = np.random.default_rng(modulus)
    src = rng.integers(0, 256, (shape[0], ld), dtype=np.uint8)
    want = oracle.pack_finite_u8(src[:, : shape[1]], modulus)
    d_out = torch.empty(shape, dtype=torch.int8, device="cuda")
    d_src = dev(src)
    assert lib.rns8_cuda_pack_finite_u8_device(0, d_src.data_ptr(), shape[0], shape[1], ld, modulus,
                                               d_out.data_ptr(), stream()) == OK
    torch.cuda.synchronize()
    np.testing.assert_array_equal(host(d_out), want)


@pytest.mark.parametrize("modulus", U8_MODULI)
@pytest.mark.parametrize("shape,ld", U8_SHAPES)
def test_export_finite_u8_canonical(lib, oracle, modulus, shape, ld):
    """Centered residues -> canonical bytes (cpu_reference.cpp:132-153); padding untouched."""
    rng = np.random.default_rng(modulus + ld)
    src = rng.integers(0, 256, shape, dtype=np.uint8)
    res = oracle.pack_finite_u8(src, modulus)
    want = (src.astype(np.int64) % modulus).astype(np.uint8)
    d_res = dev(res)
    d_out = torch.full((shape[0], ld), 7, dtype=torch.uint8, device="cuda")
    assert lib.rns8_cuda_export_finite_u8_device(0, d_res.data_ptr(), shape[0], shape[1], modulus,
                                                 d_out.data_ptr(), ld, stream()) == OK
    torch.cuda.synchronize()
    got = host(d_out)
    np.testing.assert_array_equal(got[:, : shape[1]], want)
    assert (got[:, shape[1]:] == 7).all()


# ---- plane GEMM -------------------------------------------------------------------
def run_gemm(lib, a, b, prefix, path):
    _, m, k = a.shape
    n = b.shape[2]
    d_a, d_b = dev(a), dev(b)
    d_c = torch.full((prefix, m, n), 99, dtype=torch.int8, device="cuda")
    status = torch.zeros(4, dtype=torch.int32, device="cuda")
    scratch_bytes = lib.rns8_cuda_gemm_rns_scratch_bytes(0, m, n, k, prefix)
    scratch = torch.empty(max(scratch_bytes, 1), dtype=torch.uint8, device="cuda")
    st = lib.rns8_cuda_gemm_rns_device(0, d_a.data_ptr(), d_b.data_ptr(), d_c.data_ptr(), m, n, k, prefix, path,
                                       scratch.data_ptr(), scratch_bytes, status.data_ptr(), stream())
    torch.cuda.synchronize()
    return st, host(d_c), int(status[0].item())


@pytest.mark.parametrize("m,n,k,prefix", [
    (128, 256, 128, 9),     # one tile, one K block
    (256, 512, 1024, 9),    # several tiles
    (200, 272, 336, 7),     # ragged M, N and K tails (TMA zero fill)
    (64, 16, 16, 20),       # tiny, all planes of the widest prefix
    (384, 768, 2048, 3),
    (130, 48, 4096, 2),     # few tiles -> split-K with int32 scratch
])
def test_plane_gemm_tensor_core_and_simt_match_oracle(lib, oracle, m, n, k, prefix):
    rng = np.random.default_rng(m * 7 + n * 3 + k + prefix)
    a = random_residues(rng, prefix, m, k)
    b = random_residues(rng, prefix, k, n)
    want = oracle.gemm_rns(a, b, prefix)
    for path in (1, 2):  # tensor core, SIMT
        st, got, word = run_gemm(lib, a, b, prefix, path)
        assert st == OK and word == 0, path
        np.testing.assert_array_equal(got, want, err_msg=f"path {path}")


def test_plane_gemm_unaligned_shapes_use_simt(lib, oracle):
    rng = np.random.default_rng(5)
    for m, n, k in [(1, 1, 1), (3, 5, 7), (8, 8, 8), (17, 33, 65), (5, 24, 100)]:
        a = random_residues(rng, 9, m, k)
        b = random_residues(rng, 9, k, n)
        st, got, word = run_gemm(lib, a, b, 9, 0)
        assert st == OK and word == 0
        np.testing.assert_array_equal(got, oracle.gemm_rns(a, b, 9))
        if k % 16 or n % 16:
            st, _, _ = run_gemm(lib, a, b, 9, 1)
            assert st == 1  # the tensor-core path refuses rows TMA cannot address


@pytest.mark.parametrize("m,n,k", [
    (1000, 1000, 1000),   # K and N not multiples of 16: zero-padded onto the tensor cores
    (300, 4090, 512),     # N ragged, several N tiles, C cropped back
    (200, 256, 4100),     # K ragged, few tiles: split-K on the padded problem
    (129, 17, 77),        # smallest N for the padded path
])
def test_unaligned_shapes_padded_onto_tensor_cores(lib, oracle, m, n, k):
    """Auto path with the advertised scratch: K or N not multiples of 16 run
    the tensor-core kernel on zero-padded copies; the residues must equal the
    oracle's and the CUDA-core kernel's byte for byte."""
    rng = np.random.default_rng(m + 3 * n + 7 * k)
    P = 9
    a = random_residues(rng, P, m, k)
    b = random_residues(rng, P, k, n)
    a[:, 0, :] = -128
    b[:, :, 0] = -128
    st, got, word = run_gemm(lib, a, b, P, 0)
    assert st == OK and word == 0
    st, simt, _ = run_gemm(lib, a, b, P, 2)
    assert st == OK
    np.testing.assert_array_equal(got, simt)
    if m * n * k <= 300 * 4090 * 512:
        np.testing.assert_array_equal(got, oracle.gemm_rns(a, b, P))


def test_misaligned_plane_pointers_padded(lib, oracle):
    """Plane pointers off a 16-byte boundary (aligned shapes) take the padded
    copies too."""
    rng = np.random.default_rng(12)
    P, m, n, k = 3, 64, 32, 48
    a = random_residues(rng, P, m, k)
    b = random_residues(rng, P, k, n)
    raw_a = torch.zeros(a.size + 16, dtype=torch.int8, device="cuda")
    raw_b = torch.zeros(b.size + 16, dtype=torch.int8, device="cuda")
    raw_c = torch.zeros(P * m * n + 16, dtype=torch.int8, device="cuda")
    raw_a[3:3 + a.size] = dev(a).reshape(-1)
    raw_b[5:5 + b.size] = dev(b).reshape(-1)
    status = torch.zeros(4, dtype=torch.int32, device="cuda")
    sb = lib.rns8_cuda_gemm_rns_scratch_bytes(0, m, n, k, P) + (1 << 20)  # room for the padded copies
    scratch = torch.empty(sb, dtype=torch.uint8, device="cuda")
    st = lib.rns8_cuda_gemm_rns_device(0, raw_a.data_ptr() + 3, raw_b.data_ptr() + 5, raw_c.data_ptr() + 7, m, n, k, P,
                                       0, scratch.data_ptr(), sb, status.data_ptr(), stream())
    torch.cuda.synchronize()
    assert st == OK and int(status[0].item()) == 0
    got = raw_c[7:7 + P * m * n].cpu().numpy().reshape(P, m, n)
    np.testing.assert_array_equal(got, oracle.gemm_rns(a, b, P))


def test_finite_grouped_unaligned_k(lib, oracle):
    rng = np.random.default_rng(13)
    tasks, m, n, k, mod = 40, 96, 48, 100, 251  # two launches of padded tasks
    a = rng.integers(-125, 126, (tasks, m, k)).astype(np.int8)
    b = rng.integers(-125, 126, (tasks, k, n)).astype(np.int8)
    d_a, d_b = dev(a), dev(b)
    d_c = torch.empty((tasks, m, n), dtype=torch.int8, device="cuda")
    pa = (C.c_void_p * tasks)(*[d_a[t].data_ptr() for t in range(tasks)])
    pb = (C.c_void_p * tasks)(*[d_b[t].data_ptr() for t in range(tasks)])
    pc = (C.c_void_p * tasks)(*[d_c[t].data_ptr() for t in range(tasks)])
    status = torch.zeros(4, dtype=torch.int32, device="cuda")
    sb = lib.rns8_cuda_gemm_finite_u8_scratch_bytes(0, m, n, k, tasks)
    assert sb > 0
    scratch = torch.empty(sb, dtype=torch.uint8, device="cuda")
    assert lib.rns8_cuda_gemm_finite_u8_grouped_device(0, pa, pb, pc, tasks, m, n, k, mod, 0, scratch.data_ptr(), sb,
                                                       status.data_ptr(), stream()) == OK
    torch.cuda.synchronize()
    assert int(status[0].item()) == 0
    got = host(d_c)
    for t in range(0, tasks, 7):
        np.testing.assert_array_equal(got[t], oracle.ring_gemm(a[t], b[t], mod))


@pytest.mark.parametrize("k", [65536, 65536 + 128, 2 * 65536 + 256])
def test_plane_gemm_k_longer_than_safe_block(lib, oracle, k):
    # Worst-case magnitudes: every product is (-128)(-128) on the 256 plane.
    m, n, prefix = 128, 256, 2
    a = np.full((prefix, m, k), -128, np.int8)
    b = np.full((prefix, k, n), -128, np.int8)
    a[1] = -127
    b[1] = 127
    a[:, 1, ::3] = 5
    want = oracle.gemm_rns(a, b, prefix)
    for path in (1, 2):
        st, got, word = run_gemm(lib, a, b, prefix, path)
        assert st == OK and word == 0
        np.testing.assert_array_equal(got, want, err_msg=f"path {path}")


@pytest.mark.parametrize("m,n,k", [
    (300, 1, 4096),     # GEMV
    (37, 3, 40),        # K not a multiple of 16: 4-byte steps with bounds checks
    (513, 8, 1000),
    (64, 12, 4096),
    (300, 15, 70000),   # K above 65536: two exact int32 segments per row
    (1, 15, 33),
    # Few rows: K split across warps, residues accumulated per cell, finalized.
    (1, 1, 65536),
    (1, 1, 131073),     # K above 65536 and not a multiple of 16
    (2, 7, 65537),
    (8, 8, 4096),
    (64, 1, 8192),
    (3, 15, 200000),
])
@pytest.mark.parametrize("P", [9, 20])
def test_narrow_output_gemm_matches_oracle(lib, oracle, m, n, k, P):
    """n < 16 runs the narrow-output kernel (B^T staging + dp4a stream; with
    few rows, K split across warps); it must agree with the oracle and with
    the SIMT kernel byte for byte."""
    if P == 20 and m * k > 600_000:
        pytest.skip("the 20-plane case runs on the smaller shapes")
    rng = np.random.default_rng(m * 31 + n * 7 + k + P)
    a = random_residues(rng, P, m, k)
    b = random_residues(rng, P, k, n)
    for p in range(P):  # the most negative residue of each plane along the first row
        a[p, 0, :] = -128 if LADDER[p] % 2 == 0 else -(LADDER[p] // 2)
    st, got, word = run_gemm(lib, a, b, P, 0)
    assert st == OK and word == 0
    want = oracle.gemm_rns(a, b, P)
    np.testing.assert_array_equal(got, want)
    st, simt, _ = run_gemm(lib, a, b, P, 2)
    assert st == OK
    np.testing.assert_array_equal(simt, want)


def test_finite_grouped_gemm_matches_oracle(lib, oracle):
    rng = np.random.default_rng(11)
    tasks, m, n, k, mod = 5, 256, 256, 512, 251
    a = rng.integers(-125, 126, (tasks, m, k)).astype(np.int8)
    b = rng.integers(-125, 126, (tasks, k, n)).astype(np.int8)
    d_a, d_b = dev(a), dev(b)
    d_c = torch.empty((tasks, m, n), dtype=torch.int8, device="cuda")
    pa = (C.c_void_p * tasks)(*[d_a[t].data_ptr() for t in range(tasks)])
    pb = (C.c_void_p * tasks)(*[d_b[t].data_ptr() for t in range(tasks)])
    pc = (C.c_void_p * tasks)(*[d_c[t].data_ptr() for t in range(tasks)])
    status = torch.zeros(4, dtype=torch.int32, device="cuda")
    sb = lib.rns8_cuda_gemm_finite_u8_scratch_bytes(0, m, n, k, tasks)
    scratch = torch.empty(max(sb, 1), dtype=torch.uint8, device="cuda")
    assert lib.rns8_cuda_gemm_finite_u8_grouped_device(0, pa, pb, pc, tasks, m, n, k, mod, 1, scratch.data_ptr(), sb,
                                                       status.data_ptr(), stream()) == OK
    torch.cuda.synchronize()
    assert int(status[0].item()) == 0
    got = host(d_c)
    for t in range(tasks):
        np.testing.assert_array_equal(got[t], oracle.ring_gemm(a[t], b[t], mod))


# ---- GEMM + export in one call --------------------------------------------------------
def run_gemm_export(lib, a, b, prefix, bound, signed=True, ld=None):
    _, m, k = a.shape
    n = b.shape[2]
    ld = ld or n
    d_a, d_b = dev(a), dev(b)
    out = torch.full((m, ld), -7, dtype=torch.int64, device="cuda")
    status = torch.zeros(4, dtype=torch.int32, device="cuda")
    sb = lib.rns8_cuda_gemm_export_bounded_scratch_bytes(0, m, n, k, prefix)
    scratch = torch.empty(max(sb, 1), dtype=torch.uint8, device="cuda")
    st = lib.rns8_cuda_gemm_export_bounded_device(0, d_a.data_ptr(), d_b.data_ptr(), m, n, k, prefix, int(signed),
                                                  bound, out.data_ptr(), ld, scratch.data_ptr(), sb, status.data_ptr(),
                                                  stream())
    torch.cuda.synchronize()
    return st, host(out, None if signed else np.uint64), int(status[0].item())


@pytest.mark.parametrize("m,n,k,prefix,signed", [
    (2048, 4096, 64, 9, True),
    (1920, 4352, 48, 5, False),    # ragged M, unsigned
    (512, 512, 64, 9, True),
])
def test_gemm_export_bounded_matches_oracle(lib, oracle, m, n, k, prefix, signed):
    rng = np.random.default_rng(m + n + k)
    lim = 2**12 if prefix == 5 else 2**26
    if signed:
        A = rng.integers(-lim, lim, (m, k), dtype=np.int64, endpoint=True)
        B = rng.integers(-lim, lim, (k, n), dtype=np.int64, endpoint=True)
    else:
        A = rng.integers(0, lim, (m, k), dtype=np.uint64, endpoint=True)
        B = rng.integers(0, lim, (k, n), dtype=np.uint64, endpoint=True)
    bound = k * lim * lim
    a, b = oracle.pack(A, prefix), oracle.pack(B, prefix)
    planes = oracle.gemm_rns(a, b, prefix)
    ost, want = oracle.export_i64(planes, prefix, bound) if signed else oracle.export_u64(planes, prefix, bound)
    assert ost == OK
    st, got, word = run_gemm_export(lib, a, b, prefix, bound, signed)
    assert st == OK and word == 0
    np.testing.assert_array_equal(got, want)
    # A bound the values exceed: RANGE_ERROR through the status word.
    st, _, word = run_gemm_export(lib, a, b, prefix, 1, signed)
    assert st == OK and word == RANGE
    # Strided destination: cells land at row * ld + col, the padding is untouched.
    st, got, word = run_gemm_export(lib, a, b, prefix, bound, signed, ld=n + 6)
    assert st == OK and word == 0
    np.testing.assert_array_equal(got[:, :n], want)
    assert (got[:, n:].astype(np.int64) == -7).all()


# ---- export -------------------------------------------------------------------------
def product_planes(oracle, rng, m, n, k, prefix, lo, hi, dtype=np.int64):
    A = rng.integers(lo, hi, (m, k), dtype=dtype, endpoint=True)
    B = rng.integers(lo, hi, (k, n), dtype=dtype, endpoint=True)
    return A, B, oracle.gemm_rns(oracle.pack(A, prefix), oracle.pack(B, prefix), prefix)


@pytest.mark.parametrize("prefix,bound_scale", [(9, 1), (7, 1), (20, 1), (9, 0)])
@pytest.mark.parametrize("m,n", [(48, 40), (96, 130)])  # 12480 cells: streamed kernel, partial last tile
def test_export_bounded_matches_oracle(lib, oracle, prefix, bound_scale, m, n):
    rng = np.random.default_rng(prefix + bound_scale + m)
    k = 64
    lim = 2**24 if prefix == 7 else 2**28
    A, B, planes = product_planes(oracle, rng, m, n, k, prefix, -lim, lim)
    exact = np.array(oracle.exact_product(A, B), dtype=object)
    bound = int(np.abs(exact).max()) if bound_scale else int(np.abs(exact).max()) // 2  # scale 0: forced range error
    ost, owant = oracle.export_i64(planes, prefix, bound)
    d_p = dev(planes)
    d_out = torch.zeros((m, n), dtype=torch.int64, device="cuda")
    status = torch.zeros(4, dtype=torch.int32, device="cuda")
    assert lib.rns8_cuda_export_i64_device(0, d_p.data_ptr(), m, n, prefix, bound, d_out.data_ptr(), n,
                                           status.data_ptr(), stream()) == OK
    torch.cuda.synchronize()
    word = int(status[0].item())
    assert (RANGE if word else OK) == ost
    if ost == OK:
        np.testing.assert_array_equal(host(d_out), owant)
    # Unsigned: nonnegative inputs, canonical values.
    Au, Bu, uplanes = product_planes(oracle, rng, m, n, k, prefix, 0, lim, np.uint64)
    uexact = np.array(oracle.exact_product(Au, Bu), dtype=object)
    ubound = int(uexact.max()) if bound_scale else int(uexact.max()) - 1
    ost, owant = oracle.export_u64(uplanes, prefix, ubound)
    d_p = dev(uplanes)
    status.zero_()
    assert lib.rns8_cuda_export_u64_device(0, d_p.data_ptr(), m, n, prefix, ubound, d_out.data_ptr(), n,
                                           status.data_ptr(), stream()) == OK
    torch.cuda.synchronize()
    word = int(status[0].item())
    assert (RANGE if word else OK) == ost
    if ost == OK:
        np.testing.assert_array_equal(host(d_out, np.uint64), owant)


def test_export_i64_boundaries(lib, oracle):
    # Cells at the int64 and bound edges (test_crt.cpp:92-106 style).
    P = 9
    vals = [-(2**63), 2**63 - 1, -1, 0, 1, 2**62, -(2**62) - 7, 12345]
    planes = np.stack([[[((v % m) - m if (v % m) >= (m + 1) // 2 else v % m) for v in vals]]
                       for m in LADDER[:P]]).astype(np.int8)
    for bound in (2**63, 2**63 - 1, 2**62):
        ost, owant = oracle.export_i64(planes, P, bound)
        d_p = dev(planes)
        d_out = torch.zeros((1, len(vals)), dtype=torch.int64, device="cuda")
        status = torch.zeros(4, dtype=torch.int32, device="cuda")
        assert lib.rns8_cuda_export_i64_device(0, d_p.data_ptr(), 1, len(vals), P, bound, d_out.data_ptr(),
                                               len(vals), status.data_ptr(), stream()) == OK
        torch.cuda.synchronize()
        assert (RANGE if int(status[0].item()) else OK) == ost
        if ost == OK:
            np.testing.assert_array_equal(host(d_out), owant)


def planes_of(values, prefix):
    """Centered residue planes (prefix, 1, len) of Python integers."""
    out = np.empty((prefix, 1, len(values)), dtype=np.int8)
    for p, m in enumerate(LADDER[:prefix]):
        for j, v in enumerate(values):
            r = v % m
            out[p, 0, j] = r - m if r >= (m + 1) // 2 else r
    return out


def modulus_product(prefix):
    out = 1
    for m in LADDER[:prefix]:
        out *= m
    return out


@pytest.mark.parametrize("prefix", [3, 5, 8, 9, 12, 18, 20])
@pytest.mark.parametrize("signed", [True, False])
def test_export_bounded_decision_edges(lib, oracle, prefix, signed):
    """Bounded export at the edges of the accepted interval, for bounds near
    the plan limit and far below it: every cell within a few thousand of +-bound
    (the fixed-point quotient's undecided band), random cells, and out-of-range
    cells anywhere in [0, M). Each call must match the oracle bit for bit."""
    rng = np.random.default_rng(prefix * 2 + signed)
    M = modulus_product(prefix)
    top = min((M - 1) // 2, 2**63) if signed else min(M - 1, 2**64 - 1)
    for bound in sorted({top, top // 3 + 1, max(top >> 20, 1), 1000}):
        lo = -bound if signed else 0
        hi = min(bound, 2**63 - 1) if signed else bound  # +2^63 does not fit int64
        edge = [x for c in ([lo, bound] if signed else [bound]) for x in range(c - 3000, c + 3001, 3)]
        inside = [x for x in edge if lo <= x <= hi]
        inside += [int(v) for v in rng.integers(0, 2**62, 2048)]
        inside = [lo + (x - lo) % (hi - lo + 1) for x in inside]
        inside = inside[: len(inside) // 4 * 4]
        outside = sorted((x for x in edge if not lo <= x <= hi), key=lambda x: min(abs(x - lo), abs(x - hi)))[:6]
        outside += [int(rng.integers(0, 2**62)) * M // 2**62 for _ in range(4)]
        base = planes_of(inside, prefix)
        cases = [(base, True)]
        for x in outside:
            xm = x % M
            if signed and (xm <= hi or xm >= M - bound):
                continue
            if not signed and xm <= bound:
                continue
            bad = base.copy()
            bad[:, :, -1:] = planes_of([x], prefix)
            cases.append((bad, False))
        for planes, ok in cases:
            values = inside
            ost, owant = (oracle.export_i64 if signed else oracle.export_u64)(planes, prefix, bound)
            assert (ost == OK) == ok
            d_p = dev(planes)
            d_out = torch.zeros((1, len(values)), dtype=torch.int64, device="cuda")
            status = torch.zeros(4, dtype=torch.int32, device="cuda")
            fn = lib.rns8_cuda_export_i64_device if signed else lib.rns8_cuda_export_u64_device
            assert fn(0, d_p.data_ptr(), 1, len(values), prefix, bound, d_out.data_ptr(), len(values),
                      status.data_ptr(), stream()) == OK
            torch.cuda.synchronize()
            assert (RANGE if int(status[0].item()) else OK) == ost, (prefix, signed, bound)
            if ok:
                np.testing.assert_array_equal(host(d_out, None if signed else np.uint64), owant)


@pytest.mark.parametrize("prefix", [1, 9, 18, 20])
@pytest.mark.parametrize("limbs", [1, 2, 3, 4, 8])
# 384 cells: one-cell and vector kernels; 6790 (not a multiple of 16): the
# vector kernel; 12480 (a multiple of 16, not of 128): the streamed kernel
# with a partial last tile; 13056: the tensor-core kernel with a partial last
# stage.
@pytest.mark.parametrize("m,n", [(16, 24), (70, 97), (96, 130), (96, 136)])
def test_export_limbs_match_oracle(lib, oracle, prefix, limbs, m, n):
    rng = np.random.default_rng(prefix * 31 + limbs + m)
    planes = random_residues(rng, prefix, m, n)
    planes[:, 0, 0] = 0
    for signed in (True, False):
        ost, owant = oracle.export_limbs(planes, prefix, limbs, signed)
        d_p = dev(planes)
        d_out = torch.zeros((m, n, limbs), dtype=torch.int64, device="cuda")
        status = torch.zeros(4, dtype=torch.int32, device="cuda")
        assert lib.rns8_cuda_export_limbs_device(0, d_p.data_ptr(), m, n, prefix, 1 if signed else 0, limbs,
                                                 d_out.data_ptr(), n, status.data_ptr(), stream()) == OK
        torch.cuda.synchronize()
        assert (RANGE if int(status[0].item()) else OK) == ost, (signed, prefix, limbs)
        if ost == OK:
            np.testing.assert_array_equal(host(d_out, np.uint64), owant)


@pytest.mark.parametrize("prefix", [9, 20])
@pytest.mark.parametrize("limbs", [3, 2])
def test_export_limbs_strided_destination(lib, oracle, prefix, limbs):
    """A destination with ld > n on the tensor-core limb export (8192 cells,
    whole 128-cell chunks): rows land ld cells apart and the gaps keep their
    bytes."""
    m, n, ld = 64, 128, 136
    rng = np.random.default_rng(prefix * 7 + limbs)
    planes = random_residues(rng, prefix, m, n)
    sentinel = -0x3C3C3C3C3C3C3C3D
    for signed in (True, False):
        ost, owant = oracle.export_limbs(planes, prefix, limbs, signed)
        d_p = dev(planes)
        d_out = torch.full((m, ld, limbs), sentinel, dtype=torch.int64, device="cuda")
        status = torch.zeros(4, dtype=torch.int32, device="cuda")
        assert lib.rns8_cuda_export_limbs_device(0, d_p.data_ptr(), m, n, prefix, 1 if signed else 0, limbs,
                                                 d_out.data_ptr(), ld, status.data_ptr(), stream()) == OK
        torch.cuda.synchronize()
        assert (RANGE if int(status[0].item()) else OK) == ost, (signed, prefix, limbs)
        got = host(d_out, np.uint64)
        if ost == OK:
            np.testing.assert_array_equal(got[:, :n], owant)
        assert (got[:, n:].view(np.int64) == sentinel).all()


@pytest.mark.parametrize("prefix", [2, 9, 18, 20])
@pytest.mark.parametrize("limbs", [3, 1])
@pytest.mark.parametrize("shape", [(4, 8), (16, 64)])
def test_export_limbs_near_half_range(lib, oracle, prefix, limbs, shape):
    """Values at and around +-M/2, where the fractional CRT's quotient is in
    doubt and the exact Garner path must take over, between ordinary values;
    4 x 8 cells for the vector kernel, 16 x 64 (the values repeated) for the
    tensor-core kernel."""
    M = 1
    for mm in LADDER[:prefix]:
        M *= mm
    h = M // 2
    vals = [h - 1, -h, h - 2, -h + 1, 0, 1, -1, h // 3, -(h // 5), h - (1 << 20), -h + (1 << 20), 12345]
    vals += [(i * 0x9E3779B97F4A7C15) % M - h for i in range(1, 21)]
    m, n = shape
    vals = (vals * (m * n // len(vals) + 1))[: m * n]
    centered = lambda v, mm: (lambda r: r - mm if r >= (mm + 1) // 2 else r)(v % mm)
    planes = np.array([[[centered(vals[r * n + c], mm) for c in range(n)] for r in range(m)] for mm in LADDER[:prefix]],
                      np.int8)
    for signed in (True, False):
        ost, owant = oracle.export_limbs(planes, prefix, limbs, signed)
        d_p = dev(planes)
        d_out = torch.zeros((m, n, limbs), dtype=torch.int64, device="cuda")
        status = torch.zeros(4, dtype=torch.int32, device="cuda")
        assert lib.rns8_cuda_export_limbs_device(0, d_p.data_ptr(), m, n, prefix, 1 if signed else 0, limbs,
                                                 d_out.data_ptr(), n, status.data_ptr(), stream()) == OK
        torch.cuda.synchronize()
        assert (RANGE if int(status[0].item()) else OK) == ost, (signed, prefix, limbs)
        if ost == OK:
            np.testing.assert_array_equal(host(d_out, np.uint64), owant)


@pytest.mark.parametrize("case", KATS["exact_wide_limb_boundaries"]["cases"])
@pytest.mark.parametrize("cells", [4, 1, 1024])  # vector, one-cell and tensor-core kernels
def test_export_limbs_reference_boundaries(lib, case, cells):
    """The reference's exact-wide limb boundary answers on the GPU export; on a
    range error the destination keeps its bytes."""
    prefix, signed, value, limbs, want = case

    def centered(v, m):
        r = v % m
        return r - m if r >= (m + 1) // 2 else r
    planes = np.array([[[centered(int(value), m)] * cells] for m in LADDER[:prefix]], np.int8)
    d_p = dev(planes)
    sentinel = -0x5A5A5A5A5A5A5A5B
    d_out = torch.full((1, cells, limbs), sentinel, dtype=torch.int64, device="cuda")
    status = torch.zeros(4, dtype=torch.int32, device="cuda")
    assert lib.rns8_cuda_export_limbs_device(0, d_p.data_ptr(), 1, cells, prefix, 1 if signed else 0, limbs,
                                             d_out.data_ptr(), cells, status.data_ptr(), stream()) == OK
    torch.cuda.synchronize()
    got = host(d_out, np.uint64)
    if want == "range":
        assert int(status[0].item()) == RANGE
    else:
        assert int(status[0].item()) == 0
        for c in range(cells):
            assert [int(v) for v in got[0, c]] == [int(v) for v in want]


# ---- public C ABI: the whole path ----------------------------------------------------
@pytest.fixture(scope="module")
def ctx(rns8):
    c = rns8.Context(0)
    yield c
    c.close()


def test_context_reports_the_b200(rns8, ctx):
    info = ctx.device_info()
    assert info.backend == rns8.Backend.CUDA_SM100 and info.gcn_arch == b"sm_100a"


def test_baseline_c1_oneshot_bit_exact(rns8, oracle, ctx):
    # M=N=K=512, uniform [-2^20, 2^20], bound K*2^40 = 2^49 (plan picks prefix 7).
    rng = oracle.Rng(0x5EED0001)
    A = rng.i64(-(2**20), 2**20, (512, 512))
    B = rng.i64(-(2**20), 2**20, (512, 512))
    desc = rns8.gemm_desc(rns8.Semantics.BOUNDED_I64, rns8.BoundKind.GLOBAL_MAX_ABS, 512, 512, 512, bound=2**49)
    plan = rns8.Plan(ctx, desc)
    assert plan.prefix == 7
    assert b"tcgen05" in plan.backend_info().selected_kernel
    got = rns8.gemm_i64_oneshot(ctx, desc, A, B)
    st, want, used = oracle.gemm_bounded_oneshot(A, B, 2**49)
    assert st == OK and used == 7
    np.testing.assert_array_equal(got, want)
    assert oracle.checksum(got) == oracle.checksum(want)


def test_reference_sweeps_through_public_api(rns8, oracle, ctx):
    # test_bounded_reference_sweeps.cpp:161-243 shapes, through rns8_gemm_{i64,u64}_oneshot.
    I64, U64 = rns8.Semantics.BOUNDED_I64, rns8.Semantics.BOUNDED_U64
    for m in (1, 3, 8):
        for n in (1, 5, 8):
            for k in (1, 2, 7, 8):
                A = np.array([[((r * 17 + c * 5 + m - n) % 11) - 5 for c in range(k)] for r in range(m)], np.int64)
                B = np.array([[((r * 7 - c * 13 + k + n) % 13) - 6 for c in range(n)] for r in range(k)], np.int64)
                exact = np.array(oracle.exact_product(A, B), dtype=object)
                bound = max(1, int(np.abs(exact).max()))
                got = rns8.gemm_i64_oneshot(ctx, rns8.gemm_desc(I64, rns8.BoundKind.GLOBAL_MAX_ABS, m, n, k, bound=bound),
                                            A, B)
                assert got.tolist() == exact.tolist()
    rng = oracle.Rng(0x8A5CD13F00D)
    for _ in range(32):
        m, n, k = 1 + rng.next() % 8, 1 + rng.next() % 8, 1 + rng.next() % 8
        A = np.full((m, k + 1), 12345, np.int64)
        B = np.full((k, n + 1), -12345, np.int64)
        Au = np.full((m, k + 1), 99999, np.uint64)
        Bu = np.full((k, n + 1), 99999, np.uint64)
        for r in range(m):
            for c in range(k):
                A[r, c] = rng.i64(-31, 31, 1)[0]
                Au[r, c] = rng.u64(0, 63, 1)[0]
        for r in range(k):
            for c in range(n):
                B[r, c] = rng.i64(-31, 31, 1)[0]
                Bu[r, c] = rng.u64(0, 63, 1)[0]
        exact = np.array(oracle.exact_product(A[:, :k], B[:, :n]), dtype=object)
        got = rns8.gemm_i64_oneshot(ctx, rns8.gemm_desc(I64, rns8.BoundKind.GLOBAL_MAX_ABS, m, n, k,
                                                        bound=max(1, int(np.abs(exact).max()))), A[:, :k], B[:, :n])
        assert got.tolist() == exact.tolist()
        exact = np.array(oracle.exact_product(Au[:, :k], Bu[:, :n]), dtype=object)
        got = rns8.gemm_u64_oneshot(ctx, rns8.gemm_desc(U64, rns8.BoundKind.GLOBAL_MAX_UNSIGNED, m, n, k,
                                                        bound=max(1, int(exact.max()))), Au[:, :k], Bu[:, :n])
        assert [[int(x) for x in row] for row in got] == exact.tolist()


@pytest.mark.parametrize("k", [65535, 65536, 65537])
def test_k_split_edges_padded_through_public_api(rns8, oracle, ctx, k):
    # test_bounded_reference_sweeps.cpp:370-473 (padded A, C, sentinel columns).
    m, n, sentinel = 2, 2, -0x3210FEDCBA
    A = np.full((m, k + 2), sentinel, np.int64)
    B = np.full((k, 3), sentinel, np.int64)
    kk = np.arange(k)
    A[0, :k] = np.where(kk % 2 == 0, 127, -127)
    A[1, :k] = np.where(kk % 3 == 0, -128, 127)
    B[:, 0] = np.where(kk % 5 == 0, -127, 127)
    B[:, 1] = np.where(kk % 7 == 0, 127, -127)
    exact = np.array([[int((A[r, :k].astype(object) * B[:, c].astype(object)).sum()) for c in range(n)]
                      for r in range(m)], dtype=object)
    Cpad = np.full((m, 3), sentinel, np.int64)
    desc = rns8.gemm_desc(rns8.Semantics.BOUNDED_I64, rns8.BoundKind.GLOBAL_MAX_ABS, m, n, k,
                          bound=int(np.abs(exact).max()), max_prefix=9, flags=rns8.PLAN_FORCE_FIXED_PREFIX)
    rns8.gemm_i64_oneshot(ctx, desc, A[:, :k], B[:, :n], out=Cpad[:, :n])
    assert Cpad[:, :n].tolist() == exact.tolist()
    assert (Cpad[:, n] == sentinel).all()


def test_full_width_and_range_error_leave_dst_untouched(rns8, oracle, ctx):
    s = 0x123456789ABC
    A = np.array([[-(2**63), 2**63 - 1], [-(2**63 - 1), 0]], np.int64)
    B = np.eye(2, dtype=np.int64)
    C3 = np.full((2, 3), s, np.int64)
    desc = rns8.gemm_desc(rns8.Semantics.BOUNDED_I64, rns8.BoundKind.GLOBAL_MAX_ABS, 2, 2, 2, bound=2**63)
    rns8.gemm_i64_oneshot(ctx, desc, A, B, out=C3[:, :2])
    assert C3.tolist() == [[-(2**63), 2**63 - 1, s], [-(2**63 - 1), 0, s]]
    # bound too small: RANGE_ERROR, output untouched
    A = np.array([[1000, 1000]], np.int64)
    B = np.array([[1000], [1000]], np.int64)
    out = np.full((1, 1), 77, np.int64)
    with pytest.raises(rns8.Error) as e:
        rns8.gemm_i64_oneshot(ctx, rns8.gemm_desc(rns8.Semantics.BOUNDED_I64, rns8.BoundKind.GLOBAL_MAX_ABS, 1, 1, 2,
                                                  bound=1_999_999), A, B, out=out)
    assert e.value.status == rns8.Status.RANGE_ERROR and out[0, 0] == 77


def test_persistent_path_and_source_version(rns8, oracle, ctx):
    rng = oracle.Rng(77)
    m, n, k = 130, 272, 320
    A = rng.i64(-(2**26), 2**26, (m, k))
    B = rng.i64(-(2**26), 2**26, (k, n))
    desc = rns8.gemm_desc(rns8.Semantics.BOUNDED_I64, rns8.BoundKind.GLOBAL_MAX_ABS, m, n, k, bound=k * 2**52)
    plan = rns8.Plan(ctx, desc)
    a, b, c = (rns8.Matrix.for_plan(ctx, plan, r) for r in "abc")
    ws = rns8.Workspace(ctx, plan)
    a.pack_i64(A, source_version=1)
    b.pack_i64(B, source_version=2)
    rns8.gemm_rns(ctx, plan, a, b, c, ws)
    got = rns8.export_i64(ctx, plan, c)
    st, want, _ = oracle.gemm_bounded_oneshot(A, B, k * 2**52)
    assert st == OK
    np.testing.assert_array_equal(got, want)
    info = c.storage_info()
    assert info.device_residues_current == 1 and info.device_residue_bytes == plan.prefix * m * n
    # Same source version: the pack is elided even with different host data.
    a.pack_i64(np.zeros_like(A), source_version=1)
    rns8.gemm_rns(ctx, plan, a, b, c, ws)
    np.testing.assert_array_equal(rns8.export_i64(ctx, plan, c), want)


@pytest.mark.parametrize("field,modulus", [(True, 251), (False, 256), (False, 6), (True, 2)])
def test_finite_oneshot_matches_oracle(rns8, oracle, ctx, field, modulus):
    rng = np.random.default_rng(modulus)
    for m, n, k in [(7, 9, 11), (256, 512, 384)]:
        A = rng.integers(0, 256, (m, k), dtype=np.uint8)
        B = rng.integers(0, 256, (k, n), dtype=np.uint8)
        sem = rns8.Semantics.FINITE_FIELD_U8 if field else rns8.Semantics.FINITE_RING_U8
        desc = rns8.gemm_desc(sem, rns8.BoundKind.NONE, m, n, k, finite_modulus=modulus)
        got = rns8.gemm_finite_u8_oneshot(ctx, desc, modulus, A, B, field)
        st, want = oracle.gemm_finite_u8_oneshot(A, B, modulus, field)
        assert st == OK
        np.testing.assert_array_equal(got, want)


def test_finite_grouped_public_api(rns8, oracle, ctx):
    # BASELINE config 2 shape family at a reduced batch: field 251, same-shape tasks.
    rng = np.random.default_rng(2)
    m = n = k = 256
    desc = rns8.gemm_desc(rns8.Semantics.FINITE_FIELD_U8, rns8.BoundKind.NONE, m, n, k, finite_modulus=251)
    plan = rns8.Plan(ctx, desc)
    tasks, inputs = [], []
    for t in range(6):
        A = rng.integers(0, 251, (m, k), dtype=np.uint8)
        B = rng.integers(0, 251, (k, n), dtype=np.uint8)
        a, b, c = (rns8.Matrix.for_plan(ctx, plan, r) for r in "abc")
        a.pack_finite_u8(251, A)
        b.pack_finite_u8(251, B)
        tasks.append((a, b, c, rns8.Workspace(ctx, plan)))
        inputs.append((A, B))
    rns8.gemm_finite_u8_grouped(ctx, plan, 251, tasks)
    for (A, B), (_, _, c, _) in zip(inputs, tasks):
        st, want = oracle.gemm_finite_u8_oneshot(A, B, 251, True)
        np.testing.assert_array_equal(rns8.export_finite_u8(ctx, plan, 251, c), want)


@pytest.mark.parametrize("forced", [False, True])
def test_exact_wide_signed_limbs_persistent(rns8, oracle, ctx, forced):
    # BASELINE config 5 at a reduced size: full-range int64, 3 limbs (prefix 18 default, 20 forced).
    rng = oracle.Rng(5)
    m, n, k = 64, 80, 96
    A = rng.i64(-(2**63), 2**63 - 1, (m, k))
    B = rng.i64(-(2**63), 2**63 - 1, (k, n))
    desc = rns8.gemm_desc(rns8.Semantics.EXACT_WIDE_SIGNED, rns8.BoundKind.NONE, m, n, k,
                          max_prefix=20 if forced else 0, flags=rns8.PLAN_FORCE_FIXED_PREFIX if forced else 0)
    plan = rns8.Plan(ctx, desc)
    P = plan.prefix
    assert P == (20 if forced else 18)
    a, b, c = (rns8.Matrix.for_plan(ctx, plan, r) for r in "abc")
    ws = rns8.Workspace(ctx, plan)
    a.pack_i64(A)
    b.pack_i64(B)
    rns8.gemm_rns(ctx, plan, a, b, c, ws)
    got = rns8.export_exact_wide_limbs(ctx, plan, c, 3, signed=True)
    planes = oracle.gemm_rns(oracle.pack(A, P), oracle.pack(B, P), P)
    st, want = oracle.export_limbs(planes, P, 3, signed=True)
    assert st == OK
    np.testing.assert_array_equal(got, want)
    exact = oracle.exact_product(A[:4, :], B[:, :4])
    for i in range(4):
        for j in range(4):
            v = sum(int(got[i, j, l]) << (64 * l) for l in range(3))
            assert (v - (1 << 192) if v >> 191 else v) == exact[i][j]
    with pytest.raises(rns8.Error) as e:
        rns8.export_exact_wide_limbs(ctx, plan, c, 1, signed=True)
    assert e.value.status == rns8.Status.RANGE_ERROR


# ---- full-size properties ------------------------------------------------------------
def exact_i64_matmul_fp64(A, B):
    """Exact int64 product for |A|,|B| <= 2^24, K <= 8192: split each operand
    into 13-bit limbs, four fp64 GEMMs whose sums stay below 2^53, recombine."""
    sh = 2**13
    Ah, Al = torch.div(A, sh, rounding_mode="floor"), torch.remainder(A, sh)
    Bh, Bl = torch.div(B, sh, rounding_mode="floor"), torch.remainder(B, sh)
    f = lambda x: x.to(torch.float64)
    hh = (f(Ah) @ f(Bh)).to(torch.int64)
    hl = (f(Ah) @ f(Bl)).to(torch.int64) + (f(Al) @ f(Bh)).to(torch.int64)
    ll = (f(Al) @ f(Bl)).to(torch.int64)
    return hh * (sh * sh) + hl * sh + ll


@pytest.mark.parametrize("n,forced,one_call", [(2048, False, False), (8192, True, False), (8192, True, True)])
def test_full_size_bounded_i64_exact(lib, n, forced, one_call):
    """BASELINE config 3 shape (8192^3, U[-2^24, 2^24], bound 2^61, prefix 9
    forced) through the device seam, against an independent exact product."""
    g = torch.Generator(device="cuda").manual_seed(n)
    A = torch.randint(-(2**24), 2**24 + 1, (n, n), device="cuda", dtype=torch.int64, generator=g)
    B = torch.randint(-(2**24), 2**24 + 1, (n, n), device="cuda", dtype=torch.int64, generator=g)
    P = 9 if forced else 8
    ra = torch.empty((P, n, n), dtype=torch.int8, device="cuda")
    rb = torch.empty((P, n, n), dtype=torch.int8, device="cuda")
    rc = torch.empty((P, n, n), dtype=torch.int8, device="cuda")
    out = torch.empty((n, n), dtype=torch.int64, device="cuda")
    status = torch.zeros(4, dtype=torch.int32, device="cuda")
    s = stream()
    assert lib.rns8_cuda_pack_i64_device(0, A.data_ptr(), n, n, n, P, ra.data_ptr(), s) == OK
    assert lib.rns8_cuda_pack_i64_device(0, B.data_ptr(), n, n, n, P, rb.data_ptr(), s) == OK
    if one_call:
        sb = lib.rns8_cuda_gemm_export_bounded_scratch_bytes(0, n, n, n, P)
        scratch = torch.empty(sb, dtype=torch.uint8, device="cuda")
        assert lib.rns8_cuda_gemm_export_bounded_device(0, ra.data_ptr(), rb.data_ptr(), n, n, n, P, 1, 2**61,
                                                        out.data_ptr(), n, scratch.data_ptr(), sb, status.data_ptr(),
                                                        s) == OK
    else:
        assert lib.rns8_cuda_gemm_rns_device(0, ra.data_ptr(), rb.data_ptr(), rc.data_ptr(), n, n, n, P, 1, None, 0,
                                             status.data_ptr(), s) == OK
        assert lib.rns8_cuda_export_i64_device(0, rc.data_ptr(), n, n, P, 2**61, out.data_ptr(), n,
                                               status.data_ptr(), s) == OK
    torch.cuda.synchronize()
    assert int(status[0].item()) == 0
    want = exact_i64_matmul_fp64(A, B)
    assert torch.equal(out, want)


@pytest.mark.parametrize("signed", [True, False])
def test_pipelined_oneshot_matches_exact(rns8, ctx, signed):
    """Large one-shot calls upload A in row slabs on a copy stream overlapped
    with pack / GEMM / export: 1100 rows make two slabs of 640 and 460 rows;
    pageable inputs with padded leading dimensions; a bound the values exceed
    returns RANGE_ERROR and leaves C untouched."""
    rng = np.random.default_rng(1100 + signed)
    m, n, k = 1100, 64, 8192
    lo = -(2**20) if signed else 0
    dt = np.int64 if signed else np.uint64
    A = rng.integers(lo, 2**20, (m, k + 3), dtype=dt, endpoint=True)
    B = rng.integers(lo, 2**20, (k, n + 5), dtype=dt, endpoint=True)
    want = A[:, :k] @ B[:, :n]  # |C| <= 2^53: exact in 64-bit integers
    bound = int(np.abs(want.astype(np.float64)).max()) + 1
    sem = rns8.Semantics.BOUNDED_I64 if signed else rns8.Semantics.BOUNDED_U64
    bk = rns8.BoundKind.GLOBAL_MAX_ABS if signed else rns8.BoundKind.GLOBAL_MAX_UNSIGNED
    fn = rns8.gemm_i64_oneshot if signed else rns8.gemm_u64_oneshot
    out = np.full((m, n + 2), 7, dt)
    fn(ctx, rns8.gemm_desc(sem, bk, m, n, k, bound=bound), A[:, :k], B[:, :n], out=out[:, :n])
    np.testing.assert_array_equal(out[:, :n], want)
    assert (out[:, n:] == 7).all()
    untouched = np.full((m, n), 9, dt)
    with pytest.raises(rns8.Error) as err:
        fn(ctx, rns8.gemm_desc(sem, bk, m, n, k, bound=bound // 4), A[:, :k], B[:, :n], out=untouched)
    assert err.value.status == rns8.Status.RANGE_ERROR
    assert (untouched == 9).all()


@pytest.mark.parametrize("signed", [True, False])
def test_pipelined_oneshot_with_input_proven_bound(rns8, ctx, signed):
    """When K * max|A| * max|B| <= bound (checked on host threads while the
    copies run), no cell can be a range error, and each row slab of C is
    copied back as soon as it is exported; the result and the padding of a
    strided C are the same as on the checked path."""
    rng = np.random.default_rng(2200 + signed)
    m, n, k = 1100, 64, 8192
    lo = -(2**20) if signed else 0
    dt = np.int64 if signed else np.uint64
    A = rng.integers(lo, 2**20, (m, k + 1), dtype=dt, endpoint=True)
    B = rng.integers(lo, 2**20, (k, n + 3), dtype=dt, endpoint=True)
    want = A[:, :k] @ B[:, :n]
    bound = k * 2**40  # = K * max|A| * max|B| for these ranges
    sem = rns8.Semantics.BOUNDED_I64 if signed else rns8.Semantics.BOUNDED_U64
    bk = rns8.BoundKind.GLOBAL_MAX_ABS if signed else rns8.BoundKind.GLOBAL_MAX_UNSIGNED
    fn = rns8.gemm_i64_oneshot if signed else rns8.gemm_u64_oneshot
    out = np.full((m, n + 2), 5, dt)
    fn(ctx, rns8.gemm_desc(sem, bk, m, n, k, bound=bound), A[:, :k], B[:, :n], out=out[:, :n])
    np.testing.assert_array_equal(out[:, :n], want)
    assert (out[:, n:] == 5).all()


def test_ring_gemm_centered_correction_boundaries(lib, oracle):
    """tests/differential/test_hip_direct_ring_cases.inc:182-211: modulus 255
    (plane 1), A = [1, 1], sums 128, 127, 254 and -128 reduce to the centered
    -127, 127, -1, 127 on the auto (zero-padded tensor-core) and CUDA-core
    paths."""
    a = np.zeros((2, 1, 2), np.int8)
    b = np.zeros((2, 2, 4), np.int8)
    a[1] = [[1, 1]]
    b[1] = [[64, 127, 127, -64], [64, 0, 127, -64]]
    assert oracle.gemm_rns(a, b, 2)[1].ravel().tolist() == [-127, 127, -1, 127]
    for path in (0, 2):
        st, got, word = run_gemm(lib, a, b, 2, path)
        assert st == OK and word == 0 and got[1].ravel().tolist() == [-127, 127, -1, 127], path


def test_ring_gemm_reciprocal_reduction_every_modulus(lib, oracle):
    """tests/differential/test_hip_direct_ring_cases.inc:122-180: the same
    5 x 7 x 67 patterned operands (with +-127, 126 and -128 entries) in all 20
    planes; every plane's reduction equals the oracle's ring GEMM for its
    modulus."""
    m, n, k = 5, 7, 67
    A = np.empty((m, k), np.int8)
    B = np.empty((k, n), np.int8)
    for r in range(m):
        for q in range(k):
            pattern = (r * 37 + q * 19) % 11
            mixed = (r + 113 - (2 * q) % 113) % 113
            A[r, q] = 127 if pattern == 0 else -127 if pattern == 1 else mixed - 56
    for q in range(k):
        for c in range(n):
            pattern = (q * 23 + c * 29) % 13
            B[q, c] = 126 if pattern == 0 else -128 if pattern == 1 else ((3 * q + c) % 127) - 63
    a = np.repeat(A[None], 20, axis=0)
    b = np.repeat(B[None], 20, axis=0)
    st, got, word = run_gemm(lib, a, b, 20, 0)
    assert st == OK and word == 0
    for p, modulus in enumerate(oracle.LADDER[:20]):
        np.testing.assert_array_equal(got[p], oracle.ring_gemm(A, B, modulus), err_msg=f"modulus {modulus}")


@pytest.mark.parametrize("field,modulus", [(False, 255), (False, 256), (True, 251)])
def test_finite_oneshot_patterned_padded(rns8, oracle, ctx, field, modulus):
    """tests/differential/test_hip_direct_finite_native_cases.inc:1-85: 17 x 19
    x 33 patterned bytes with padded lda 40, ldb 23, ldc 29 (pad bytes 0xa5,
    0x5a in the inputs, 0xcc in C) for ring 255, ring 256 and field 251; C
    equals the oracle and its padding keeps 0xcc."""
    m, n, k, lda, ldb, ldc = 17, 19, 33, 40, 23, 29
    A = np.full((m, lda), 0xA5, np.uint8)
    B = np.full((k, ldb), 0x5A, np.uint8)
    for r in range(m):
        for q in range(k):
            A[r, q] = (r * 37 + q * 19 + (r ^ q) * 11) & 0xFF
    for q in range(k):
        for c in range(n):
            B[q, c] = (q * 23 + c * 41 + (q + c) * 7) & 0xFF
    sem = rns8.Semantics.FINITE_FIELD_U8 if field else rns8.Semantics.FINITE_RING_U8
    desc = rns8.gemm_desc(sem, rns8.BoundKind.NONE, m, n, k, finite_modulus=modulus)
    out = np.full((m, ldc), 0xCC, np.uint8)
    rns8.gemm_finite_u8_oneshot(ctx, desc, modulus, A[:, :k], B[:, :n], field, out=out[:, :n])
    st, want = oracle.gemm_finite_u8_oneshot(np.ascontiguousarray(A[:, :k]), np.ascontiguousarray(B[:, :n]),
                                             modulus, field)
    assert st == OK
    np.testing.assert_array_equal(out[:, :n], want)
    assert (out[:, n:] == 0xCC).all()


def test_pipelined_oneshot_output_overlapping_an_input(rns8, ctx):
    """C's host buffer may overlap A's (here C starts at A's row 1024): the
    result is that of the original A even though the inputs prove the bound
    (the overlapping call waits for every upload before writing C)."""
    m, n, k = 2048, 4096, 4096
    rng = np.random.default_rng(77)
    X = np.zeros((m + 1024, k), np.int64)
    X[:m] = rng.integers(-(2**10), 2**10, (m, k), dtype=np.int64, endpoint=True)
    B = rng.integers(-(2**10), 2**10, (k, n), dtype=np.int64, endpoint=True)
    want = (X[:m].astype(np.float64) @ B.astype(np.float64)).astype(np.int64)  # |C| <= 2^32: exact
    desc = rns8.gemm_desc(rns8.Semantics.BOUNDED_I64, rns8.BoundKind.GLOBAL_MAX_ABS, m, n, k, bound=k * 2**20)
    rns8.gemm_i64_oneshot(ctx, desc, X[:m], B, out=X[1024:])
    np.testing.assert_array_equal(X[1024:], want)
