"""The reference's semantics-validation unit cases
(tests/unit/test_semantics_validation_cases.inc:1-56, 364-451 and
test_semantics_workspace_cases.inc:1-25): bounded plans need a bound kind,
reserved flags are refused, unknown enum values are INVALID_ARGUMENT before
any backend routing (an unknown backend is UNSUPPORTED_BACKEND), tile sizes
are powers of two in [64, 512], and column-major storage is a known but
unsupported contract. Plans are checked on the host (rns8_cuda_plan_probe);
matrix creation needs a context, so those cases run with the GPU tests."""

from __future__ import annotations

import ctypes as C

import pytest

OK, INVALID, UNSUPPORTED = 0, 1, 4
UNKNOWN = 0x7FFF  # an enum value no header defines


@pytest.fixture(scope="module")
def r8():
    import rns8_b200

    rns8_b200.lib()
    return rns8_b200


def gdesc(r8, semantics, bound_kind, backend=None, **kw):
    d = r8.gemm_desc(semantics, bound_kind, 1, 1, 1, bound=kw.pop("bound", 1), **kw)
    if backend is not None:
        d.requested_backend = int(backend)
    return d


def probe(r8, d):
    return r8.api.plan_probe(d)[0]


def test_plan_descriptor_cases(r8):
    S, BK, B = r8.Semantics, r8.BoundKind, r8.Backend
    assert probe(r8, gdesc(r8, S.BOUNDED_I64, BK.NONE)) == INVALID
    assert probe(r8, gdesc(r8, S.BOUNDED_U64, BK.NONE)) == INVALID
    d = gdesc(r8, S.BOUNDED_U64, BK.GLOBAL_MAX_UNSIGNED)
    d.flags = 0x80000000
    assert probe(r8, d) == INVALID                                            # reserved flag
    assert probe(r8, gdesc(r8, S.BOUNDED_U64, UNKNOWN, B.HIPBLASLT)) == INVALID   # enum first
    assert probe(r8, gdesc(r8, UNKNOWN, BK.NONE, B.CK, bound=0)) == INVALID
    assert probe(r8, gdesc(r8, S.BOUNDED_U64, BK.GLOBAL_MAX_UNSIGNED, UNKNOWN)) == UNSUPPORTED
    assert probe(r8, gdesc(r8, S.FINITE_RING_U8, BK.GLOBAL_MAX_UNSIGNED, B.ROCWMMA)) == INVALID


def BOUNDED_KINDS(BK):
    return (BK.GLOBAL_MAX_ABS, BK.GLOBAL_MAX_UNSIGNED, BK.PER_TILE_MAX_ABS, BK.PER_TILE_MAX_UNSIGNED,
            BK.INPUT_RANGE_AND_K)


def test_contract_selection_descriptors(r8):
    """test_semantics_contract_selection_cases.inc:1-111: exact-wide plans
    take BOUND_NONE with no bound, no stray tile bounds (pointer or count),
    and no bounded-looking CRT metadata; wrap64 plans accept none of the
    bounded descriptors either, whichever backend is requested."""
    S, BK, B = r8.Semantics, r8.BoundKind, r8.Backend
    for sem in (S.EXACT_WIDE_SIGNED, S.EXACT_WIDE_UNSIGNED):
        d = r8.gemm_desc(sem, BK.NONE, 1, 1, 1, max_prefix=20)
        assert probe(r8, d) == OK
        d.bound = 1
        assert probe(r8, d) == INVALID
        for bk in BOUNDED_KINDS(BK):
            d = r8.gemm_desc(sem, bk, 1, 1, 1, bound=2**64 - 1, max_prefix=9, requested_backend=B.CPU_REFERENCE)
            assert probe(r8, d) == INVALID
    d = r8.gemm_desc(S.BOUNDED_U64, BK.GLOBAL_MAX_UNSIGNED, 1, 1, 1, bound=1)
    stale = (C.c_uint64 * 1)(100)
    d.tile_bounds = C.cast(stale, C.POINTER(C.c_uint64))
    d.tile_bounds_count = 1
    assert probe(r8, d) == INVALID
    d = r8.gemm_desc(S.EXACT_WIDE_UNSIGNED, BK.NONE, 1, 1, 1, max_prefix=20)
    d.tile_bounds_count = 1
    assert probe(r8, d) == INVALID
    for bk in (BK.NONE, BK.GLOBAL_MAX_UNSIGNED, BK.PER_TILE_MAX_ABS, BK.PER_TILE_MAX_UNSIGNED,
               BK.INPUT_RANGE_AND_K):
        for backend in (B.CPU_REFERENCE, B.WRAP64_BYTE_LIMB):
            d = r8.gemm_desc(S.WRAP_U64_MOD_2_64, bk, 1, 1, 1, bound=2**64 - 1, max_prefix=9,
                             requested_backend=backend)
            assert probe(r8, d) == INVALID


def test_tile_sizes_are_powers_of_two_64_to_512(r8):
    S, BK = r8.Semantics, r8.BoundKind
    assert probe(r8, gdesc(r8, S.BOUNDED_U64, BK.GLOBAL_MAX_UNSIGNED, tile_m=256, tile_n=512)) == OK
    for bad in (32, 96, 513):
        assert probe(r8, gdesc(r8, S.BOUNDED_U64, BK.GLOBAL_MAX_UNSIGNED, tile_m=bad, tile_n=512)) == INVALID


def test_context_options(r8):
    lib = r8.lib()
    opts = r8.abi.ContextOptions(requested_backend=int(r8.Backend.AUTO), flags=1)
    h = C.c_void_p()
    assert lib.rns8_create_context(-1, C.byref(opts), C.byref(h)) == INVALID and not h.value
    opts = r8.abi.ContextOptions(requested_backend=UNKNOWN, flags=0)
    assert lib.rns8_create_context(0, C.byref(opts), C.byref(h)) == UNSUPPORTED and not h.value


@pytest.mark.gpu
def test_matrix_descriptor_cases(r8):
    S, BK, abi = r8.Semantics, r8.BoundKind, r8.abi
    lib = r8.lib()
    with r8.Context(0) as ctx:
        def create(sem, bk, layout=abi.Layout.ROW_MAJOR, flags=0, tile_n=0, max_prefix=0):
            md = abi.MatrixDesc(rows=1, cols=1, logical_ld=1, semantics=int(sem), logical_layout=int(layout),
                                bound_kind=int(bk), tile_n=tile_n, max_prefix=max_prefix, flags=flags)
            h = C.c_void_p()
            st = lib.rns8_create_matrix(ctx.handle, C.byref(md), C.byref(h))
            if h.value:
                lib.rns8_destroy_matrix(h)
            assert st != OK or h.value
            return st, bool(h.value)

        assert create(S.BOUNDED_U64, BK.GLOBAL_MAX_UNSIGNED, flags=1) == (INVALID, False)
        assert create(S.BOUNDED_U64, UNKNOWN) == (INVALID, False)
        assert create(UNKNOWN, BK.NONE) == (INVALID, False)
        assert create(S.BOUNDED_U64, BK.GLOBAL_MAX_UNSIGNED, layout=UNKNOWN) == (INVALID, False)
        assert create(S.EXACT_WIDE_UNSIGNED, BK.GLOBAL_MAX_UNSIGNED, layout=abi.Layout.COLUMN_MAJOR,
                      max_prefix=20) == (INVALID, False)
        assert create(S.BOUNDED_U64, BK.GLOBAL_MAX_UNSIGNED, layout=abi.Layout.COLUMN_MAJOR) == (UNSUPPORTED, False)
        for bad in (32, 96, 513):
            assert create(S.BOUNDED_U64, BK.GLOBAL_MAX_UNSIGNED, tile_n=bad) == (INVALID, False)
        assert create(S.BOUNDED_U64, BK.GLOBAL_MAX_UNSIGNED)[0] == OK
        # test_semantics_contract_selection_cases.inc:1-111: exact-wide storage
        # is unbounded only; bounded-looking exact-wide or wrap64 storage is
        # refused with no handle.
        for sem in (S.EXACT_WIDE_SIGNED, S.EXACT_WIDE_UNSIGNED):
            assert create(sem, BK.NONE, max_prefix=20)[0] == OK
            for bk in BOUNDED_KINDS(BK):
                assert create(sem, bk, max_prefix=9) == (INVALID, False)
        for bk in (BK.NONE, *BOUNDED_KINDS(BK)[1:]):
            assert create(S.WRAP_U64_MOD_2_64, bk, max_prefix=9) == (INVALID, False)


def test_accelerator_backends_fail_fast(r8):
    """test_api_backend_info_cases.inc (context kinds fail fast; malformed
    descriptors fail before unsupported routing): every backend other than
    this library's is UNSUPPORTED_BACKEND at context creation with no
    handle; plan descriptors naming them are INVALID_ARGUMENT when malformed
    (reserved flag, m = 0) and UNSUPPORTED_BACKEND when well formed."""
    S, BK, B = r8.Semantics, r8.BoundKind, r8.Backend
    lib = r8.lib()
    for b in (B.ROCWMMA, B.CK, B.HIPBLASLT, B.AMDGPU_BUILTINS, B.HIP_DIRECT, B.CPU_REFERENCE,
              B.WRAP64_BYTE_LIMB, B.HIP_VECTOR_ALU_INT64):
        opts = r8.abi.ContextOptions(requested_backend=int(b))
        h = C.c_void_p()
        assert lib.rns8_create_context(0, C.byref(opts), C.byref(h)) == UNSUPPORTED and not h.value
    for b in (B.CK, B.ROCWMMA, B.AMDGPU_BUILTINS):
        def d(**kw):
            g = r8.gemm_desc(S.BOUNDED_I64, BK.GLOBAL_MAX_ABS, 1, 1, 1, bound=1, max_prefix=9, requested_backend=b)
            for key, val in kw.items():
                setattr(g, key, val)
            return g
        assert probe(r8, d(flags=0x80000000)) == INVALID
        assert probe(r8, d(m=0)) == INVALID
        assert probe(r8, d()) == UNSUPPORTED
