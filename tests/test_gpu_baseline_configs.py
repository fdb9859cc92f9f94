"""BASELINE configs C2-C5 at their configured shapes, through the public C ABI,
on the reference benchmark's seeded inputs (one std::mt19937_64(1) drawing A
then B, uniform_int_distribution over the config's range;
benchmarks/rns8_bench_bounded_i64_lane.inc:11-16, rns8_bench_types.hpp:72),
checked bit for bit against the CPU oracle on sampled rows or tasks, and where
the values allow it against an independent exact product on the GPU (fp64
limb-split matmul) over every cell. The tolerance is zero: this is integer
work."""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

SEED = 1


@pytest.fixture(scope="module")
def ctx(rns8):
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    c = rns8.Context(0)
    yield c
    c.close()


def exact_matmul_fp64(A: np.ndarray, B: np.ndarray, limb_bits: int) -> torch.Tensor:
    """Exact A x B for non-negative or signed operands whose limb products
    summed over K stay below 2^53: each operand split into two limb_bits-bit
    limbs (floor division), four fp64 GEMMs on the GPU, recombined in int64."""
    a = torch.from_numpy(A.view(np.int64)).cuda()
    b = torch.from_numpy(B.view(np.int64)).cuda()
    sh = 1 << limb_bits
    ah, al = torch.div(a, sh, rounding_mode="floor"), torch.remainder(a, sh)
    bh, bl = torch.div(b, sh, rounding_mode="floor"), torch.remainder(b, sh)
    f = lambda x: x.to(torch.float64)
    hh = (f(ah) @ f(bh)).to(torch.int64)
    hl = (f(ah) @ f(bl)).to(torch.int64) + (f(al) @ f(bh)).to(torch.int64)
    ll = (f(al) @ f(bl)).to(torch.int64)
    return hh * (sh * sh) + hl * sh + ll


def test_c3_bounded_i64_8192_oneshot(rns8, oracle, ctx):
    """C3: 8192^3, U[-2^24, 2^24], bound 2^61, prefix 9 forced, through
    rns8_gemm_i64_oneshot; every cell against the exact product, 32 rows
    against the oracle's pack / plane GEMMs / export."""
    m = n = k = 8192
    rng = oracle.Rng(SEED)
    A = rng.i64(-(2**24), 2**24, (m, k))
    B = rng.i64(-(2**24), 2**24, (k, n))
    desc = rns8.gemm_desc(rns8.Semantics.BOUNDED_I64, rns8.BoundKind.GLOBAL_MAX_ABS, m, n, k, bound=2**61,
                          max_prefix=9, flags=rns8.PLAN_FORCE_FIXED_PREFIX)
    got = rns8.gemm_i64_oneshot(ctx, desc, A, B)
    want = exact_matmul_fp64(A, B, 13)  # |limb| <= 2^12: 2^24 * 8192 < 2^53
    assert torch.equal(torch.from_numpy(got).cuda(), want)
    rows = np.linspace(0, m - 1, 32).astype(np.int64)
    planes = oracle.gemm_rns(oracle.pack(np.ascontiguousarray(A[rows]), 9), oracle.pack(B, 9), 9)
    st, ref = oracle.export_i64(planes, 9, 2**61)
    assert st == 0
    np.testing.assert_array_equal(got[rows], ref)


def test_c4_bounded_u64_tall_k(rns8, oracle, ctx):
    """C4: 256 x 256 x 262144, U[0, 2^22), bound 2^62, default prefix (8),
    through rns8_gemm_u64_oneshot (K split across 4 safe blocks of 65536 and
    across CTAs); every cell against the oracle's one-shot and the exact
    product."""
    m = n = 256
    k = 262144
    rng = oracle.Rng(SEED)
    A = rng.u64(0, 2**22 - 1, (m, k))
    B = rng.u64(0, 2**22 - 1, (k, n))
    desc = rns8.gemm_desc(rns8.Semantics.BOUNDED_U64, rns8.BoundKind.GLOBAL_MAX_UNSIGNED, m, n, k, bound=2**62)
    plan = rns8.Plan(ctx, desc)
    assert plan.prefix == 8
    plan.close()
    got = rns8.gemm_u64_oneshot(ctx, desc, A, B)
    st, ref, used = oracle.gemm_bounded_oneshot(A, B, 2**62)
    assert st == 0 and used == 8
    np.testing.assert_array_equal(got, ref)
    want = exact_matmul_fp64(A, B, 11)  # limbs < 2^11: 2^22 * 2^18 = 2^40 < 2^53
    assert torch.equal(torch.from_numpy(got.view(np.int64)).cuda(), want)


def test_c5_exact_wide_signed_4096(rns8, oracle, ctx):
    """C5: 4096^3, full int64 range, EXACT_WIDE_SIGNED with prefix 20 forced,
    3 two's-complement limbs, through the matrix API (pack, rns8_gemm_rns,
    rns8_export_exact_wide_signed_limbs); 64 rows spread over the output
    against the oracle, 16 cells against Python big-int products."""
    m = n = k = 4096
    rng = oracle.Rng(SEED)
    A = rng.i64(-(2**63), 2**63 - 1, (m, k))
    B = rng.i64(-(2**63), 2**63 - 1, (k, n))
    desc = rns8.gemm_desc(rns8.Semantics.EXACT_WIDE_SIGNED, rns8.BoundKind.NONE, m, n, k, max_prefix=20,
                          flags=rns8.PLAN_FORCE_FIXED_PREFIX)
    plan = rns8.Plan(ctx, desc)
    assert plan.prefix == 20
    a, b, c = (rns8.Matrix.for_plan(ctx, plan, r) for r in "abc")
    ws = rns8.Workspace(ctx, plan)
    a.pack_i64(A)
    b.pack_i64(B)
    rns8.gemm_rns(ctx, plan, a, b, c, ws)
    got = rns8.export_exact_wide_limbs(ctx, plan, c, 3, signed=True)
    rows = np.linspace(0, m - 1, 64).astype(np.int64)
    planes = oracle.gemm_rns(oracle.pack(np.ascontiguousarray(A[rows]), 20), oracle.pack(B, 20), 20)
    st, ref = oracle.export_limbs(planes, 20, 3, signed=True)
    assert st == 0
    np.testing.assert_array_equal(got[rows], ref)
    for i in (0, 1, 2047, 4095):
        for j in (0, 5, 3000, 4095):
            exact = sum(int(A[i, t]) * int(B[t, j]) for t in range(k))
            v = sum(int(got[i, j, l]) << (64 * l) for l in range(3))
            assert (v - (1 << 192) if v >> 191 else v) == exact
    for h in (a, b, c, ws, plan):
        h.close()


def test_c2_finite_field_251_batch_64(rns8, oracle, ctx):
    """C2: 64 independent 2048^3 products modulo 251, U[0, 250] drawn per byte
    (uniform_int_distribution<uint32_t>, rns8_bench_finite_lanes.inc:28-31),
    A_t then B_t per task; rns8_pack_finite_u8 x 128, one grouped
    rns8_gemm_finite_u8_grouped call, rns8_export_finite_u8 x 64; four tasks
    against the oracle's one-shot."""
    m = n = k = 2048
    batch = 64
    rng = oracle.Rng(SEED)
    desc = rns8.gemm_desc(rns8.Semantics.FINITE_FIELD_U8, rns8.BoundKind.NONE, m, n, k, finite_modulus=251)
    plan = rns8.Plan(ctx, desc)
    tasks, inputs = [], []
    for _ in range(batch):
        A = rng.u8(250, (m, k))
        B = rng.u8(250, (k, n))
        a, b, c = (rns8.Matrix.for_plan(ctx, plan, r) for r in "abc")
        a.pack_finite_u8(251, A)
        b.pack_finite_u8(251, B)
        tasks.append((a, b, c, rns8.Workspace(ctx, plan)))
        inputs.append((A, B))
    rns8.gemm_finite_u8_grouped(ctx, plan, 251, tasks)
    for t in (0, 21, 42, 63):
        A, B = inputs[t]
        st, want = oracle.gemm_finite_u8_oneshot(A, B, 251, True)
        assert st == 0
        np.testing.assert_array_equal(rns8.export_finite_u8(ctx, plan, 251, tasks[t][2]), want)
    for handles in tasks:
        for h in handles:
            h.close()
    plan.close()
