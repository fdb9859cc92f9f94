"""Row-slab sharding of the RNS8 GEMM across GPUs (one process per GPU).

Output rows are independent: rank r of `world` computes rows
[row0, row0 + rows) of C from the same rows of A and all of B, with no
exchange between ranks: output row slabs are independent units.
The split is as even as possible; earlier ranks take the remainder rows.
"""

from __future__ import annotations


def row_slab(rank: int, world: int, m: int) -> tuple[int, int]:
    """(first row, row count) of rank's slab of an m-row output."""
    if world <= 0 or not 0 <= rank < world or m < 0:
        raise ValueError("need 0 <= rank < world and m >= 0")
    base, extra = divmod(m, world)
    rows = base + (1 if rank < extra else 0)
    row0 = rank * base + min(rank, extra)
    return row0, rows


def gemm_i64_row_sharded(ctx, desc, A, B, rank: int, world: int, out=None):
    """This rank's slab of C = A x B through rns8_gemm_i64_oneshot.

    A and B are this process's host arrays (A may be the full matrix or just
    the slab); desc describes the full problem. Returns (row0, C_slab)."""
    import numpy as np

    from . import api

    row0, rows = row_slab(rank, world, desc.m)
    if rows == 0:
        return row0, np.zeros((0, desc.n), np.int64)
    a = A[row0 : row0 + rows] if A.shape[0] == desc.m else A
    d = api.gemm_desc(desc.semantics, desc.bound_kind, rows, desc.n, desc.k, bound=desc.bound,
                      max_prefix=desc.max_prefix, flags=desc.flags, lhs_bound=desc.lhs_bound, rhs_bound=desc.rhs_bound)
    return row0, api.gemm_i64_oneshot(ctx, d, a, B, out=out)
