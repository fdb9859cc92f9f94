"""Sharding of the RNS8 GEMM across GPUs (one process per GPU).

Output rows are independent: rank r of `world` computes rows
[row0, row0 + rows) of C from the same rows of A and all of B, with no
exchange between ranks: output row slabs are independent units.
The split is as even as possible; earlier ranks take the remainder rows.
The 2-D partition (output_tile) also splits the columns, so that each rank
packs a column slab of B instead of all of it.
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


def grid_shape(world: int) -> tuple[int, int]:
    """(row_groups, col_groups) of the 2-D output partition: the factor pair of
    world closest to square, with at least as many row groups as column
    groups (1 -> 1x1, 2 -> 2x1, 4 -> 2x2, 8 -> 4x2)."""
    if world <= 0:
        raise ValueError("need world >= 1")
    cols = max(c for c in range(1, int(world**0.5) + 1) if world % c == 0)
    return world // cols, cols


def output_tile(rank: int, world: int, m: int, n: int) -> tuple[int, int, int, int]:
    """(row0, rows, col0, cols) of rank's block of an m x n output under the
    2-D partition: rank = i * col_groups + j owns row slab i of A and C and
    column slab j of B and C, so it packs only its own slabs and no rank
    exchanges anything."""
    r, c = grid_shape(world)
    if not 0 <= rank < world:
        raise ValueError("need 0 <= rank < world")
    row0, rows = row_slab(rank // c, r, m)
    col0, cols = row_slab(rank % c, c, n)
    return row0, rows, col0, cols


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


def gemm_i64_block_sharded(ctx, desc, A, B, rank: int, world: int, out=None):
    """This rank's block of C = A x B under the 2-D partition (output_tile),
    through rns8_gemm_i64_oneshot on the rank's row slab of A and column slab
    of B (a strided view: the one-shot reads it in place with ldb = n).

    A and B are the full host arrays; desc describes the full problem.
    Returns (row0, col0, C_block)."""
    import numpy as np

    from . import api

    row0, rows, col0, cols = output_tile(rank, world, desc.m, desc.n)
    if rows == 0 or cols == 0:
        return row0, col0, np.zeros((rows, cols), np.int64)
    d = api.gemm_desc(desc.semantics, desc.bound_kind, rows, cols, desc.k, bound=desc.bound,
                      max_prefix=desc.max_prefix, flags=desc.flags, lhs_bound=desc.lhs_bound, rhs_bound=desc.rhs_bound)
    return row0, col0, api.gemm_i64_oneshot(ctx, d, A[row0:row0 + rows], B[:, col0:col0 + cols], out=out)


# ---- plane sharding ---------------------------------------------------------------
# The alternative split for wide prefixes: rank r computes the residue planes
# {p : p mod world == r} of ALL of C, then the planes are exchanged so that
# every rank holds all planes of its own row slab of C and reconstructs it.
# The exchange is fused into the plane GEMM (rns8_cuda_gemm_rns_slabs_device):
# its epilogue stores each output row into the owning rank's receive buffer,
# mapped into this process through CUDA IPC.

TILE_ROWS = 128  # rows of one plane-GEMM output tile


def planes_of_rank(rank: int, world: int, prefix: int) -> list[int]:
    """Ladder indices of the planes rank computes (round robin)."""
    if world <= 0 or not 0 <= rank < world or not 1 <= prefix <= 20:
        raise ValueError("need 0 <= rank < world and 1 <= prefix <= 20")
    return [p for p in range(prefix) if p % world == rank]


def plane_slabs(m: int, world: int) -> tuple[int, int]:
    """(slab_rows, slab_count) of the exchange: slabs of whole output tiles,
    as even as tiles allow; slab s (s < slab_count) belongs to rank s, and
    ranks at or above slab_count own no rows (they only compute planes)."""
    if world <= 0 or world > 8 or m <= 0:
        raise ValueError("need 1 <= world <= 8 and m > 0")
    per = -(-m // world)
    slab_rows = -(-per // TILE_ROWS) * TILE_ROWS
    return slab_rows, -(-m // slab_rows)


def slab_of_rank(rank: int, m: int, world: int) -> tuple[int, int]:
    """(first row, row count) of rank's slab under plane_slabs (count 0: none)."""
    slab_rows, count = plane_slabs(m, world)
    if rank >= count:
        return m, 0
    row0 = rank * slab_rows
    return row0, min(slab_rows, m - row0)


class LibraryIpc:
    """CUDA IPC through the library: allocate, export, open, close, free."""

    HANDLE_BYTES = 64

    def __init__(self, lib, device: int):
        self.lib, self.device = lib, device

    def alloc(self, nbytes: int) -> tuple[int, bytes]:
        import ctypes as C

        ptr, handle = C.c_void_p(), (C.c_uint8 * self.HANDLE_BYTES)()
        st = self.lib.rns8_cuda_ipc_alloc(self.device, nbytes, C.byref(ptr), handle)
        if st != 0:
            raise RuntimeError(f"rns8_cuda_ipc_alloc failed with status {st}")
        return ptr.value, bytes(handle)

    def open(self, handle: bytes) -> int:
        import ctypes as C

        ptr = C.c_void_p()
        buf = (C.c_uint8 * self.HANDLE_BYTES).from_buffer_copy(handle)
        st = self.lib.rns8_cuda_ipc_open(self.device, buf, C.byref(ptr))
        if st != 0:
            raise RuntimeError(f"rns8_cuda_ipc_open failed with status {st}")
        return ptr.value

    def close(self, ptr: int) -> None:
        self.lib.rns8_cuda_ipc_close(self.device, ptr)

    def free(self, ptr: int) -> None:
        self.lib.rns8_cuda_ipc_free(self.device, ptr)


class PlaneExchange:
    """Receive buffers of the plane exchange and every rank's view of them.

    Each rank owning rows allocates `buffers` receive buffers of
    prefix x rows x n bytes (all planes of its slab; two let step i+1's GEMM
    write while step i's export still reads). Handles are all-gathered over
    torch.distributed, and each rank opens the others' buffers, so that
    slab_table(b)[s] is rank s's buffer b as seen from this process.
    `ipc` is LibraryIpc or a stand-in with the same methods."""

    def __init__(self, ipc, rank: int, world: int, m: int, n: int, prefix: int, buffers: int = 2, group=None):
        import torch.distributed as dist  # the handle exchange (not used for world == 1)

        self.ipc, self.rank, self.world = ipc, rank, world
        self.slab_rows, self.slab_count = plane_slabs(m, world)
        self.row0, self.rows = slab_of_rank(rank, m, world)
        self.own: list[int] = []
        handles: list[bytes | None] = []
        for _ in range(buffers):
            if self.rows:
                ptr, h = ipc.alloc(prefix * self.rows * n)
                self.own.append(ptr)
                handles.append(h)
            else:
                handles.append(None)
        everyone: list = [None] * world
        if world == 1:
            everyone[0] = handles
        else:
            dist.all_gather_object(everyone, handles, group=group)
        self.opened: list[int] = []
        self.tables: list[list[int]] = []
        for b in range(buffers):
            table = []
            for s in range(self.slab_count):
                if s == rank:
                    table.append(self.own[b])
                else:
                    ptr = ipc.open(everyone[s][b])
                    self.opened.append(ptr)
                    table.append(ptr)
            self.tables.append(table)

    def slab_table(self, b: int) -> list[int]:
        return self.tables[b]

    def receive_buffer(self, b: int) -> int | None:
        return self.own[b] if self.rows else None

    def close(self) -> None:
        for ptr in self.opened:
            self.ipc.close(ptr)
        for ptr in self.own:
            self.ipc.free(ptr)
        self.opened, self.own, self.tables = [], [], []
