"""2-D sharding of the CRT matmul over ranks (one process per GPU, torch.distributed).

The product shards with no exchange step: row exponents depend only on A's rows and column
exponents only on B's columns (src/tensor_inv/crt_matmul.py:38-44), so the output block
C[rows_i, cols_j] of a pr x pc rank grid is exactly ``crt_matmul(A[rows_i], B[:, cols_j])``,
bit for bit, computed from the rank's own A row panel and B column panel.

Ranks are laid out row-major on the grid: rank r owns grid row r // pc and grid column
r % pc.  Collectives (NCCL over NVLink on GPUs, gloo on CPU) appear only where data has to
move: placing the panels from one rank (``scatter_panels``) and assembling C
(``gather_blocks``).  ``crt_matmul_2d`` itself runs no collective.
"""

from __future__ import annotations

import math

import torch


def grid_shape(world: int) -> tuple[int, int]:
    """pr x pc with pr <= pc as square as possible: 1x1, 1x2, 2x2, 2x4, 3x3, ..."""
    pr = int(math.isqrt(world))
    while world % pr:
        pr -= 1
    return pr, world // pr


def block_range(size: int, parts: int, index: int, align: int = 128) -> tuple[int, int]:
    """[start, stop) of block `index` when `size` is cut into `parts` contiguous blocks whose
    boundaries fall on multiples of `align` (whole GEMM tiles) wherever the size allows."""
    if not 0 <= index < parts:
        raise IndexError(index)
    units = -(-size // align)
    base, extra = divmod(units, parts)
    start_u = index * base + min(index, extra)
    stop_u = start_u + base + (1 if index < extra else 0)
    return min(size, start_u * align), min(size, stop_u * align)


def grid_coords(rank: int, world: int) -> tuple[int, int]:
    pr, pc = grid_shape(world)
    return rank // pc, rank % pc


def my_ranges(m: int, n: int, rank: int, world: int):
    """(row range, column range) of the C block owned by `rank`."""
    pr, pc = grid_shape(world)
    i, j = grid_coords(rank, world)
    return block_range(m, pr, i), block_range(n, pc, j)


def crt_matmul_2d(A_panel, B_panel, *, matmul=None, moduli=None, n_moduli=None):
    """This rank's block of C = A @ B from its A row panel and B column panel (no
    collective).  ``matmul`` defaults to :func:`tensor_inv_b200.crt_matmul`."""
    if matmul is None:
        from tensor_inv_b200.crt_matmul import crt_matmul

        return crt_matmul(A_panel, B_panel, moduli=moduli, n_moduli=n_moduli)
    return matmul(A_panel, B_panel)


def scatter_panels(A, B, m: int, n: int, k: int, *, src: int = 0, group=None,
                   device=None, dtype=torch.float64):
    """Place panels from rank `src`: every rank receives its A row panel (rows of its grid
    row, all k columns) and its B column panel (all k rows, columns of its grid column).

    A and B are only read on `src` (others may pass None).  Uses one broadcast per grid row
    and per grid column from `src` (NCCL over NVLink on GPUs); returns (A_panel, B_panel).
    """
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    pr, pc = grid_shape(world)
    me_i, me_j = grid_coords(rank, world)
    dev = device if device is not None else (A.device if A is not None else torch.device("cpu"))
    A_panel = B_panel = None
    for i in range(pr):
        r0, r1 = block_range(m, pr, i)
        buf = (A[r0:r1].to(device=dev, dtype=dtype).contiguous() if rank == src
               else torch.empty((r1 - r0, k), dtype=dtype, device=dev))
        dist.broadcast(buf, src, group=group)
        if i == me_i:
            A_panel = buf
    for j in range(pc):
        c0, c1 = block_range(n, pc, j)
        buf = (B[:, c0:c1].to(device=dev, dtype=dtype).contiguous() if rank == src
               else torch.empty((k, c1 - c0), dtype=dtype, device=dev))
        dist.broadcast(buf, src, group=group)
        if j == me_j:
            B_panel = buf
    return A_panel, B_panel


def gather_blocks(C_block, m: int, n: int, *, group=None):
    """All-gather every rank's C block into the full m x n C on every rank."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    dev, dtype = C_block.device, C_block.dtype
    ranges = [my_ranges(m, n, r, world) for r in range(world)]
    # all_gather moves equal-size tensors: pad every block to the largest block's shape
    hr = max(r1 - r0 for (r0, r1), _ in ranges)
    hc = max(c1 - c0 for _, (c0, c1) in ranges)
    mine = torch.zeros((hr, hc), dtype=dtype, device=dev)
    mine[:C_block.shape[0], :C_block.shape[1]] = C_block
    blocks = [torch.empty((hr, hc), dtype=dtype, device=dev) for _ in range(world)]
    dist.all_gather(blocks, mine, group=group)
    C = torch.empty((m, n), dtype=dtype, device=dev)
    for blk, ((r0, r1), (c0, c1)) in zip(blocks, ranges):
        C[r0:r1, c0:c1] = blk[:r1 - r0, :c1 - c0]
    return C
