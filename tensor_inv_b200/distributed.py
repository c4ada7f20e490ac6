"""Sharding of the CRT matmul and of rSVD over ranks (one process per GPU, torch.distributed).

The product shards with no exchange step: row exponents depend only on A's rows and column
exponents only on B's columns (src/tensor_inv/crt_matmul.py:38-44), so the output block
C[rows_i, cols_j] of a pr x pc rank grid is exactly ``crt_matmul(A[rows_i], B[:, cols_j])``,
bit for bit, computed from the rank's own A row panel and B column panel.

Ranks are laid out row-major on the grid: rank r owns grid row r // pc and grid column
r % pc.  Collectives (NCCL over NVLink on GPUs, gloo on CPU) appear only where data has to
move: placing the panels from one rank (``scatter_panels``) and assembling C
(``gather_blocks``).  ``crt_matmul_2d`` itself runs no collective.

A product whose inner dimension is split across ranks (the contractions over the row-sharded
dimension of rSVD, A^T Q and Q^T A) needs a reduction, and it stays exact:
``crt_matmul_sharded_k`` all-reduces the exponents (a max over every rank's slice), splits
each rank's slice with them, all-reduces the int32 residue products (a sum of residues below
ranks * 127, exact) and reconstructs -- bit-identical to ``crt_matmul`` of the whole product
on one GPU.  ``rsvd_rows`` is the reference's randomized SVD (src/tensor_inv/rsvd.py:6-32) with
A's rows sharded, built on it.
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


# ---------------------------------------------------------------------------------------
# products over a sharded inner dimension, and rSVD with A's rows sharded
# ---------------------------------------------------------------------------------------
_NONFINITE_EXP = -(2**31)


def _global_exponents(X, dim, group):
    """frexp exponents of max |X| along `dim` over every rank's slice (the reference's
    ``amax().clamp(min=1e-300).frexp()[1]``, crt_matmul.py:38-44), with the non-finite marker.
    The maxima are all-reduced as int64 bit patterns: for non-negative float64 the integer
    order is the float order, and NaN's pattern lies above inf's, so the max is exact."""
    import torch.distributed as dist

    if X.shape[dim] > 0:
        mx = X.abs().amax(dim=dim).to(torch.float64)
    else:
        mx = torch.zeros(X.shape[1 - dim], dtype=torch.float64, device=X.device)
    bits = mx.contiguous().view(torch.int64).clone()
    dist.all_reduce(bits, op=dist.ReduceOp.MAX, group=group)
    mx = bits.view(torch.float64)
    e = torch.frexp(mx.clamp(min=1e-300))[1].to(torch.int32)
    return torch.where(torch.isfinite(mx), e, torch.full_like(e, _NONFINITE_EXP))


def crt_matmul_sharded_k(A_local, B_local, *, group=None):
    """C = A @ B where this rank holds A's columns and B's matching rows (any split of the
    inner dimension over the ranks of `group`; every rank gets the whole C).

    Bit-identical to ``crt_matmul(A, B)`` of the whole operands with the reference's primes:
    the same exponents (all-reduced), residues, residue products (an exact int32 all-reduce of
    each rank's ``ti_crt_residue_partial``) and reconstruction.  Raises the reference's errors
    (TypeError for the dtype, IndexError for an empty inner dimension, ValueError from
    _n_moduli)."""
    import ctypes

    import torch.distributed as dist

    from tensor_inv_b200 import _native as nat
    from tensor_inv_b200.crt_matmul import _PRIMES, _check_dtype, _n_moduli, _strides_2d

    bits = _check_dtype(A_local)
    if not A_local.is_cuda:
        raise RuntimeError("crt_matmul_sharded_k needs CUDA tensors")
    dev = A_local.device
    m, kl = A_local.shape
    if B_local.shape[0] != kl:
        raise RuntimeError("crt_matmul_sharded_k: shape mismatch")
    n = B_local.shape[1]
    kt = torch.tensor([kl], dtype=torch.int64, device=dev)
    dist.all_reduce(kt, group=group)
    k = int(kt.item())
    if k == 0:
        raise IndexError("crt_matmul_sharded_k: empty inner dimension")
    n_mod = _n_moduli(k, bits)
    A = A_local.to(torch.float64)
    B = B_local.to(torch.float64)
    row_exp = _global_exponents(A, 1, group)
    col_exp = _global_exponents(B, 0, group)
    partial = torch.zeros((n_mod, m, n), dtype=torch.int32, device=dev)
    if kl > 0 and m > 0 and n > 0:
        sa, sb = _strides_2d(A), _strides_2d(B)
        if sa is None:
            A = A.contiguous()
            sa = A.stride()
        if sb is None:
            B = B.contiguous()
            sb = B.stride()
        ws_b = ctypes.c_size_t(0)
        nat.check("ti_crt_residue_partial_workspace_size",
                  nat.lib().ti_crt_residue_partial_workspace_size(m, n, kl, n_mod,
                                                                  ctypes.byref(ws_b)))
        ws = torch.empty(max(ws_b.value, 256), dtype=torch.uint8, device=dev)
        with torch.cuda.device(dev):
            nat.check("ti_crt_residue_partial", nat.lib().ti_crt_residue_partial(
                A.data_ptr(), sa[0], sa[1], B.data_ptr(), sb[0], sb[1], m, n, kl, bits, n_mod,
                row_exp.data_ptr(), col_exp.data_ptr(), partial.data_ptr(), ws.data_ptr(),
                ws.numel(), torch.cuda.current_stream(dev).cuda_stream))
    dist.all_reduce(partial, group=group)
    C = torch.empty((m, n), dtype=torch.float64, device=dev)
    if m > 0 and n > 0:
        mods = (ctypes.c_int32 * n_mod)(*_PRIMES[:n_mod])
        with torch.cuda.device(dev):
            nat.check("ti_crt_reconstruct", nat.lib().ti_crt_reconstruct(
                partial.data_ptr(), ctypes.cast(mods, ctypes.c_void_p), n_mod, bits,
                row_exp.data_ptr(), col_exp.data_ptr(), m, n, C.data_ptr(), n,
                torch.cuda.current_stream(dev).cuda_stream))
    return C


def _row_counts(m_local, group):
    import torch.distributed as dist

    world = dist.get_world_size(group)
    counts = [0] * world
    dist.all_gather_object(counts, int(m_local), group=group)
    return counts


def _gather_rows(X_local, counts, group):
    """All ranks' row blocks stacked in rank order, exactly: each rank writes its rows into a
    zero buffer and the buffers are summed as int64 bit patterns (x + 0 is x for every
    pattern, -0.0 included), which any backend can all-reduce."""
    import torch.distributed as dist

    rank = dist.get_rank(group)
    r0 = sum(counts[:rank])
    full = torch.zeros((sum(counts), X_local.shape[1]), dtype=X_local.dtype, device=X_local.device)
    full[r0:r0 + X_local.shape[0]] = X_local
    bits = full.view(torch.int64)
    dist.all_reduce(bits, group=group)
    return bits.view(X_local.dtype)


def rsvd_rows(A_local, rank, n_oversamples=10, n_power_iter=1, *, group=None):
    """The reference's randomized SVD (rsvd.py:6-32) with A's rows sharded over `group`.

    This rank holds rows [r0, r0 + m_local) of A (ranks in order).  Every rank must have the
    same torch RNG state on entry (Omega is drawn as in the reference).  Returns this rank's
    rows of U, and S and Vt (the same on every rank).  Products whose inner dimension is the
    row dimension (A^T Q, Q^T A) go through crt_matmul_sharded_k; the others are row-local;
    the QR factorisations run on the gathered (m x r) matrices.  Every value is bit-identical
    to ``rsvd`` of the whole A on one GPU.
    """
    import torch.distributed as dist

    from tensor_inv_b200.rsvd import _mm

    m_local, n = A_local.shape
    r = rank + n_oversamples
    counts = _row_counts(m_local, group)
    r0 = sum(counts[:dist.get_rank(group)])

    # random projection (rsvd.py:18-20)
    Omega = torch.randn(n, r, dtype=A_local.dtype, device=A_local.device)
    Y = _gather_rows(_mm(A_local, Omega), counts, group)
    Q, _ = torch.linalg.qr(Y)

    # power iterations (rsvd.py:23-25)
    for _ in range(n_power_iter):
        Q_local = Q[r0:r0 + m_local]
        Z = crt_matmul_sharded_k(A_local.T, Q_local, group=group)
        Y = _gather_rows(_mm(A_local, Z), counts, group)
        Q, _ = torch.linalg.qr(Y)

    # project to the low-rank subspace (rsvd.py:28-30)
    Q_local = Q[r0:r0 + m_local]
    B = crt_matmul_sharded_k(Q_local.T, A_local, group=group)
    Ub, S, Vt = torch.linalg.svd(B, full_matrices=False)
    U_local = _mm(Q_local, Ub)

    return U_local[:, :rank], S[:rank], Vt[:rank]
