"""Sharding of the CRT matmul and of rSVD over ranks (one process per GPU, torch.distributed).

The product shards with no exchange step: row exponents depend only on A's rows and column
exponents only on B's columns (src/tensor_inv/crt_matmul.py:32-38), so the output block
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

import importlib
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


def grid_groups(group=None, shape=None):
    """(row groups, column groups) of the pr x pc rank grid (``shape``, default
    ``grid_shape``): ``row[i]`` holds the ranks of grid row i, ``col[j]`` those of grid column
    j, rank r at (r // pc, r % pc).  Every rank must call this (it creates process groups, in
    the same order on every rank)."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    pr, pc = shape if shape is not None else grid_shape(world)
    if pr * pc != world:
        raise ValueError(f"grid {pr}x{pc} does not hold {world} ranks")
    glob = [_global_rank(group, r) for r in range(world)]
    rows = [dist.new_group([glob[i * pc + j] for j in range(pc)]) for i in range(pr)]
    cols = [dist.new_group([glob[i * pc + j] for i in range(pr)]) for j in range(pc)]
    return rows, cols


def crt_matmul_grid_host(A_slices, B_slice, *, row_group, col_group, out=None, moduli=None,
                         n_moduli=None, matmul=None, device=None):
    """This rank's block C = A_panel @ B_panel of a product whose operands are in host memory,
    each byte held by exactly one rank of the grid: the ranks of a grid row share its A row
    panel and those of a grid column its B column panel, so every operand byte crosses PCIe
    once and reaches the other ranks that need it over NVLink.

    A_slices (bands, r, k): this rank's share of its A row panel, which is cut into `bands`
    row bands of q*r rows (q the ranks of the grid row); band b of the panel is the rows
    ``A_slices[b]`` of the row's ranks in group order.  B_slice (k/p, n_b): this rank's rows
    of its B column panel (p the ranks of the grid column, rows in group order).  Returns the
    (bands*q*r) x n_b block in host memory (``out`` if given, else pinned).

    On CUDA each band's A rows are copied in and all-gathered over the grid row (NCCL), its
    block of C is computed (``crt_matmul``, bit-identical to the product of the whole panels:
    row exponents depend on their row only) and copied out while later bands arrive; the B
    panel is gathered first (its column exponents need every row).  Synchronous: returns once
    C is in host memory.  ``matmul`` replaces the product (CPU tests)."""
    import torch.distributed as dist

    from tensor_inv_b200.crt_matmul import crt_matmul

    bands, r, k = A_slices.shape
    q = dist.get_world_size(row_group)
    p = dist.get_world_size(col_group)
    if B_slice.shape[0] * p != k:
        raise RuntimeError("crt_matmul_grid_host: B slices do not cover k")
    n_b = B_slice.shape[1]
    rows = q * r
    dev = torch.device(device) if device is not None else (
        torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available()
        else torch.device("cpu"))
    cuda = dev.type == "cuda"
    if out is None:
        out = torch.empty((bands * rows, n_b), dtype=torch.float64, pin_memory=cuda)

    def product(a, b_):
        if matmul is not None:
            return matmul(a, b_)
        return crt_matmul(a, b_, moduli=moduli, n_moduli=n_moduli)

    if not cuda:  # gloo ranks on the host: the same data flow, in order
        B = torch.empty((k, n_b), dtype=torch.float64)
        dist.all_gather_into_tensor(B, B_slice.to(torch.float64).contiguous(), group=col_group)
        for b in range(bands):
            Ab = torch.empty((rows, k), dtype=torch.float64)
            dist.all_gather_into_tensor(Ab, A_slices[b].to(torch.float64).contiguous(),
                                        group=row_group)
            out[b * rows:(b + 1) * rows] = product(Ab, B)
        return out

    compute = torch.cuda.current_stream(dev)
    h2d = torch.cuda.Stream(dev)      # PCIe in: B's rows, then the A bands, never waiting
    gather = torch.cuda.Stream(dev)   # NCCL: B's gather, then the A bands' gathers, in order
    d2h = torch.cuda.Stream(dev)      # PCIe out: each band of C as soon as it is computed
    h2d.wait_stream(compute)
    gather.wait_stream(compute)

    def copied(src):
        with torch.cuda.stream(h2d):
            t = src.to(dev, torch.float64, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(h2d)
        return t, ev

    B_part, ev_b = copied(B_slice)
    parts = [copied(A_slices[b]) for b in range(bands)]
    with torch.cuda.stream(gather):
        B = torch.empty((k, n_b), dtype=torch.float64, device=dev)
        gather.wait_event(ev_b)
        # one order of collectives on every rank: B's gather completes before the A bands'
        dist.all_gather_into_tensor(B, B_part, group=col_group, async_op=True).wait()
        b_in = torch.cuda.Event()
        b_in.record(gather)
        panels, works = [], []
        for b in range(bands):
            gather.wait_event(parts[b][1])
            panels.append(torch.empty((rows, k), dtype=torch.float64, device=dev))
            works.append(dist.all_gather_into_tensor(panels[b], parts[b][0], group=row_group,
                                                     async_op=True))
    compute.wait_event(b_in)  # B is in (the band gathers are waited on one by one)
    for b in range(bands):
        works[b].wait()  # the compute stream waits for band b's gather
        Cb = product(panels[b], B)
        done = torch.cuda.Event()
        done.record(compute)
        d2h.wait_event(done)
        with torch.cuda.stream(d2h):
            out[b * rows:(b + 1) * rows].copy_(Cb, non_blocking=True)
            Cb.record_stream(d2h)
    d2h.synchronize()
    # every side-stream buffer is done: h2d -> gather -> compute -> d2h, and d2h has finished
    return out


# ---------------------------------------------------------------------------------------
# products over a sharded inner dimension, and rSVD with A's rows sharded
# ---------------------------------------------------------------------------------------
_NONFINITE_EXP = -(2**31)


def _global_exponents(X, dim, group):
    """frexp exponents of max |X| along `dim` over every rank's slice (the reference's
    ``amax().clamp(min=1e-300).frexp()[1]``, crt_matmul.py:32-38), with the non-finite marker.
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
    # every rank sees the same total, so every rank raises together: the whole product's
    # inner dimension has the single-GPU bound (the sum of the ranks' planes would stay exact
    # beyond it, but crt_matmul of the whole product raises there, and so does this)
    if k > nat.TI_MAX_K:
        raise ValueError(f"inner dim {k} exceeds {nat.TI_MAX_K}, the bound that keeps the int32 "
                         f"residue accumulators exact for moduli 'primes'")
    n_mod = _n_moduli(k, bits)
    if not A_local.is_cuda:
        raise RuntimeError("crt_matmul_sharded_k needs CUDA tensors")
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


# ---------------------------------------------------------------------------------------
# Block-cyclic LU and Cholesky: block column c (columns [c*b, c*b + b)) lives on rank
# c % world.  Each step broadcasts the panel from its owner and updates every rank's own
# trailing columns, so the results are bit-identical to ``lu`` / ``cholesky`` on one GPU.
# ---------------------------------------------------------------------------------------
def cyclic_blocks(n: int, block_size: int, rank: int, world: int) -> list[int]:
    """Block-column indices owned by `rank` when block c goes to rank c % world."""
    return list(range(rank, -(-n // block_size), world))


def cyclic_columns(n: int, block_size: int, rank: int, world: int) -> torch.Tensor:
    """Global column indices held by `rank`, in the order of its local columns."""
    cols = [torch.arange(c * block_size, min(n, (c + 1) * block_size))
            for c in cyclic_blocks(n, block_size, rank, world)]
    return torch.cat(cols) if cols else torch.zeros(0, dtype=torch.long)


def _exact_sum_(X, group):
    """All-reduce of a float64 tensor in which every element is nonzero on at most one rank:
    summing the int64 bit patterns (x + 0 is x for every pattern) copies each value exactly."""
    import torch.distributed as dist

    dist.all_reduce(X.view(torch.int64), group=group)
    return X


def _global_rank(group, rank):
    import torch.distributed as dist

    return rank if group is None else dist.get_global_rank(group, rank)


def _panel_torch_cols(W, piv, j, jb, pc):
    """The reference's unblocked panel (lu.py:24-34) with the panel's column k held in W's
    column pc + k - j; row swaps exchange all of W's columns."""
    c1 = pc + jb - j
    for k in range(j, jb):
        ck = pc + k - j
        max_idx = W[k:, ck].abs().argmax() + k
        if max_idx != k:
            W[k], W[max_idx] = W[max_idx].clone(), W[k].clone()
            piv[k], piv[max_idx] = piv[max_idx].clone(), piv[k].clone()

        if W[k, ck].abs() > 1e-15:
            W[k + 1:, ck] /= W[k, ck]
            W[k + 1:, ck + 1:c1] -= W[k + 1:, ck:ck + 1] @ W[k:k + 1, ck + 1:c1]


def _trailing_update(Wv, A, B, k, matmul, lower=False):
    """Wv -= A @ B through the CRT kernels (fused into the reconstruction on CUDA), or through
    `matmul` when given."""
    from tensor_inv_b200.crt_matmul import caller_moduli, crt_matmul, crt_matmul_update

    if matmul is not None:
        Wv -= matmul(A, B)
    elif Wv.is_cuda and Wv.dtype == torch.float64 and Wv.stride(1) == 1:
        crt_matmul_update(Wv, A, B, alpha=-1, moduli=caller_moduli(k), lower=lower)
    else:
        Wv -= crt_matmul(A, B, moduli=caller_moduli(k))


def _inverse_perm(piv):
    """pos with pos[piv[i]] = i: the current position of each original row."""
    pos = torch.empty_like(piv)
    pos[piv] = torch.arange(piv.numel(), device=piv.device)
    return pos


def _apply_row_perm_(W, piv, new_piv, j, max_moved):
    """Reorder W's rows from the order `piv` to `new_piv` (both list the original row at each
    position), moving only the rows whose position changed: at most `max_moved` (a panel's
    swaps touch its own rows and the rows they were exchanged with).  No host round trip."""
    src = _inverse_perm(piv)[new_piv]
    moved = src != torch.arange(src.numel(), device=src.device)
    idx = torch.nonzero_static(moved, size=max_moved, fill_value=j).flatten()
    W[idx] = W[src[idx]]  # the right side is gathered before any row is written


def _post_broadcast(tensors, src, group, world):
    """Asynchronous broadcasts from `src` (none with one rank); returns the works to wait on."""
    import torch.distributed as dist

    if world == 1:
        return []
    return [dist.broadcast(t, src=src, group=group, async_op=True) for t in tensors]


def lu_cyclic(W_local, n: int, block_size: int = 64, *, group=None, matmul=None):
    """Blocked LU with partial pivoting (lu.py:6-54) on block-cyclic columns, with one step of
    look-ahead.

    W_local holds this rank's block columns of the n x n matrix (``cyclic_columns``), all n
    rows.  Per block column c: the pivot vector and the panel (factorised by the owner with
    row swaps across its local columns: ``ti_lu_panel_ex`` on CUDA float64, else the
    reference's torch loop) are broadcast and the other ranks apply the same row permutation
    to their columns (only the rows that moved).  Each rank solves the U block row at its full
    width with the other ranks' columns zero (the reference's call on the same shape; a
    column's solution depends only on that column and L, so its own columns carry the
    whole-row solve's bits, and no exchange is needed).  Look-ahead: the owner of block c + 1 updates that block first, factorises it and
    posts its broadcast before its remaining update of step c, so the next panel is
    factorised while the other ranks update; its remaining update then uses L21's rows in the
    new panel's row order (each entry of W still meets the same row of L21).  Every trailing
    update is a column subset of the reference's product, which the CRT kernels compute bit
    for bit (column exponents depend on their column only).  Returns this rank's factored
    columns and the pivot vector (the same on every rank)."""
    import torch.distributed as dist

    rank, world = dist.get_rank(group), dist.get_world_size(group)
    b = block_size
    nb = -(-n // b)
    W = W_local.clone()
    dev = W.device
    mine = cyclic_blocks(n, b, rank, world)
    local_off = {c: i * b for i, c in enumerate(mine)}
    # global column of each local column, on the device once (no host copies in the loop,
    # which would make the host wait for the queued work and end the overlap)
    gcol = cyclic_columns(n, b, rank, world).to(dev)
    piv = torch.arange(n, device=dev)
    lu_mod = importlib.import_module("tensor_inv_b200.lu")  # the module, not the function
    device_panel = W.is_cuda and W.dtype == torch.float64 and not lu_mod._TORCH_PANEL
    if device_panel:
        from tensor_inv_b200 import _native as nat

        ws = torch.empty(nat.lu_panel_workspace_size(), dtype=torch.uint8, device=dev)
        stream = torch.cuda.current_stream(dev)

    def width(c):
        return min(b, n - c * b)

    def factor(c):
        """The owner's panel of block c; returns the broadcast buffers (panel, pivots)."""
        nonlocal piv
        j, bw = c * b, width(c)
        lc = local_off[c]
        if device_panel and bw <= 1024:
            nat.lu_panel_cols(W, j, j + bw, lc, piv, ws, stream)
        else:
            _panel_torch_cols(W, piv, j, j + bw, lc)
        return W[j:, lc:lc + bw].contiguous(), piv.clone()

    def post(c, bufs):
        owner = c % world
        if bufs is None:  # receivers
            bufs = (torch.empty((n - c * b, width(c)), dtype=W.dtype, device=dev),
                    torch.empty_like(piv))
        return bufs, _post_broadcast([bufs[1], bufs[0]], _global_rank(group, 0 if world == 1
                                                                       else owner), group, world)

    pending = post(0, factor(0) if rank == 0 else None)
    for c in range(nb):
        (panel, new_piv), works = pending
        for w in works:
            w.wait()
        j, bw = c * b, width(c)
        jb = j + bw
        owner = c % world
        if rank != owner:
            # the owner's row swaps, as one permutation of rows j.. (piv moved with the rows)
            _apply_row_perm_(W, piv, new_piv, j, 2 * bw)
            piv = new_piv
        if jb >= n:
            break
        L_panel = torch.tril(panel[:bw], diagonal=-1) + torch.eye(bw, dtype=W.dtype, device=dev)
        later = [c2 for c2 in mine if c2 > c]
        row = torch.zeros((bw, n - jb), dtype=W.dtype, device=dev)
        if later:
            lo = local_off[later[0]]
            gcols = gcol[lo:] - jb
            row[:, gcols] = W[j:jb, lo:]
        # triangular solve for the U block row (lu.py:38-43): the reference's call on the whole
        # block row's shape, with the other ranks' columns zero.  Each column of the solution
        # depends only on its own column and L (the same call on the same shape), so this
        # rank's columns carry the bits of the whole-row solve, with no exchange
        U = torch.linalg.solve_triangular(L_panel, row, upper=False)
        L21 = panel[bw:]
        c1 = c + 1
        next_bufs = None
        if later:
            U_mine = U[:, gcols]
            W[j:jb, lo:] = U_mine
            if later[0] == c1:
                # look-ahead: block c + 1 first (lu.py:46 restricted to its columns), then its
                # panel, whose broadcast is posted before the rest of this update
                w1 = width(c1)
                _trailing_update(W[jb:, lo:lo + w1], L21, U_mine[:, :w1], bw, matmul)
                pos_before = _inverse_perm(piv)
                next_bufs = factor(c1)
                L21 = L21[pos_before[piv[jb:]] - jb]  # L21's rows in the new row order
                lo, U_mine = lo + w1, U_mine[:, w1:]
        pending = post(c1, next_bufs)
        if later and U_mine.shape[1]:
            # trailing update of this rank's remaining columns (lu.py:46)
            _trailing_update(W[jb:, lo:], L21, U_mine, bw, matmul)
    return W, piv


def lu_distributed(A, block_size: int = 64, *, group=None, matmul=None):
    """``lu(A, block_size)`` computed block-cyclically over the ranks of `group`; every rank
    passes the same A and gets the same P, L, U as one GPU's ``lu``, bit for bit."""
    import torch.distributed as dist

    if A.shape[0] != A.shape[1]:
        raise ValueError(f"expected square matrix, got {A.shape}")
    n = A.shape[0]
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    cols = cyclic_columns(n, block_size, rank, world).to(A.device)
    W_local, piv = lu_cyclic(A[:, cols].contiguous(), n, block_size, group=group,
                             matmul=matmul)
    W = torch.zeros((n, n), dtype=A.dtype, device=A.device)
    W[:, cols] = W_local
    _exact_sum_(W, group)
    L = torch.tril(W, diagonal=-1) + torch.eye(n, dtype=A.dtype, device=A.device)
    U = torch.triu(W)
    P = torch.zeros(n, n, dtype=A.dtype, device=A.device)
    P[torch.arange(n, device=A.device), piv] = 1.0
    return P, L, U


def _contiguous_runs(blocks, parts):
    """`blocks` (ascending) cut into at most `parts` runs of consecutive entries."""
    if not blocks:
        return []
    parts = max(1, min(parts, len(blocks)))
    size = -(-len(blocks) // parts)
    return [blocks[i:i + size] for i in range(0, len(blocks), size)]


def cholesky_cyclic(A_local, n: int, block_size: int = 64, *, group=None, matmul=None,
                    update_parts: int = 4):
    """Blocked right-looking Cholesky (cholesky.py:6-35) on block-cyclic columns, with one step
    of look-ahead.

    The owner of a block column computes its diagonal block's Cholesky factor
    (``torch.linalg.cholesky_ex``: the reference's factorisation without a host round trip
    per block) and the panel below it (the reference's triangular solve), and broadcasts the
    panel with the block's error code.  Every rank updates its own trailing columns,
    W[:, cols] -= L21 @ L21[cols]^T, only from each column's diagonal block down (the rows the
    factorisation reads again), in up to `update_parts` pieces of consecutive local blocks,
    each from its first block's diagonal down.  Look-ahead: the owner of block c + 1 updates
    that block first, factorises it and posts its broadcast before the rest of its update
    of step c.  The factor is the reference's bit for bit; the error codes are checked once
    at the end, and every rank raises the error the first failing block gives
    ``torch.linalg.cholesky``.  Returns this rank's columns of L."""
    import torch.distributed as dist

    from tensor_inv_b200.cholesky import _raise_first_failure

    rank, world = dist.get_rank(group), dist.get_world_size(group)
    b = block_size
    nb = -(-n // b)
    W = A_local.clone()
    L = torch.zeros_like(W)
    dev = W.device
    mine = cyclic_blocks(n, b, rank, world)
    local_off = {c: i * b for i, c in enumerate(mine)}
    gcol = cyclic_columns(n, b, rank, world).to(dev)  # global column of each local column
    infos = []

    def width(c):
        return min(b, n - c * b)

    def factor(c):
        """The owner's diagonal block and panel of block c; returns the broadcast buffers."""
        j, bw = c * b, width(c)
        jb, lc = j + bw, local_off[c]
        # panel: small Cholesky on the diagonal block (cholesky.py:24)
        Lkk, info = torch.linalg.cholesky_ex(W[j:jb, lc:lc + bw])
        L[j:jb, lc:lc + bw] = Lkk
        if jb < n:
            # triangular solve for the sub-diagonal block (cholesky.py:28-30)
            L[jb:, lc:lc + bw] = torch.linalg.solve_triangular(
                Lkk, W[jb:, lc:lc + bw].T, upper=False).T
        return L[jb:, lc:lc + bw].contiguous(), info.reshape(1).to(torch.int32)

    def post(c, bufs):
        if bufs is None:  # receivers
            bufs = (torch.empty((n - c * b - width(c), width(c)), dtype=W.dtype, device=dev),
                    torch.empty(1, dtype=torch.int32, device=dev))
        return bufs, _post_broadcast([bufs[1], bufs[0]],
                                     _global_rank(group, 0 if world == 1 else c % world),
                                     group, world)

    def update(blocks, L21, jb, bw):
        """W[:, blocks] -= L21 @ L21[blocks]^T from the first block's diagonal down
        (cholesky.py:33 restricted to these columns and rows)."""
        c0 = blocks[0]
        lo = local_off[c0]
        hi = local_off[blocks[-1]] + width(blocks[-1])
        r0 = c0 * b
        _trailing_update(W[r0:, lo:hi], L21[r0 - jb:], L21[gcol[lo:hi] - jb].T, bw, matmul)

    pending = post(0, factor(0) if rank == 0 else None)
    for c in range(nb):
        (L21, info), works = pending
        for w in works:
            w.wait()
        infos.append(info)
        j, bw = c * b, width(c)
        jb = j + bw
        if jb >= n:
            break
        later = [c2 for c2 in mine if c2 > c]
        c1 = c + 1
        next_bufs = None
        if later and later[0] == c1:
            # look-ahead: block c + 1 first, then its panel, broadcast before the rest
            update([c1], L21, jb, bw)
            next_bufs = factor(c1)
            later = later[1:]
        pending = post(c1, next_bufs)
        for run in _contiguous_runs(later, update_parts):
            update(run, L21, jb, bw)
    _raise_first_failure(torch.cat(infos).cpu())
    return L


def cholesky_distributed(A, block_size: int = 64, *, group=None, matmul=None):
    """``cholesky(A, block_size)`` computed block-cyclically over the ranks of `group`; every
    rank passes the same A and gets the same L as one GPU's ``cholesky``, bit for bit."""
    import torch.distributed as dist

    if A.shape[0] != A.shape[1]:
        raise ValueError(f"expected square matrix, got {A.shape}")
    n = A.shape[0]
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    cols = cyclic_columns(n, block_size, rank, world).to(A.device)
    L_local = cholesky_cyclic(A[:, cols].contiguous(), n, block_size, group=group,
                              matmul=matmul)
    L = torch.zeros((n, n), dtype=A.dtype, device=A.device)
    L[:, cols] = L_local
    return _exact_sum_(L, group)
