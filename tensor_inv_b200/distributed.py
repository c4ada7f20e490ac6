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


def lu_cyclic(W_local, n: int, block_size: int = 64, *, group=None, matmul=None):
    """Blocked LU with partial pivoting (lu.py:6-54) on block-cyclic columns.

    W_local holds this rank's block columns of the n x n matrix (``cyclic_columns``), all n
    rows.  Per block column: its owner factorises the panel (``ti_lu_panel_ex`` on CUDA
    float64, else the reference's torch loop) with row swaps across its local columns, then
    broadcasts the pivot vector and the panel; the other ranks apply the same row permutation
    to their columns.  The U block row is assembled exactly from every rank's columns and
    solved whole on each rank (the reference's call, so the same bits), and each rank updates
    its own trailing columns: a column subset of the reference's product, which the CRT
    kernels compute bit for bit (column exponents depend on their column only).  Returns this
    rank's factored columns and the pivot vector (the same on every rank)."""
    import torch.distributed as dist

    rank, world = dist.get_rank(group), dist.get_world_size(group)
    b = block_size
    W = W_local.clone()
    dev = W.device
    mine = cyclic_blocks(n, b, rank, world)
    local_off = {c: i * b for i, c in enumerate(mine)}
    piv = torch.arange(n, device=dev)
    lu_mod = importlib.import_module("tensor_inv_b200.lu")  # the module, not the function
    device_panel = W.is_cuda and W.dtype == torch.float64 and not lu_mod._TORCH_PANEL
    if device_panel:
        from tensor_inv_b200 import _native as nat

        ws = torch.empty(nat.lu_panel_workspace_size(), dtype=torch.uint8, device=dev)
        stream = torch.cuda.current_stream(dev)
    for j in range(0, n, b):
        c = j // b
        bw = min(b, n - j)
        jb = j + bw
        owner = c % world
        if rank == owner:
            lc = local_off[c]
            if device_panel and bw <= 1024:
                nat.lu_panel_cols(W, j, jb, lc, piv, ws, stream)
            else:
                _panel_torch_cols(W, piv, j, jb, lc)
            panel = W[j:, lc:lc + bw].contiguous()
            new_piv = piv.clone()
        else:
            panel = torch.empty((n - j, bw), dtype=W.dtype, device=dev)
            new_piv = torch.empty_like(piv)
        src = _global_rank(group, owner)
        dist.broadcast(new_piv, src=src, group=group)
        dist.broadcast(panel, src=src, group=group)
        if rank != owner:
            # the owner's row swaps, as one permutation of rows j.. (piv moved with the rows)
            pos = torch.empty_like(piv)
            pos[piv] = torch.arange(n, device=dev)
            W[j:] = W[pos[new_piv[j:]]]
            piv = new_piv
        if jb < n:
            L_panel = torch.tril(panel[:bw], diagonal=-1) + torch.eye(bw, dtype=W.dtype,
                                                                       device=dev)
            later = [c2 for c2 in mine if c2 > c]
            row = torch.zeros((bw, n - jb), dtype=W.dtype, device=dev)
            if later:
                lo = local_off[later[0]]
                gcols = torch.cat([torch.arange(c2 * b, min(n, (c2 + 1) * b))
                                   for c2 in later]).to(dev) - jb
                row[:, gcols] = W[j:jb, lo:]
            _exact_sum_(row, group)
            # triangular solve for the U block row (lu.py:38-43), whole on every rank
            U = torch.linalg.solve_triangular(L_panel, row, upper=False)
            if later:
                U_mine = U[:, gcols]
                W[j:jb, lo:] = U_mine
                # trailing update of this rank's columns (lu.py:46)
                _trailing_update(W[jb:, lo:], panel[bw:], U_mine, bw, matmul)
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


def cholesky_cyclic(A_local, n: int, block_size: int = 64, *, group=None, matmul=None):
    """Blocked right-looking Cholesky (cholesky.py:6-35) on block-cyclic columns.

    The owner of a block column computes its diagonal block's Cholesky factor and the panel
    below it (the reference's calls), broadcasts the panel, and every rank updates its own
    trailing columns with W[:, cols] -= L21 @ L21[cols]^T (all rows below the panel: the
    lower-triangle tile skip of one GPU needs whole columns).  The factor's values are the
    reference's bit for bit.  Returns this rank's columns of L."""
    import torch.distributed as dist

    rank, world = dist.get_rank(group), dist.get_world_size(group)
    b = block_size
    W = A_local.clone()
    L = torch.zeros_like(W)
    dev = W.device
    mine = cyclic_blocks(n, b, rank, world)
    local_off = {c: i * b for i, c in enumerate(mine)}
    for j in range(0, n, b):
        c = j // b
        bw = min(b, n - j)
        jb = j + bw
        owner = c % world
        failure = None
        if rank == owner:
            lc = local_off[c]
            try:
                # panel: small Cholesky on the diagonal block (cholesky.py:24)
                L[j:jb, lc:lc + bw] = torch.linalg.cholesky(W[j:jb, lc:lc + bw])
                if jb < n:
                    # triangular solve for the sub-diagonal block (cholesky.py:28-30)
                    L[jb:, lc:lc + bw] = torch.linalg.solve_triangular(
                        L[j:jb, lc:lc + bw], W[jb:, lc:lc + bw].T, upper=False
                    ).T
            except RuntimeError as e:  # not positive definite: every rank must learn of it
                failure = e
        if world > 1:
            flag = torch.tensor([1 if failure is not None else 0], device=dev)
            dist.broadcast(flag, src=_global_rank(group, owner), group=group)
            if int(flag.item()) and failure is None:
                raise RuntimeError(f"cholesky_distributed: the panel at column {j} failed on "
                                   f"rank {owner} (matrix not positive definite?)")
        if failure is not None:
            raise failure
        if jb >= n:
            break
        if rank == owner:
            L21 = L[jb:, lc:lc + bw].contiguous()
        else:
            L21 = torch.empty((n - jb, bw), dtype=W.dtype, device=dev)
        dist.broadcast(L21, src=_global_rank(group, owner), group=group)
        later = [c2 for c2 in mine if c2 > c]
        if later:
            lo = local_off[later[0]]
            gcols = torch.cat([torch.arange(c2 * b, min(n, (c2 + 1) * b))
                               for c2 in later]).to(dev) - jb
            # trailing update of this rank's columns (cholesky.py:33)
            _trailing_update(W[jb:, lo:], L21, L21[gcols].T, bw, matmul)
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
