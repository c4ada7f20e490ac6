"""Blocked right-looking Cholesky; trailing update through the CRT kernels.

Same algorithm and arithmetic as the reference (src/tensor_inv/cholesky.py:6-35).  The
trailing update ``W[jb:, jb:] -= crt_matmul(L21, L21.T)`` runs fused on CUDA
(``crt_matmul_update``) with ``L21.T`` consumed as a transposed view (no copy).

On CUDA the diagonal blocks go through ``torch.linalg.cholesky_ex``, the same factorization
as the reference's ``torch.linalg.cholesky`` without its per-call host synchronisation for
the error check; the blocks' error codes are checked once at the end, and the first failing
block raises the error ``torch.linalg.cholesky`` would have raised there.
"""

import torch

from tensor_inv_b200.crt_matmul import caller_moduli, crt_matmul, crt_matmul_update


def cholesky(A, block_size=64):
    """
    Blocked Cholesky: panel via torch, trailing GEMM via CRT int8.

    A must be symmetric positive definite.
    """
    if A.shape[0] != A.shape[1]:
        raise ValueError(f"expected square matrix, got {A.shape}")

    n = A.shape[0]
    L = torch.zeros_like(A)
    W = A.clone()
    infos = [] if A.is_cuda else None  # error codes of the diagonal blocks, checked at the end

    for j in range(0, n, block_size):
        b = min(block_size, n - j)
        jb = j + b

        # panel: small Cholesky on the diagonal block (cholesky.py:24)
        if infos is None:
            L[j:jb, j:jb] = torch.linalg.cholesky(W[j:jb, j:jb])
        else:
            L[j:jb, j:jb], info = torch.linalg.cholesky_ex(W[j:jb, j:jb])
            infos.append(info)

        if jb < n:
            # panel: triangular solve for the sub-diagonal block (cholesky.py:28-30)
            L[jb:, j:jb] = torch.linalg.solve_triangular(
                L[j:jb, j:jb], W[jb:, j:jb].T, upper=False
            ).T

            # trailing GEMM update via CRT (cholesky.py:33)
            L21 = L[jb:, j:jb]
            mods = caller_moduli(b)  # same bits as the reference's primes, fewer GEMMs
            if W.is_cuda and W.dtype == torch.float64 and W.stride(1) == 1:
                # only W's lower triangle is read again (cholesky.py:24-30), so tiles
                # entirely above the diagonal are skipped: the same L, half the update
                crt_matmul_update(W[jb:, jb:], L21, L21.T, alpha=-1, moduli=mods, lower=True)
            else:
                W[jb:, jb:] -= crt_matmul(L21, L21.T, moduli=mods)

    if infos:
        _raise_first_failure(torch.stack(infos).cpu())
    return L


def _raise_first_failure(infos):
    """torch.linalg.cholesky's error for the first diagonal block whose factorization failed
    (info = the order of its first leading minor that is not positive-definite)."""
    bad = torch.nonzero(infos)
    if bad.numel():
        order = int(infos[bad[0, 0]])
        raise torch.linalg.LinAlgError(
            "linalg.cholesky: The factorization could not be completed because the input is not "
            f"positive-definite (the leading minor of order {order} is not positive-definite).")
