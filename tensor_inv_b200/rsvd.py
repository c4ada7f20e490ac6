"""Randomized SVD (Halko-Martinsson-Tropp) with every GEMM through the CRT kernels.

Same algorithm, RNG consumption and call order as the reference
(src/tensor_inv/rsvd.py:6-32); ``A.T`` and ``Q.T`` are consumed as transposed views.
"""

import torch

from tensor_inv_b200.crt_matmul import caller_moduli, crt_matmul


def _mm(X, Y):
    """crt_matmul with the moduli set that keeps every bit at this inner dimension (the
    same result as the reference's primes, fewer residue GEMMs)."""
    return crt_matmul(X, Y, moduli=caller_moduli(X.shape[1]))


def rsvd(A, rank, n_oversamples=10, n_power_iter=1):
    """
    Rank-``rank`` SVD of A from a random range finder (Halko, Martinsson and Tropp) whose
    products all run on the CRT-emulated float64 GEMM.

    Returns U (m x rank), S (rank,), Vt (rank x n).
    """
    m, n = A.shape
    r = rank + n_oversamples
    dtype = A.dtype
    device = A.device

    # random projection (rsvd.py:18-20)
    Omega = torch.randn(n, r, dtype=dtype, device=device)
    Y = _mm(A, Omega)
    Q, _ = torch.linalg.qr(Y)

    # power iterations (rsvd.py:23-25)
    for _ in range(n_power_iter):
        Y = _mm(A, _mm(A.T, Q))
        Q, _ = torch.linalg.qr(Y)

    # project to the low-rank subspace (rsvd.py:28-30)
    B = _mm(Q.T, A)
    Ub, S, Vt = torch.linalg.svd(B, full_matrices=False)
    U = _mm(Q, Ub)

    return U[:, :rank], S[:rank], Vt[:rank]
