"""Randomized SVD (Halko-Martinsson-Tropp) with every GEMM through the CRT kernels.

Same algorithm, RNG consumption and call order as the reference
(src/tensor_inv/rsvd.py:6-32); ``A.T`` and ``Q.T`` are consumed as transposed views.
"""

import torch

from tensor_inv_b200.crt_matmul import crt_matmul


def rsvd(A, rank, n_oversamples=10, n_power_iter=1):
    """
    Randomized SVD via CRT int8 GEMM (Halko-Martinsson-Tropp).

    Returns U (m x rank), S (rank,), Vt (rank x n).
    """
    m, n = A.shape
    r = rank + n_oversamples
    dtype = A.dtype
    device = A.device

    # random projection (rsvd.py:18-20)
    Omega = torch.randn(n, r, dtype=dtype, device=device)
    Y = crt_matmul(A, Omega)
    Q, _ = torch.linalg.qr(Y)

    # power iterations (rsvd.py:23-25)
    for _ in range(n_power_iter):
        Y = crt_matmul(A, crt_matmul(A.T, Q))
        Q, _ = torch.linalg.qr(Y)

    # project to the low-rank subspace (rsvd.py:28-30)
    B = crt_matmul(Q.T, A)
    Ub, S, Vt = torch.linalg.svd(B, full_matrices=False)
    U = crt_matmul(Q, Ub)

    return U[:, :rank], S[:rank], Vt[:rank]
