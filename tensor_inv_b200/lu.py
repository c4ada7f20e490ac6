"""Blocked LU with partial pivoting; trailing update through the CRT kernels.

Same algorithm, pivot order and arithmetic as the reference (src/tensor_inv/lu.py:6-54):
an unblocked panel with partial pivoting, a triangular solve for the U block row, and the
trailing update ``W[jb:, jb:] -= crt_matmul(W[jb:, j:jb], W[j:jb, jb:])``.  On CUDA with
float64 the panel is one cooperative kernel per block column (``ti_lu_panel``: the same IEEE
operations in the same order, without the reference's two host round trips per column) and
the update is fused into the CRT reconstruction (``crt_matmul_update``): identical bits, no
temporary product.
"""

import torch

from tensor_inv_b200.crt_matmul import caller_moduli, crt_matmul, crt_matmul_update


def _panel_torch(W, piv, j, jb):
    """The reference's unblocked panel (lu.py:24-34), op for op."""
    for k in range(j, jb):
        max_idx = W[k:, k].abs().argmax() + k
        if max_idx != k:
            W[k], W[max_idx] = W[max_idx].clone(), W[k].clone()
            piv[k], piv[max_idx] = piv[max_idx].clone(), piv[k].clone()

        if W[k, k].abs() > 1e-15:
            W[k + 1 :, k] /= W[k, k]
            W[k + 1 :, k + 1 : jb] -= W[k + 1 :, k : k + 1] @ W[k : k + 1, k + 1 : jb]


# Set by tests to run the reference's torch panel loop on CUDA as well (for comparisons).
_TORCH_PANEL = False


def _trailing_update(W, j, jb):
    # fused into the reconstruction when W is row-major (the kernel's output layout); the
    # same bits either way
    mods = caller_moduli(jb - j)  # same bits as the reference's primes, fewer GEMMs
    if W.is_cuda and W.dtype == torch.float64 and W.stride(1) == 1:
        crt_matmul_update(W[jb:, jb:], W[jb:, j:jb], W[j:jb, jb:], alpha=-1, moduli=mods)
    else:
        W[jb:, jb:] -= crt_matmul(W[jb:, j:jb], W[j:jb, jb:], moduli=mods)


def lu(A, block_size=64):
    """
    Blocked LU with partial pivoting: panel via torch, trailing GEMM via CRT int8.

    Returns P, L, U such that PA = LU.
    """
    if A.shape[0] != A.shape[1]:
        raise ValueError(f"expected square matrix, got {A.shape}")

    n = A.shape[0]
    device_panel = A.is_cuda and A.dtype == torch.float64 and not _TORCH_PANEL
    # the device panel wants a row-major W; the values (and so every result bit) are the same
    W = A.contiguous().clone() if device_panel else A.clone()
    piv = torch.arange(n, device=A.device)
    if device_panel:
        from tensor_inv_b200 import _native as nat

        ws = torch.empty(nat.lu_panel_workspace_size(), dtype=torch.uint8, device=A.device)
        stream = torch.cuda.current_stream(A.device)

    for j in range(0, n, block_size):
        b = min(block_size, n - j)
        jb = j + b

        # panel: unblocked LU with partial pivoting (lu.py:24-34)
        if device_panel and b <= 1024:
            nat.lu_panel(W, j, jb, piv, ws, stream)
        else:
            _panel_torch(W, piv, j, jb)

        if jb < n:
            # triangular solve for the U block row (lu.py:38-43)
            L_panel = torch.tril(W[j:jb, j:jb], diagonal=-1) + torch.eye(
                b, dtype=A.dtype, device=A.device
            )
            W[j:jb, jb:] = torch.linalg.solve_triangular(L_panel, W[j:jb, jb:], upper=False)

            # trailing GEMM update via CRT (lu.py:46)
            _trailing_update(W, j, jb)

    L = torch.tril(W, diagonal=-1) + torch.eye(n, dtype=A.dtype, device=A.device)
    U = torch.triu(W)

    P = torch.zeros(n, n, dtype=A.dtype, device=A.device)
    P[torch.arange(n, device=A.device), piv] = 1.0

    return P, L, U
