"""Cholesky: the CUDA-input variant of the reference's test, the device kernels against the
reference's own loop bit for bit, edge sizes and error behaviour (tensor_inv_b200)."""
import pytest
import torch

from tensor_inv_b200.cholesky import cholesky

pytestmark = pytest.mark.gpu


def test_cholesky_cuda_input():
    torch.manual_seed(42)
    n = 128
    A = torch.randn(n, n, dtype=torch.float64)
    A = (A @ A.T + n * torch.eye(n, dtype=torch.float64)).cuda()  # SPD

    L = cholesky(A, block_size=32)
    err = (L @ L.T - A).abs().max().item()
    assert err < 1e-8, f"reconstruction error {err:.2e}"
    assert (torch.diag(L) > 0).all(), "diagonal should be positive"


def test_cholesky_column_major_input():
    """A transposed (column-major) CUDA input gives the same L as the row-major one."""
    g = torch.Generator().manual_seed(5)
    X = torch.randn(200, 200, generator=g, dtype=torch.float64)
    A = X @ X.T / 200 + torch.eye(200, dtype=torch.float64)
    L_row = cholesky(A.cuda(), block_size=64)
    L_col = cholesky(A.cuda().t().contiguous().t(), block_size=64)
    assert torch.equal(L_row.cpu().view(torch.int64), L_col.cpu().contiguous().view(torch.int64))


def test_cholesky_lower_update_is_bit_identical(monkeypatch):
    """Skipping the tiles above the diagonal in the trailing update leaves L unchanged."""
    import importlib

    ch = importlib.import_module("tensor_inv_b200.cholesky")
    g = torch.Generator().manual_seed(6)
    X = torch.randn(900, 900, generator=g, dtype=torch.float64)
    A = (X @ X.T / 900 + torch.eye(900, dtype=torch.float64)).cuda()
    L_low = cholesky(A, block_size=128)
    full = ch.crt_matmul_update

    def update_full(C, A_, B_, alpha=-1, **kw):
        kw["lower"] = False
        return full(C, A_, B_, alpha, **kw)

    monkeypatch.setattr(ch, "crt_matmul_update", update_full)
    L_full = cholesky(A, block_size=128)
    assert torch.equal(L_low.view(torch.int64), L_full.view(torch.int64))


def _reference_loop(A, block_size):
    """The reference's blocked loop (cholesky.py:6-35) with torch.linalg.cholesky per block."""
    from tensor_inv_b200.crt_matmul import crt_matmul

    n = A.shape[0]
    L = torch.zeros_like(A)
    W = A.clone()
    for j in range(0, n, block_size):
        jb = min(j + block_size, n)
        L[j:jb, j:jb] = torch.linalg.cholesky(W[j:jb, j:jb])
        if jb < n:
            L[jb:, j:jb] = torch.linalg.solve_triangular(
                L[j:jb, j:jb], W[jb:, j:jb].T, upper=False).T
            L21 = L[jb:, j:jb]
            W[jb:, jb:] -= crt_matmul(L21, L21.T)
    return L


@pytest.mark.parametrize("n", [700, 4096])
def test_cholesky_matches_reference_loop_bitwise(n):
    """The diagonal blocks through cholesky_ex (no host sync per block) give the reference
    loop's L bit for bit (4096: trailing updates large enough for every tile path)."""
    g = torch.Generator().manual_seed(7)
    X = torch.randn(n, n, generator=g, dtype=torch.float64)
    A = (X @ X.T / n + 1e-3 * torch.eye(n, dtype=torch.float64)).cuda()
    got = cholesky(A, block_size=256)
    want = _reference_loop(A, 256)
    assert torch.equal(got.view(torch.int64), want.view(torch.int64))


def test_cholesky_not_positive_definite_raises_torch_error():
    """A block that fails raises what torch.linalg.cholesky raises on that block."""
    A = torch.eye(600, dtype=torch.float64)
    A[300, 300] = -1.0  # the second diagonal block (rows 256..511) fails at its minor 45
    with pytest.raises(torch.linalg.LinAlgError) as want:
        torch.linalg.cholesky(A[256:512, 256:512])
    with pytest.raises(torch.linalg.LinAlgError) as got:
        cholesky(A.cuda(), block_size=256)
    assert str(got.value) == str(want.value)
    assert "order 45 " in str(got.value)
