"""The reference's tests/test_cholesky.py, run against tensor_inv_b200."""
import pytest
import torch

from tensor_inv_b200.cholesky import cholesky

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("device", ["cpu", "cuda"])
def test_cholesky(device):
    torch.manual_seed(42)
    n = 128
    A = torch.randn(n, n, dtype=torch.float64)
    A = (A @ A.T + n * torch.eye(n, dtype=torch.float64)).to(device)  # SPD

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
