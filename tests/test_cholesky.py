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
