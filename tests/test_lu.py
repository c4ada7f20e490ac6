"""The reference's tests/test_lu.py, run against tensor_inv_b200 (CPU and CUDA inputs)."""
import pytest
import torch

from tensor_inv_b200.lu import lu

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("device", ["cpu", "cuda"])
def test_lu(device):
    torch.manual_seed(42)
    n = 128
    A = torch.randn(n, n, dtype=torch.float64).to(device)

    P, L, U = lu(A, block_size=32)
    err = (P @ A - L @ U).abs().max().item()
    assert err < 1e-8, f"reconstruction error {err:.2e}"


def test_lu_rejects_non_square():
    with pytest.raises(ValueError):
        lu(torch.zeros(3, 4, dtype=torch.float64))
