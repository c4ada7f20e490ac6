"""Host logic of tensor_inv_b200.cholesky (no GPU): the deferred error check of the diagonal
blocks raises exactly what torch.linalg.cholesky raises on the first failing block."""
import pytest
import torch

from tensor_inv_b200.cholesky import _raise_first_failure


def _torch_error(order):
    A = torch.eye(order + 2, dtype=torch.float64)
    A[order - 1, order - 1] = -1.0  # leading minor `order` is the first that is not positive
    with pytest.raises(torch.linalg.LinAlgError) as e:
        torch.linalg.cholesky(A)
    return str(e.value)


def test_no_failure_raises_nothing():
    _raise_first_failure(torch.zeros(5, dtype=torch.int32))


@pytest.mark.parametrize("infos,order", [([0, 45, 3], 45), ([7, 0], 7), ([0, 0, 1], 1)])
def test_first_failing_block_gives_torch_error(infos, order):
    with pytest.raises(torch.linalg.LinAlgError) as e:
        _raise_first_failure(torch.tensor(infos, dtype=torch.int32))
    assert str(e.value) == _torch_error(order)
