"""The callers (lu, cholesky, rsvd) use the wide moduli wherever those keep every bit: their
results must be bit-identical to the same callers on the reference's primes."""
import importlib

import pytest
import torch

pytestmark = pytest.mark.gpu


def _same(a, b):
    return torch.equal(a.contiguous().view(torch.int64), b.contiguous().view(torch.int64))


def _both(monkeypatch, module, fn):
    mod = importlib.import_module(module)
    monkeypatch.setattr(mod, "caller_moduli", lambda k: None)  # the reference's primes
    ref = fn()
    monkeypatch.undo()
    return ref, fn()


def test_lu_wide_equals_primes(monkeypatch):
    from tensor_inv_b200 import lu

    g = torch.Generator().manual_seed(3)
    A = torch.randn(700, 700, generator=g, dtype=torch.float64).cuda()
    ref, got = _both(monkeypatch, "tensor_inv_b200.lu", lambda: lu(A, block_size=128))
    assert all(_same(x, y) for x, y in zip(ref, got))


def test_cholesky_wide_equals_primes(monkeypatch):
    from tensor_inv_b200 import cholesky

    g = torch.Generator().manual_seed(4)
    X = torch.randn(600, 600, generator=g, dtype=torch.float64)
    A = (X @ X.T / 600 + torch.eye(600, dtype=torch.float64)).cuda()
    ref, got = _both(monkeypatch, "tensor_inv_b200.cholesky", lambda: cholesky(A, block_size=128))
    assert _same(ref, got)


def test_rsvd_wide_equals_primes(monkeypatch):
    from tensor_inv_b200 import rsvd

    g = torch.Generator().manual_seed(5)
    A = torch.randn(3000, 400, generator=g, dtype=torch.float64).cuda()

    def run():
        torch.manual_seed(9)
        return rsvd(A, rank=20, n_oversamples=10, n_power_iter=2)

    ref, got = _both(monkeypatch, "tensor_inv_b200.rsvd", run)
    assert all(_same(x, y) for x, y in zip(ref, got))
