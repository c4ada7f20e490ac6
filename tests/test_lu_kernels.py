"""LU: the CUDA-input variant of the reference's test, the device kernels against the
reference's own loop bit for bit, edge sizes and error behaviour (tensor_inv_b200)."""
import pytest
import torch

from tensor_inv_b200.lu import lu

pytestmark = pytest.mark.gpu


def test_lu_cuda_input():
    torch.manual_seed(42)
    n = 128
    A = torch.randn(n, n, dtype=torch.float64).cuda()

    P, L, U = lu(A, block_size=32)
    err = (P @ A - L @ U).abs().max().item()
    assert err < 1e-8, f"reconstruction error {err:.2e}"


def test_lu_rejects_non_square():
    with pytest.raises(ValueError):
        lu(torch.zeros(3, 4, dtype=torch.float64))


def _lu_both(A, block_size, monkeypatch):
    import importlib

    lu_mod = importlib.import_module("tensor_inv_b200.lu")  # the module, not the function

    monkeypatch.setattr(lu_mod, "_TORCH_PANEL", True)
    ref = lu(A, block_size=block_size)
    monkeypatch.setattr(lu_mod, "_TORCH_PANEL", False)
    got = lu(A, block_size=block_size)
    return ref, got


def _same_bits(a, b):
    return torch.equal(a.contiguous().view(torch.int64), b.contiguous().view(torch.int64))


def _ties(n):
    # small integers: many equal |entries| in a column, so the argmax tie rule decides pivots
    g = torch.Generator().manual_seed(7)
    return torch.randint(-3, 4, (n, n), generator=g).to(torch.float64)


def _zero_column(n):
    g = torch.Generator().manual_seed(8)
    A = torch.randn(n, n, generator=g, dtype=torch.float64)
    A[:, 5] = 0.0       # a pivot below 1e-15: the reference skips that column
    A[:, 40] = 1e-17
    return A


@pytest.mark.parametrize("n,block,make", [
    (128, 32, None), (300, 64, None), (1000, 256, None), (257, 256, None), (4096, 256, None),
    (96, 32, _ties), (200, 64, _zero_column),
])
def test_device_panel_is_bit_identical(monkeypatch, n, block, make):
    """The cooperative panel kernel gives exactly the reference's torch loop's P, L, U."""
    if make is None:
        g = torch.Generator().manual_seed(n)
        A = torch.randn(n, n, generator=g, dtype=torch.float64)
    else:
        A = make(n)
    (P0, L0, U0), (P1, L1, U1) = _lu_both(A.cuda(), block, monkeypatch)
    assert _same_bits(P0, P1) and _same_bits(L0, L1) and _same_bits(U0, U1)
    if make is None:
        err = ((P1 @ A.cuda() - L1 @ U1).abs().max() / A.abs().max()).item()
        assert err < 1e-10


def _same_bits_or_nan(a, b):
    a, b = a.contiguous(), b.contiguous()
    na, nb = torch.isnan(a), torch.isnan(b)
    if not torch.equal(na, nb):
        return False
    return torch.equal(a.masked_fill(na, 0).view(torch.int64), b.masked_fill(nb, 0).view(torch.int64))


def test_device_panel_nan_pivots(monkeypatch):
    """NaN counts as the largest |entry| (torch.argmax), the first NaN row wins, and a NaN
    pivot fails the 1e-15 test, so the column is skipped: the device panel does the same."""
    g = torch.Generator().manual_seed(12)
    A = torch.randn(300, 300, generator=g, dtype=torch.float64)
    A[150, 3] = float("nan")
    A[90, 3] = float("nan")    # two NaNs in one column: the smaller row index is the pivot
    A[200, 70] = float("nan")  # and one in a later panel
    (P0, L0, U0), (P1, L1, U1) = _lu_both(A.cuda(), 64, monkeypatch)
    assert torch.equal(P0, P1)
    assert _same_bits_or_nan(L0, L1) and _same_bits_or_nan(U0, U1)


def test_device_panel_transposed_input(monkeypatch):
    g = torch.Generator().manual_seed(11)
    A = torch.randn(150, 150, generator=g, dtype=torch.float64).cuda().t()  # column-major view
    (P0, L0, U0), (P1, L1, U1) = _lu_both(A, 64, monkeypatch)
    assert _same_bits(P0, P1) and _same_bits(L0, L1) and _same_bits(U0, U1)


@pytest.mark.parametrize("n,block", [(1, 64), (31, 64), (33, 32), (64, 1), (100, 256), (513, 128)])
def test_device_panel_edge_sizes(monkeypatch, n, block):
    """Tiny panels, one-column blocks, a block wider than the matrix, a ragged last panel."""
    g = torch.Generator().manual_seed(100 + n)
    A = torch.randn(n, n, generator=g, dtype=torch.float64)
    (P0, L0, U0), (P1, L1, U1) = _lu_both(A.cuda(), block, monkeypatch)
    assert _same_bits(P0, P1) and _same_bits(L0, L1) and _same_bits(U0, U1)


@pytest.mark.parametrize("n,ncols,j,b,pc", [
    (700, 380, 0, 64, 0), (700, 380, 128, 64, 64), (700, 380, 640, 60, 320),
    (300, 500, 40, 64, 300), (900, 600, 100, 300, 150),   # b > 256: the global-memory kernel
    (16384, 400, 0, 256, 100),  # 111 rows of 256 columns per CTA: ~223 KB of shared memory
])
def test_panel_at_shifted_columns(n, ncols, j, b, pc):
    """ti_lu_panel_ex: the panel of rows [j, n) in columns [pc, pc + b) of a rectangular W,
    row swaps across all of W's columns, equals the reference loop with shifted columns."""
    from tensor_inv_b200 import _native as nat
    from tensor_inv_b200 import distributed as D

    g = torch.Generator().manual_seed(n + j)
    W0 = torch.randn(n, ncols, generator=g, dtype=torch.float64).cuda()
    Wt, pt = W0.clone(), torch.arange(n, device="cuda")
    D._panel_torch_cols(Wt, pt, j, j + b, pc)
    Wd, pd = W0.clone(), torch.arange(n, device="cuda")
    ws = torch.empty(nat.lu_panel_workspace_size(), dtype=torch.uint8, device="cuda")
    nat.lu_panel_cols(Wd, j, j + b, pc, pd, ws, torch.cuda.current_stream())
    torch.cuda.synchronize()
    assert torch.equal(pt, pd) and _same_bits(Wt, Wd)
    assert nat.device_error(reset=True) == 0
