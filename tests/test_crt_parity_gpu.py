"""Parity of the sm_100a CRT matmul with the reference (golden fixtures) and the oracle.

Bit-exact throughout: float64 outputs are compared as uint64 bit patterns, residues and
exponents as integers.  Sizes stay where the C oracle answers in seconds; beyond that,
sub-blocks of a large product are checked (row exponents depend only on A's rows and
column exponents only on B's columns, so every output block of the full product equals
the product of the matching panels).
"""

import ctypes
import importlib

import numpy as np
import pytest
import torch

from conftest import GOLDEN, golden_cases

pytestmark = pytest.mark.gpu

DTYPES = {"float64": torch.float64, "float32": torch.float32, "float16": torch.float16,
          "bfloat16": torch.bfloat16}


def _bits(t):
    return t.detach().cpu().contiguous().view(torch.int64).numpy()


def _assert_bitexact(got, want):
    got = got.detach().cpu().to(torch.float64).contiguous()
    want = np.ascontiguousarray(want, np.float64)
    g, w = got.numpy().view(np.uint64), want.view(np.uint64)
    if not np.array_equal(g, w):
        bad = np.argwhere(g != w)
        i, j = bad[0]
        raise AssertionError(f"{len(bad)} mismatches; first at {(i, j)}: got "
                             f"{got.numpy()[i, j]!r} want {want[i, j]!r}")


@pytest.fixture(scope="module")
def ti():
    import tensor_inv_b200

    assert torch.cuda.is_available()
    return tensor_inv_b200


@pytest.fixture(autouse=True)
def _no_device_error():
    from tensor_inv_b200 import _native

    yield
    torch.cuda.synchronize()
    assert _native.device_error(reset=True) == 0


def _golden(case):
    return dict(np.load(GOLDEN / f"{case}.npz"))


@pytest.mark.parametrize("case", golden_cases())
def test_golden_full_path(ti, case):
    g = _golden(case)
    dt = DTYPES[str(g["dtype"])]
    A = torch.from_numpy(g["A"]).to(dt).cuda()
    B = torch.from_numpy(g["B"]).to(dt).cuda()
    C = ti.crt_matmul(A, B)
    assert C.dtype == torch.float64 and C.is_cuda
    _assert_bitexact(C, g["out"])


@pytest.mark.parametrize("case", golden_cases())
def test_golden_stages(ti, case):
    cm = importlib.import_module("tensor_inv_b200.crt_matmul")

    g = _golden(case)
    bits, moduli = int(g["bits"]), [int(p) for p in g["moduli"]]
    A = torch.from_numpy(g["A"]).cuda()
    B = torch.from_numpy(g["B"]).cuda()
    re, ares = cm._split(A, bits, len(moduli), axis_k=1)
    ce, bres = cm._split(B, bits, len(moduli), axis_k=0)
    np.testing.assert_array_equal(re.cpu().numpy(), g["row_exp"])
    np.testing.assert_array_equal(ce.cpu().numpy(), g["col_exp"])
    np.testing.assert_array_equal(ares.cpu().numpy(), g["a_res"])
    np.testing.assert_array_equal(bres.cpu().numpy().transpose(0, 2, 1), g["b_res"])
    # residue GEMM on the reference's own residues, reference layout
    c = cm._matmul_residues(torch.from_numpy(g["a_res"]).cuda(),
                            torch.from_numpy(g["b_res"]).cuda(), moduli)
    np.testing.assert_array_equal(torch.stack(c).cpu().numpy(), g["c_res"])
    # CRT on the reference's own residue products
    out = cm._crt_reconstruct(torch.from_numpy(g["c_res"]).cuda(), moduli, bits,
                              torch.from_numpy(g["row_exp"]), torch.from_numpy(g["col_exp"]))
    _assert_bitexact(out, g["out"])


def _rand(shape, seed, phi=None, dtype=torch.float64):
    gen = torch.Generator().manual_seed(seed)
    if phi is None:
        x = torch.randn(*shape, generator=gen, dtype=torch.float64)
    else:
        u = torch.rand(*shape, generator=gen, dtype=torch.float64) - 0.5
        x = u * torch.exp(phi * torch.randn(*shape, generator=gen, dtype=torch.float64))
    return x.to(dtype)


SHAPES = [
    (1024, 1024, 1024, None),   # 1024^3, N(0,1)
    (300, 500, 257, 2.0),
    (129, 257, 1, None),
    (133, 77, 1100, 1.0),
    (1, 300, 40, None),
    (257, 1, 129, 0.5),
    (128, 256, 128, None),      # exactly one tile
    (200, 600, 7200, 0.5),      # N = 25 moduli
]


@pytest.mark.parametrize("m,n,k,phi", SHAPES)
def test_vs_oracle(ti, oracle, m, n, k, phi):
    A = _rand((m, k), 1000 + m, phi)
    B = _rand((k, n), 2000 + n, phi)
    want = oracle.crt_matmul(A.numpy(), B.numpy(), 53)
    _assert_bitexact(ti.crt_matmul(A.cuda(), B.cuda()), want)


@pytest.mark.parametrize("ta,tb", [(True, False), (False, True), (True, True)])
def test_transposed_views(ti, oracle, ta, tb):
    m, n, k = 190, 150, 333
    A = _rand((k, m), 7, 1.0).T if ta else _rand((m, k), 7, 1.0)
    B = _rand((n, k), 8, 1.0).T if tb else _rand((k, n), 8, 1.0)
    want = oracle.crt_matmul(A.numpy(), B.numpy(), 53)
    _assert_bitexact(ti.crt_matmul(A.cuda(), B.cuda()), want)


def test_strided_view_is_copied(ti, oracle):
    A = _rand((120, 300), 3)[:, ::3]      # neither stride is 1
    B = _rand((100, 90), 4)
    want = oracle.crt_matmul(A.numpy(), B.numpy(), 53)
    _assert_bitexact(ti.crt_matmul(A.cuda(), B.cuda()), want)


@pytest.mark.parametrize("dtype,bits", [(torch.float32, 24), (torch.bfloat16, 8),
                                        (torch.float16, 11)])
def test_reduced_precision(ti, oracle, dtype, bits):
    A = _rand((150, 700), 11, 0.5, dtype)
    B = _rand((700, 130), 12, 0.5, dtype)
    want = oracle.crt_matmul(A.double().numpy(), B.double().numpy(), bits)
    _assert_bitexact(ti.crt_matmul(A.cuda(), B.cuda()), want)


def test_cpu_inputs_round_trip(ti, oracle):
    A = _rand((37, 51), 42)
    B = _rand((51, 29), 43)
    C = ti.crt_matmul(A, B)
    assert C.device.type == "cpu"
    _assert_bitexact(C, oracle.crt_matmul(A.numpy(), B.numpy(), 53))


@pytest.mark.parametrize("alpha", [-1, 1])
def test_fused_update(ti, oracle, alpha):
    m, n, k = 300, 270, 256
    A = _rand((m, k), 21)
    B = _rand((k, n), 22)
    C0 = _rand((m, n), 23)
    prod = oracle.crt_matmul(A.numpy(), B.numpy(), 53)
    want = C0.numpy() - prod if alpha == -1 else C0.numpy() + prod
    C = C0.cuda()
    ti.crt_matmul_update(C, A.cuda(), B.cuda(), alpha=alpha)
    _assert_bitexact(C, want)


def test_update_on_submatrix_view(ti, oracle):
    W = _rand((400, 400), 31)
    want = W.numpy().copy()
    want[100:, 100:] -= oracle.crt_matmul(W.numpy()[100:, 36:100], W.numpy()[36:100, 100:], 53)
    Wd = W.cuda()
    ti.crt_matmul_update(Wd[100:, 100:], Wd[100:, 36:100], Wd[36:100, 100:], alpha=-1)
    _assert_bitexact(Wd, want)


@pytest.mark.parametrize("k", [60, 1100])  # 1100: the two-pass column exponents
def test_nonfinite_rows_and_cols(ti, oracle, k):
    A = _rand((40, k), 51)
    B = _rand((k, 30), 52)
    A[3, 7] = float("nan")
    A[9, 0] = float("inf")
    B[5, 11] = float("-inf")
    B[k - 1, 20] = 1e300  # a large entry in the last slice of k
    C = ti.crt_matmul(A.cuda(), B.cuda()).cpu()
    assert torch.isnan(C[3]).all() and torch.isnan(C[9]).all() and torch.isnan(C[:, 11]).all()
    keep_r = [i for i in range(40) if i not in (3, 9)]
    keep_c = [j for j in range(30) if j != 11]
    want = oracle.crt_matmul(A[keep_r].numpy(), B[:, keep_c].numpy(), 53)
    _assert_bitexact(C[keep_r][:, keep_c], want)


def test_overflow_gives_inf(ti):
    # the reference raises OverflowError from math.ldexp; the kernel returns +-inf
    A = torch.full((2, 4), 1e200, dtype=torch.float64)
    B = torch.full((4, 2), 1e200, dtype=torch.float64)
    C = ti.crt_matmul(A.cuda(), B.cuda()).cpu()
    assert torch.isinf(C).all() and (C > 0).all()


def test_large_blocks_vs_oracle(ti, oracle):
    """4096^3 product; three output blocks checked bit for bit against panel products."""
    m = n = k = 4096
    A = _rand((m, k), 61, 1.0)
    B = _rand((k, n), 62, 1.0)
    C = ti.crt_matmul(A.cuda(), B.cuda()).cpu()
    for (r0, r1, c0, c1) in [(0, 96, 0, 80), (4000, 4096, 4017, 4096), (1234, 1300, 2900, 3000)]:
        want = oracle.crt_matmul(A[r0:r1].numpy(), B[:, c0:c1].numpy(), 53)
        _assert_bitexact(C[r0:r1, c0:c1], want)


def test_residue_gemm_signed_inputs(ti, oracle):
    """The reference-layout GEMM entry point accepts any int8 and any modulus in [2, 256)."""
    cm = importlib.import_module("tensor_inv_b200.crt_matmul")

    gen = torch.Generator().manual_seed(5)
    a = torch.randint(-128, 128, (4, 70, 300), generator=gen, dtype=torch.int8)
    b = torch.randint(-128, 128, (4, 300, 50), generator=gen, dtype=torch.int8)
    moduli = [3, 251, 128, 97]
    got = torch.stack(cm._matmul_residues(a.cuda(), b.cuda(), moduli)).cpu().numpy()
    want = oracle.residue_gemm(a.numpy(), b.numpy(), moduli)
    np.testing.assert_array_equal(got, want)


def test_errors(ti):
    A = torch.randn(4, 5, dtype=torch.float64, device="cuda")
    with pytest.raises(TypeError):
        ti.crt_matmul(A.int(), A.int())
    with pytest.raises(IndexError):
        ti.crt_matmul(A[:, :0], A[:0])
    with pytest.raises(RuntimeError):
        ti.crt_matmul(A, A)
    with pytest.raises(ValueError):
        from tensor_inv_b200.crt_matmul import _n_moduli
        _n_moduli(2**62, 53)
    with pytest.raises(ValueError, match="accumulator"):
        big = torch.zeros(1, 135264, dtype=torch.float64, device="cuda")
        ti.crt_matmul(big, big.T)


def test_empty_outputs(ti):
    A = torch.randn(0, 5, dtype=torch.float64, device="cuda")
    B = torch.randn(5, 3, dtype=torch.float64, device="cuda")
    assert ti.crt_matmul(A, B).shape == (0, 3)
    assert ti.crt_matmul(B.T, B[:, :0]).shape == (3, 0)


# ---------------------------------------------------------------------------------------
# fused GEMM+CRT kernel (opt-in with TI_CRT_PATH=fused)
# ---------------------------------------------------------------------------------------
@pytest.fixture
def crt_path(monkeypatch):
    def set_path(p):
        monkeypatch.setenv("TI_CRT_PATH", p)
    return set_path


@pytest.mark.parametrize("m,n,k,phi", [(300, 500, 257, 2.0), (129, 257, 1, None),
                                       (133, 77, 1100, 1.0), (128, 256, 128, None),
                                       (200, 600, 7200, 0.5)])
def test_fused_path_vs_oracle(ti, oracle, crt_path, m, n, k, phi):
    crt_path("fused")
    A = _rand((m, k), 3000 + m, phi)
    B = _rand((k, n), 4000 + n, phi)
    want = oracle.crt_matmul(A.numpy(), B.numpy(), 53)
    _assert_bitexact(ti.crt_matmul(A.cuda(), B.cuda()), want)


def test_fused_equals_unfused_large(ti, oracle, crt_path):
    m, n, k = 2304, 4100, 513      # 18 x 17 = 306 output tiles
    A = _rand((m, k), 71, 1.5).cuda()
    B = _rand((k, n), 72, 1.5).cuda()
    crt_path("fused")
    C_auto = ti.crt_matmul(A, B)
    crt_path("unfused")
    C_unf = ti.crt_matmul(A, B)
    _assert_bitexact(C_auto, C_unf.cpu().numpy())
    for (r0, r1, c0, c1) in [(0, 64, 0, 64), (2250, 2304, 4050, 4100)]:
        want = oracle.crt_matmul(A[r0:r1].cpu().numpy(), B[:, c0:c1].cpu().numpy(), 53)
        _assert_bitexact(C_auto[r0:r1, c0:c1], want)


@pytest.mark.parametrize("alpha", [-1, 1])
def test_fused_update_modes(ti, oracle, crt_path, alpha):
    crt_path("fused")
    m, n, k = 300, 270, 256
    A = _rand((m, k), 81)
    B = _rand((k, n), 82)
    C0 = _rand((m, n), 83)
    prod = oracle.crt_matmul(A.numpy(), B.numpy(), 53)
    want = C0.numpy() - prod if alpha == -1 else C0.numpy() + prod
    C = C0.cuda()
    ti.crt_matmul_update(C, A.cuda(), B.cuda(), alpha=alpha)
    _assert_bitexact(C, want)


# ---------------------------------------------------------------------------------------
# the two reconstruction kernels (tensor-core default, SIMT with TI_CRT_K3=simt)
# ---------------------------------------------------------------------------------------
@pytest.mark.parametrize("m,n,k,phi,moduli", [(1, 1, 1, None, None), (3, 129, 40, 2.0, None),
                                              (130, 255, 300, 1.0, "wide"),
                                              (517, 1000, 2049, 0.5, None),
                                              (257, 384, 7200, 3.0, "wide")])
def test_k3_kernels_agree(ti, oracle, monkeypatch, m, n, k, phi, moduli):
    A = _rand((m, k), 6100 + m, phi).cuda()
    B = _rand((k, n), 6200 + n, phi).cuda()
    monkeypatch.setenv("TI_CRT_K3", "simt")
    C_simt = ti.crt_matmul(A, B, moduli=moduli)
    monkeypatch.delenv("TI_CRT_K3")
    C_tc = ti.crt_matmul(A, B, moduli=moduli)
    _assert_bitexact(C_tc, C_simt.cpu().numpy())
    r1, c1 = min(m, 96), min(n, 160)
    want = oracle.crt_matmul(A[:r1].cpu().numpy(), B[:, :c1].cpu().numpy(), 53)
    _assert_bitexact(C_tc[:r1, :c1], want)


# ---------------------------------------------------------------------------------------
# the two split kernels (tensor-core default, SIMT with TI_SPLIT=simt)
# ---------------------------------------------------------------------------------------
def _view(X, layout):
    """The same matrix as a row-major tensor ("c"), a transposed view ("t"), or a view with
    an odd row stride ("odd"), which the tensor-core split hands to the SIMT kernels."""
    if layout == "c":
        return X.contiguous()
    if layout == "t":
        return X.t().contiguous().t()
    big = torch.empty((X.shape[0], X.shape[1] + 1), dtype=X.dtype, device=X.device)
    big[:, : X.shape[1]] = X
    return big[:, : X.shape[1]]


def _tc_layout_ok(X, k_axis):
    """Whether the tensor-core split takes this operand (an even stride between the float64
    rows or columns it copies), as the library decides."""
    so, sk = (X.stride(0), X.stride(1)) if k_axis == 1 else (X.stride(1), X.stride(0))
    st = so if sk == 1 else sk
    return st >= 2 and st % 2 == 0


@pytest.mark.parametrize("m,n,k,phi,moduli,la,lb", [
    (1, 1, 1, None, None, "c", "c"),          # unit strides: SIMT fallback
    (9, 8, 300, 2.0, "wide", "c", "c"),       # ragged vector block, k not a multiple of 256
    (130, 254, 514, 1.0, None, "t", "t"),     # 25 primes: 4 groups per MMA; transposed views
    (258, 384, 1024, 3.0, "wide", "t", "c"),
    (1001, 64, 2, 1.0, "wide", "c", "c"),     # k = 2: one k block holding padding
    (64, 96, 777, 0.5, "wide", "odd", "c"),   # odd stride: SIMT fallback for A
    (500, 520, 2048, 1.0, "wide", "c", "t"),
])
def test_split_kernels_agree(ti, oracle, monkeypatch, m, n, k, phi, moduli, la, lb):
    A = _view(_rand((m, k), 6400 + m, phi).cuda(), la)
    B = _view(_rand((k, n), 6500 + n, phi).cuda(), lb)
    monkeypatch.setenv("TI_SPLIT", "simt")
    C_simt = ti.crt_matmul(A, B, moduli=moduli)
    # tensor cores only (an unsuitable layout is an error) when both operands suit them
    strict = _tc_layout_ok(A, 1) and _tc_layout_ok(B, 0)
    monkeypatch.setenv("TI_SPLIT", "tc" if strict else "auto")
    C_tc = ti.crt_matmul(A, B, moduli=moduli)
    _assert_bitexact(C_tc, C_simt.cpu().numpy())
    r1, c1 = min(m, 64), min(n, 96)
    want = oracle.crt_matmul(A[:r1].cpu().numpy(), B[:, :c1].cpu().numpy(), 53)
    _assert_bitexact(C_tc[:r1, :c1], want)


def test_split_tensor_core_nonfinite_and_extremes(ti, oracle, monkeypatch):
    m, n, k = 40, 48, 600
    A = _rand((m, k), 6601, 4.0)
    B = _rand((k, n), 6602, 4.0)
    A[3, 7] = float("nan")
    B[5, 11] = float("-inf")
    A[10] = 0.0                                  # zero row: exponent clamp
    A[11, :5] = torch.tensor([5e-324, -5e-324, 2.2e-308, -1.7e308, 1.7e308], dtype=torch.float64)
    B[:, 20] = -2.0 ** -1070                     # subnormal column
    monkeypatch.setenv("TI_SPLIT", "simt")
    C = ti.crt_matmul(A.cuda(), B.cuda(), moduli="wide").cpu()
    assert torch.isnan(C[3]).all() and torch.isnan(C[:, 11]).all()
    monkeypatch.setenv("TI_SPLIT", "tc")
    _assert_bitexact(ti.crt_matmul(A.cuda(), B.cuda(), moduli="wide"), C.numpy())
    keep_r = [i for i in range(m) if i != 3]
    keep_c = [j for j in range(n) if j != 11]
    want = oracle.crt_matmul(A[keep_r].numpy(), B[:, keep_c].numpy(), 53)
    _assert_bitexact(C[keep_r][:, keep_c], want)


@pytest.mark.parametrize("alpha", [-1, 1])
def test_k3_tensor_core_update_modes(ti, oracle, alpha):
    m, n, k = 301, 259, 129
    A = _rand((m, k), 6301)
    B = _rand((k, n), 6302)
    C0 = _rand((m, n), 6303)
    prod = oracle.crt_matmul(A.numpy(), B.numpy(), 53)
    want = C0.numpy() - prod if alpha == -1 else C0.numpy() + prod
    C = C0.cuda()
    ti.crt_matmul_update(C, A.cuda(), B.cuda(), alpha=alpha)
    _assert_bitexact(C, want)


def test_fused_nonfinite(ti, oracle, crt_path):
    crt_path("fused")
    A = _rand((40, 60), 91)
    B = _rand((60, 30), 92)
    A[3, 7] = float("nan")
    B[5, 11] = float("inf")
    C = ti.crt_matmul(A.cuda(), B.cuda()).cpu()
    assert torch.isnan(C[3]).all() and torch.isnan(C[:, 11]).all()
    keep_r = [i for i in range(40) if i != 3]
    keep_c = [j for j in range(30) if j != 11]
    want = oracle.crt_matmul(A[keep_r].numpy(), B[:, keep_c].numpy(), 53)
    _assert_bitexact(C[keep_r][:, keep_c], want)


# ---------------------------------------------------------------------------------------
# opt-in wide moduli (pairwise-coprime odd moduli <= 255)
# ---------------------------------------------------------------------------------------
@pytest.mark.parametrize("case", golden_cases())
def test_wide_moduli_full_precision_is_bit_identical(ti, case):
    """Automatic wide count keeps every bit: the reference's own outputs, bit for bit."""
    g = _golden(case)
    dt = DTYPES[str(g["dtype"])]
    A = torch.from_numpy(g["A"]).to(dt).cuda()
    B = torch.from_numpy(g["B"]).to(dt).cuda()
    _assert_bitexact(ti.crt_matmul(A, B, moduli="wide"), g["out"])


@pytest.mark.parametrize("m,n,k,phi", [(300, 500, 257, 2.0), (133, 77, 1100, 1.0),
                                       (200, 600, 7200, 0.5), (1024, 1024, 1024, None)])
def test_wide_moduli_vs_reference_scheme(ti, oracle, m, n, k, phi):
    A = _rand((m, k), 5000 + m, phi)
    B = _rand((k, n), 6000 + n, phi)
    want = oracle.crt_matmul(A.numpy(), B.numpy(), 53)
    _assert_bitexact(ti.crt_matmul(A.cuda(), B.cuda(), moduli="wide"), want)


@pytest.mark.parametrize("moduli,n_mod", [(mod, n) for mod in ("wide", "primes")
                                          for n in (12, 13, 14, 15, 16)]
                         + [("primes", 17), ("primes", 18)])
def test_moduli_sweep_vs_oracle(ti, oracle, n_mod, moduli):
    """Moduli-count sweep: N moduli, precision lowered to what N moduli can hold; bit-exact
    against the reference algorithm restated with the same moduli and precision."""
    from tensor_inv_b200 import _native

    m, n, k = 96, 80, 8192
    A = _rand((m, k), 7000 + n_mod, 2.0)
    B = _rand((k, n), 8000 + n_mod, 2.0)
    N, bits, mods = _native.crt_plan(k, 53, moduli, n_mod)
    assert N == n_mod and bits <= 53
    want = oracle.crt_matmul_moduli(A.numpy(), B.numpy(), mods, bits)
    got = ti.crt_matmul(A.cuda(), B.cuda(), moduli=moduli, n_moduli=n_mod)
    _assert_bitexact(got, want)


def test_wide_moduli_transposed_and_update(ti, oracle, crt_path):
    m, n, k = 190, 150, 333
    A = _rand((k, m), 17, 1.0).T
    B = _rand((n, k), 18, 1.0).T
    want = oracle.crt_matmul(A.numpy(), B.numpy(), 53)
    _assert_bitexact(ti.crt_matmul(A.cuda(), B.cuda(), moduli="wide"), want)
    crt_path("fused")
    _assert_bitexact(ti.crt_matmul(A.cuda(), B.cuda(), moduli="wide"), want)
    C0 = _rand((m, n), 19)
    C = C0.cuda()
    ti.crt_matmul_update(C, A.cuda(), B.cuda(), alpha=-1, moduli="wide")
    _assert_bitexact(C, C0.numpy() - want)


def test_wide_moduli_large_blocks(ti, oracle):
    m = n = k = 4096
    A = _rand((m, k), 63, 2.0)
    B = _rand((k, n), 64, 2.0)
    C = ti.crt_matmul(A.cuda(), B.cuda(), moduli="wide").cpu()
    for (r0, r1, c0, c1) in [(0, 64, 0, 48), (4030, 4096, 4040, 4096)]:
        want = oracle.crt_matmul(A[r0:r1].numpy(), B[:, c0:c1].numpy(), 53)
        _assert_bitexact(C[r0:r1, c0:c1], want)


def test_moduli_errors(ti):
    A = torch.randn(4, 5, dtype=torch.float64, device="cuda")
    with pytest.raises(ValueError):
        ti.crt_matmul(A, A.T, moduli="octal")
    with pytest.raises(ValueError):
        ti.crt_matmul(A, A.T, moduli="wide", n_moduli=17)
    with pytest.raises(ValueError):
        big = torch.zeros(1, 133145, dtype=torch.float64, device="cuda")
        ti.crt_matmul(big, big.T, moduli="wide")


# ---------------------------------------------------------------------------------------
# banded pipeline (row bands over two internal streams) against one in-order band
# ---------------------------------------------------------------------------------------
def _run_ex(A, B, C, out_mode, bands, moduli=None):
    from tensor_inv_b200 import _native as nat

    m, k = A.shape
    n = B.shape[1]
    opt = nat.options(moduli, None, None, bands)
    ws_bytes = nat.crt_workspace_size_ex(m, n, k, 53, opt)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    st = nat.lib().ti_crt_matmul_ex(A.data_ptr(), A.stride(0), A.stride(1), B.data_ptr(),
                                    B.stride(0), B.stride(1), C.data_ptr(), C.stride(0), m, n, k,
                                    53, out_mode, ws.data_ptr(), ws_bytes,
                                    torch.cuda.current_stream().cuda_stream, ctypes.byref(opt))
    nat.check("ti_crt_matmul_ex", st)
    return C


@pytest.mark.parametrize("moduli", [None, "wide"])
def test_banded_pipeline_matches_single_band(ti, oracle, moduli):
    m, n, k = 2500, 700, 1500   # 3 bands of 896, 896 and 708 rows
    A = _rand((m, k), 101, 1.0).cuda()
    B = _rand((n, k), 102, 1.0).T.cuda()      # transposed view: column split path
    C1 = _run_ex(A, B, torch.empty(m, n, dtype=torch.float64, device="cuda"), 0, 1, moduli)
    for bands in (2, 3, 8):
        Cb = _run_ex(A, B, torch.full((m, n), float("nan"), dtype=torch.float64, device="cuda"),
                     0, bands, moduli)
        _assert_bitexact(Cb, C1.cpu().numpy())
    want = oracle.crt_matmul(A[2400:2500].cpu().numpy(), B[:, 600:700].cpu().numpy(), 53)
    _assert_bitexact(C1[2400:2500, 600:700], want)


def test_banded_update_mode(ti, oracle):
    m, n, k = 2100, 300, 256
    A = _rand((m, k), 111)
    B = _rand((k, n), 112)
    C0 = _rand((m, n), 113)
    want = C0.numpy() - oracle.crt_matmul(A.numpy(), B.numpy(), 53)
    C = _run_ex(A.cuda(), B.cuda(), C0.cuda(), 1, 4)
    _assert_bitexact(C, want)


def test_banded_on_side_stream(ti, oracle):
    """The pipeline forks from and joins back to the caller's (non-default) stream."""
    m, n, k = 4096, 512, 700
    A = _rand((m, k), 121).cuda()
    B = _rand((k, n), 122).cuda()
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        C = ti.crt_matmul(A, B)
        D = C * 1.0   # consumer on the same stream must see the finished product
    s.synchronize()
    want = oracle.crt_matmul(A[:64].cpu().numpy(), B.cpu().numpy(), 53)
    _assert_bitexact(D[:64], want)


# ---------------------------------------------------------------------------------------
# host operands: copies pipelined with the kernels (ti_crt_matmul_host)
# ---------------------------------------------------------------------------------------
@pytest.mark.parametrize("pinned", [True, False])
@pytest.mark.parametrize("moduli", [None, "wide"])
def test_host_pipeline_matches_device_path(ti, pinned, moduli):
    m, n, k = 2500, 333, 1100   # 4 bands of 640 rows (the last 580)
    A = _rand((m, k), 131, 1.0)
    B = _rand((k, n), 132, 1.0)
    if pinned:
        A, B = A.pin_memory(), B.pin_memory()
    C = ti.crt_matmul(A, B, moduli=moduli)
    assert C.device.type == "cpu" and C.shape == (m, n)
    want = ti.crt_matmul(A.cuda(), B.cuda(), moduli=moduli)
    _assert_bitexact(C, want.cpu().numpy())


@pytest.mark.parametrize("b_colmajor", [False, True])
def test_host_pipeline_uneven_bands(ti, b_colmajor):
    """m >= 4096: a 256-row first band, ~1024-row middle bands and 512/256/128-row last
    bands (m = 4100: 256, 1024, 1024, 900, 512, 256, 128); B split before A's first band."""
    m, n, k = 4100, 200, 160
    A = _rand((m, k), 171, 1.0).pin_memory()
    B = _rand((k, n), 172, 1.0)
    B = B.T.contiguous().pin_memory().T if b_colmajor else B.pin_memory()
    C = ti.crt_matmul(A, B, moduli="wide")
    want = ti.crt_matmul(A.cuda(), B.cuda(), moduli="wide")
    _assert_bitexact(C, want.cpu().numpy())


def test_host_pipeline_bands_on_pair_gemm(ti):
    """Uneven host bands with K >= 1024 and n >= 256: each band's GEMM runs on CTA pairs."""
    m, n, k = 4100, 300, 1100
    A = _rand((m, k), 175, 1.0).pin_memory()
    B = _rand((k, n), 176, 1.0).pin_memory()
    C = ti.crt_matmul(A, B, moduli="wide")
    want = ti.crt_matmul(A.cuda(), B.cuda(), moduli="wide")
    _assert_bitexact(C, want.cpu().numpy())


def test_host_pipeline_transposed_views(ti, oracle):
    A = _rand((300, 900), 141, 0.5).T     # 900 x 300, column-major view
    B = _rand((250, 300), 142, 0.5).T     # 300 x 250, column-major view
    want = oracle.crt_matmul(A.numpy(), B.numpy(), 53)
    _assert_bitexact(ti.crt_matmul(A, B), want)


def test_host_results_are_never_overwritten(ti):
    """Results returned on the CPU come from a pool of pinned blocks; a block still referred
    to (by the result, a view of it or a numpy array) must not be handed out again."""
    A = _rand((300, 200), 151)
    B = _rand((200, 100), 152)
    C1 = ti.crt_matmul(A, B)
    keep_view = C1[10:20]
    keep_np = C1.numpy()
    snap = C1.clone()
    del C1
    C2 = ti.crt_matmul(2 * A, B)
    assert C2.data_ptr() != keep_view.data_ptr() - 10 * 100 * 8
    assert torch.equal(keep_view, snap[10:20])
    del keep_view
    assert np.array_equal(keep_np, snap.numpy())
    assert torch.equal(C2, ti.crt_matmul((2 * A).cuda(), B.cuda()).cpu())


def test_host_result_blocks_are_reused(ti):
    """Dropped results give their pinned block back: steady state allocates nothing."""
    A = _rand((256, 128), 161)
    B = _rand((128, 64), 162)
    ptrs = set()
    C = None
    for _ in range(6):
        C = ti.crt_matmul(A, B)   # the previous result dies when C is rebound
        ptrs.add(C.data_ptr())
    assert len(ptrs) <= 2


# ---------------------------------------------------------------------------------------
# lower-triangle updates (symmetric trailing updates)
# ---------------------------------------------------------------------------------------
@pytest.mark.parametrize("n,k,k3", [(300, 256, "tc"), (1030, 129, "tc"), (517, 64, "simt"),
                                    (2000, 256, "tc")])
def test_lower_update_matches_full_on_lower_triangle(ti, monkeypatch, n, k, k3):
    if k3 == "simt":
        monkeypatch.setenv("TI_CRT_K3", "simt")
    L21 = _rand((n, k), 7100 + n, 1.0).cuda()
    W0 = _rand((n, n), 7200 + n).cuda()
    full = W0.clone()
    ti.crt_matmul_update(full, L21, L21.T, alpha=-1, moduli="wide")
    low = W0.clone()
    ti.crt_matmul_update(low, L21, L21.T, alpha=-1, moduli="wide", lower=True)
    mask = torch.ones(n, n, dtype=torch.bool, device="cuda").tril()
    assert torch.equal(full[mask].view(torch.int64), low[mask].view(torch.int64))


# ---------------------------------------------------------------------------------------
# residue GEMM on CTA pairs (tcgen05.mma.cta_group::2, K >= 1024) against the one-CTA kernel
# ---------------------------------------------------------------------------------------
def _both_gemm_kernels(monkeypatch, fn):
    monkeypatch.setenv("TI_GEMM_PAIR", "1")
    got = fn()
    torch.cuda.synchronize()
    monkeypatch.setenv("TI_GEMM_PAIR", "0")
    want = fn()
    torch.cuda.synchronize()
    monkeypatch.delenv("TI_GEMM_PAIR")
    return got, want


@pytest.mark.parametrize("m,n,k,moduli", [
    (256, 256, 1024, "wide"), (300, 700, 1100, None), (257, 513, 2048, None),
    (1000, 260, 1024, "wide"), (129, 1030, 4100, "wide"),
])
def test_pair_gemm_matches_one_cta(ti, monkeypatch, m, n, k, moduli):
    A = _rand((m, k), 181, 1.0).cuda()
    B = _rand((k, n), 182, 1.0).cuda()
    got, want = _both_gemm_kernels(monkeypatch, lambda: ti.crt_matmul(A, B, moduli=moduli))
    _assert_bitexact(got, want.cpu().numpy())


def test_pair_gemm_lower_update(ti, monkeypatch):
    n, k = 700, 1024
    L = _rand((n, k), 191).cuda()
    C0 = _rand((n, n), 192).cuda()

    def upd():
        C = C0.clone()
        ti.crt_matmul_update(C, L, L.T, alpha=-1, moduli="wide", lower=True)
        return C

    got, want = _both_gemm_kernels(monkeypatch, upd)
    _assert_bitexact(torch.tril(got), torch.tril(want).cpu().numpy())


def test_pair_gemm_int32_partials(ti, monkeypatch):
    """ti_crt_residue_partial writes int32 residue products (the sharded-k path)."""
    from tensor_inv_b200 import _native as nat

    m, n, k, n_mod, bits = 300, 260, 1100, 25, 53
    A = _rand((m, k), 201, 1.0).cuda()
    B = _rand((k, n), 202, 1.0).cuda()
    cm = importlib.import_module("tensor_inv_b200.crt_matmul")
    re, _ = cm._split(A, bits, n_mod, axis_k=1)
    ce, _ = cm._split(B, bits, n_mod, axis_k=0)

    def partial():
        out = torch.zeros((n_mod, m, n), dtype=torch.int32, device="cuda")
        ws_b = ctypes.c_size_t(0)
        nat.check("ws", nat.lib().ti_crt_residue_partial_workspace_size(m, n, k, n_mod,
                                                                      ctypes.byref(ws_b)))
        ws = torch.empty(max(ws_b.value, 256), dtype=torch.uint8, device="cuda")
        nat.check("partial", nat.lib().ti_crt_residue_partial(
            A.data_ptr(), k, 1, B.data_ptr(), n, 1, m, n, k, bits, n_mod,
            re.int().contiguous().data_ptr(), ce.int().contiguous().data_ptr(), out.data_ptr(),
            ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream))
        return out

    got, want = _both_gemm_kernels(monkeypatch, partial)
    assert torch.equal(got, want)
