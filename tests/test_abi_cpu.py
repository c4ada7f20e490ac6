"""Host-side checks of the C-ABI library and the Python front end (no GPU needed).

No compute entry point is called here: only symbol exports, the exact modulus count,
workspace sizing and the reference's error behaviour that triggers before any device work.
"""

import re
from pathlib import Path

import numpy as np
import pytest
import torch

from conftest import GOLDEN, ROOT


@pytest.fixture(scope="module")
def nat():
    from tensor_inv_b200 import _build, _native

    _build.build()
    return _native


def _declared_functions():
    text = (ROOT / "include" / "tensor_inv_crt.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(ti_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_entry_points():
    names = _declared_functions()
    for must in ["ti_crt_matmul", "ti_crt_split", "ti_batched_int8_gemm_mod",
                 "ti_crt_reconstruct", "ti_n_moduli", "ti_crt_workspace_size"]:
        assert must in names


def test_library_exports_every_declared_symbol(nat):
    lib = nat.lib()
    for name in _declared_functions():
        assert hasattr(lib, name), f"{name} declared in include/ but not exported"
    assert set(nat.SIGNATURES) == set(_declared_functions())


def test_n_moduli_matches_reference_table(nat):
    table = np.load(GOLDEN / "n_moduli.npz")["table"]
    from tensor_inv_b200.crt_matmul import _n_moduli

    for k, bits, n in table:
        assert _n_moduli(int(k), int(bits)) == n, (k, bits)
    with pytest.raises(ValueError):
        _n_moduli(2**62, 53)


def test_primes_and_strings(nat):
    from tensor_inv_b200.crt_matmul import _PRIMES

    assert nat.primes() == _PRIMES
    assert nat.status_string(0) == "ok"
    assert "device" in nat.status_string(nat.TI_ERR_NO_DEVICE)
    assert nat.lib().ti_version().decode().count(".") == 2


def test_workspace_sizes(nat):
    # 8192^3 at float64: 25 moduli x (A + B + product) int8 planes + exponents
    ws = nat.crt_workspace_size(8192, 8192, 8192, 53)
    assert 25 * 3 * 8192 * 8192 <= ws <= 25 * 3 * 8192 * 8192 + 4 * 2 * 8192 + 4096
    # the wide moduli need 16 planes instead of 25 at the same precision
    ws16 = nat.crt_workspace_size_ex(8192, 8192, 8192, 53, nat.options("wide"))
    assert 16 * 3 * 8192 * 8192 <= ws16 <= 16 * 3 * 8192 * 8192 + 4 * 2 * 8192 + 4096
    # 1024^3: A, B and product planes
    ws = nat.crt_workspace_size(1024, 1024, 1024, 53)
    assert 24 * 3 * 1024 * 1024 <= ws <= 24 * 3 * 1024 * 1024 + 4 * 2 * 1024 + 4096
    assert nat.crt_workspace_size(37, 29, 51, 53) > 0
    with pytest.raises(nat.NativeError):
        nat.crt_workspace_size(10, 10, nat.TI_MAX_K + 1, 53)
    with pytest.raises(nat.NativeError):
        nat.crt_workspace_size(10, 10, 10, 52)  # not a supported precision


def test_reference_errors_before_device_work(nat):
    from tensor_inv_b200 import crt_matmul

    A = torch.randn(4, 5, dtype=torch.float64)
    with pytest.raises(TypeError, match="unsupported dtype"):
        crt_matmul(A.int(), A.int())
    with pytest.raises(IndexError):
        crt_matmul(A[:, :0], A[:0])
    with pytest.raises(RuntimeError):
        crt_matmul(A, A)


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU behaviour")
def test_no_cpu_fallback(nat):
    from tensor_inv_b200 import crt_matmul

    with pytest.raises(RuntimeError, match="CUDA"):
        crt_matmul(torch.randn(3, 4, dtype=torch.float64), torch.randn(4, 2, dtype=torch.float64))


def test_product_does_not_import_oracle():
    pkg = ROOT / "tensor_inv_b200"
    for src in list(pkg.rglob("*.py")) + list(pkg.rglob("*.cu")) + list(pkg.rglob("*.cuh")):
        text = src.read_text()
        assert "oracle" not in re.sub(r"(#|//).*", "", text), src


def test_moduli_plans(nat):
    """Wide moduli: the fewest that keep 53 bits; a fixed count lowers the precision."""
    assert nat.crt_plan(8192, 53) == (25, 53, [3, 5, 7, 11, 13, 17, 19, 23, 29, 31, 37, 41,
                                                43, 47, 53, 59, 61, 67, 71, 73, 79, 83, 89, 97, 101])
    n, b, mods = nat.crt_plan(8192, 53, "wide")
    assert (n, b) == (16, 53) and mods[:4] == [255, 253, 251, 247]
    assert [nat.crt_plan(8192, 53, "wide", N)[1] for N in (12, 13, 14, 15, 16)] == [40, 44, 47,
                                                                                      51, 53]
    assert nat.crt_plan(1024, 53, "wide")[:2] == (15, 53)
    import math
    for N in range(1, 17):  # the wide moduli are pairwise coprime and below 2^127 together
        mods = nat.crt_plan(8, 53, "wide", N)[2]
        assert all(math.gcd(a, c) == 1 for i, a in enumerate(mods) for c in mods[i + 1:])
        assert math.prod(mods) < 2**127
    # counts past a set's size: a clear error (17 and 18 moduli come from the primes)
    with pytest.raises(ValueError, match="exceeds the 16 moduli"):
        nat.crt_plan(8192, 53, "wide", 17)
    with pytest.raises(ValueError, match="exceeds the 25 moduli"):
        nat.crt_plan(8192, 53, "primes", 26)
    assert [nat.crt_plan(8192, 53, "primes", N)[:2] for N in (17, 18)] == [(17, 30), (18, 33)]
