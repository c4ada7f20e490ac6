"""The CPU oracle against fixtures produced by the reference itself (no GPU).

Pins ``oracle/oracle_crt.c`` bit for bit to the reference's CPU path, stage by stage:
exponents, int8 residues, int32 residue products and the float64 output.
"""

import numpy as np
import pytest

from conftest import GOLDEN, golden_cases


def _load(case):
    return dict(np.load(GOLDEN / f"{case}.npz"))


@pytest.mark.parametrize("case", golden_cases())
def test_split_matches_reference(oracle, case):
    g = _load(case)
    n_mod = len(g["moduli"])
    re, ar = oracle.split(g["A"], int(g["bits"]), n_mod, axis_k=1)
    ce, brt = oracle.split(g["B"], int(g["bits"]), n_mod, axis_k=0)
    np.testing.assert_array_equal(re, g["row_exp"])
    np.testing.assert_array_equal(ce, g["col_exp"])
    np.testing.assert_array_equal(ar, g["a_res"])
    np.testing.assert_array_equal(brt.transpose(0, 2, 1), g["b_res"])


@pytest.mark.parametrize("case", golden_cases())
def test_residue_gemm_matches_reference(oracle, case):
    g = _load(case)
    c = oracle.residue_gemm(g["a_res"], g["b_res"], g["moduli"])
    np.testing.assert_array_equal(c, g["c_res"])


@pytest.mark.parametrize("case", golden_cases())
def test_crt_reconstruct_matches_reference(oracle, case):
    g = _load(case)
    out = oracle.crt_reconstruct(g["c_res"], g["moduli"], int(g["bits"]), g["row_exp"],
                                 g["col_exp"])
    np.testing.assert_array_equal(out.view(np.uint64), g["out"].view(np.uint64))


@pytest.mark.parametrize("case", golden_cases())
def test_full_path_matches_reference(oracle, case):
    g = _load(case)
    out = oracle.crt_matmul(g["A"], g["B"], int(g["bits"]))
    np.testing.assert_array_equal(out.view(np.uint64), g["out"].view(np.uint64))
    # transposed storage of both operands gives the same bits
    out_t = oracle.crt_matmul(np.asfortranarray(g["A"]), np.asfortranarray(g["B"]),
                              int(g["bits"]))
    np.testing.assert_array_equal(out_t.view(np.uint64), g["out"].view(np.uint64))


def test_n_moduli_table(oracle):
    table = np.load(GOLDEN / "n_moduli.npz")["table"]
    for k, bits, n in table:
        assert oracle.n_moduli(int(k), int(bits)) == n, (k, bits)
    with pytest.raises(ValueError):
        oracle.n_moduli(2**62, 53)


def test_planted_mistake_is_caught(oracle):
    """A one-ulp error planted in the oracle's output must fail the bit-exact check."""
    g = _load("crt37x51x29_fp64")
    out = oracle.crt_matmul(g["A"], g["B"], int(g["bits"]))
    bad = out.copy()
    bad.view(np.uint64)[3, 4] += 1
    assert not np.array_equal(bad.view(np.uint64), g["out"].view(np.uint64))


def test_exact_rounded_matmul_against_fractions(oracle):
    """The accuracy reference (exactly rounded dot products) against exact rationals, on
    wide-spread inputs, ties-prone integers, cancellation and the rational fallback."""
    from fractions import Fraction

    rng = np.random.default_rng(3)
    cases = []
    for phi in (0.5, 2.0, 6.0):
        A = (rng.random((5, 300)) - 0.5) * np.exp(phi * rng.standard_normal((5, 300)))
        B = (rng.random((300, 4)) - 0.5) * np.exp(phi * rng.standard_normal((300, 4)))
        cases.append((A, B))
    A = rng.standard_normal((3, 50))
    cases.append((np.vstack([A, -A]), np.vstack([A, A]).T))           # exact cancellation
    cases.append((np.full((2, 3), 2.0**53 + 1.0), np.full((3, 2), 1.0 + 2.0**-52)))
    cases.append((np.array([[1e-200, 3.0]]), np.array([[1e-200], [1.0]])))  # fallback path
    for A, B in cases:
        got = oracle.exact_rounded_matmul(A, B)
        want = np.array([[float(sum(Fraction(x) * Fraction(y) for x, y in zip(A[i], B[:, j])))
                          for j in range(B.shape[1])] for i in range(A.shape[0])])
        assert np.array_equal(got.view(np.uint64), want.view(np.uint64))
