"""Python handle on the CPU oracle (``liboracle_crt.so``, built from ``oracle_crt.c``).

TEST INFRASTRUCTURE ONLY: imported by ``tests/``, ``__graft_entry__.smoke()`` and the
CPU legs of ``bench.py`` as the checker.  The product package never imports it.

Each wrapper restates one function of the reference module
``src/tensor_inv/crt_matmul.py`` on numpy arrays:

=====================  ==============================================
``n_moduli``           ``_n_moduli``            crt_matmul.py:20-29
``split``              ``_scale_to_int`` +
                       ``_residues``            crt_matmul.py:32-46
``residue_gemm``       ``_matmul_residues``     crt_matmul.py:49-59
``crt_reconstruct``    ``_crt_reconstruct``     crt_matmul.py:62-92
``crt_matmul``         ``crt_matmul``           crt_matmul.py:95-120
``crt_matmul_moduli``  the same with explicit moduli and precision
=====================  ==============================================
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "liboracle_crt.so"
NONFINITE_EXP = -(2**31)

PRIMES = [
    3, 5, 7, 11, 13, 17, 19, 23, 29, 31, 37, 41, 43, 47, 53,
    59, 61, 67, 71, 73, 79, 83, 89, 97, 101, 103, 107, 109, 113, 127,
]  # fmt: skip
PRECISION_BITS = {"float16": 11, "bfloat16": 8, "float32": 24, "float64": 53}

_lib = None


def build(force: bool = False) -> Path:
    """Compile the oracle with its Makefile (gcc + OpenMP)."""
    if force or not _LIB_PATH.exists() or (
        _LIB_PATH.stat().st_mtime < (_HERE / "oracle_crt.c").stat().st_mtime
    ):
        subprocess.run(["make", "-s", "-C", str(_HERE), "-B" if force else "liboracle_crt.so"],
                       check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(str(_LIB_PATH))
        i64, i32, p = ctypes.c_int64, ctypes.c_int, ctypes.c_void_p
        L.or_n_moduli.argtypes = [i64, i32]
        L.or_n_moduli.restype = i32
        L.or_split.argtypes = [p, i64, i64, i64, i64, i32, i32, p, p, p]
        L.or_split.restype = None
        L.or_residue_gemm.argtypes = [p, p, i32, p, i64, i64, i64, p]
        L.or_residue_gemm.restype = None
        L.or_crt_reconstruct.argtypes = [p, i32, p, i32, p, p, i64, i64, p, i64]
        L.or_crt_reconstruct.restype = i32
        L.or_crt_matmul.argtypes = [p, i64, i64, p, i64, i64, i64, i64, i64, i32, p, i64]
        L.or_crt_matmul.restype = i32
        L.or_crt_matmul_moduli.argtypes = [p, i64, i64, p, i64, i64, i64, i64, i64, p, i32, i32,
                                           p, i64]
        L.or_crt_matmul_moduli.restype = i32
        _lib = L
    return _lib


def _ptr(a: np.ndarray):
    return ctypes.c_void_p(a.ctypes.data)


def n_moduli(k: int, bits: int) -> int:
    n = lib().or_n_moduli(int(k), int(bits))
    if n < 0:
        raise ValueError(f"not enough primes for inner dim {k}, bits {bits}")
    return n


def split(X: np.ndarray, bits: int, n_mod: int, axis_k: int):
    """Exponents and residues of one operand.

    ``axis_k`` is the reduction axis: 1 for A (rows are the outer vectors), 0 for B
    (columns are the outer vectors).  Returns ``(exp int32[outer], res int8[n_mod, outer, k])``.
    """
    X = np.asarray(X, dtype=np.float64)
    outer_axis = 1 - axis_k
    outer, kdim = X.shape[outer_axis], X.shape[axis_k]
    s = [st // 8 for st in X.strides]
    exp = np.empty(outer, np.int32)
    res = np.empty((n_mod, outer, kdim), np.int8)
    moduli = np.asarray(PRIMES[:n_mod], np.int32)
    lib().or_split(_ptr(X), outer, kdim, s[outer_axis], s[axis_k], bits, n_mod, _ptr(moduli),
                   _ptr(exp), _ptr(res))
    return exp, res


def residue_gemm(a_res: np.ndarray, b_res: np.ndarray, moduli) -> np.ndarray:
    """``(a_res[i] @ b_res[i]) mod moduli[i]``: a_res [N,m,k], b_res [N,k,n] -> int32 [N,m,n]."""
    a_res = np.ascontiguousarray(a_res, np.int8)
    b_res = np.ascontiguousarray(b_res, np.int8)
    N, m, k = a_res.shape
    n = b_res.shape[2]
    moduli = np.asarray(moduli, np.int32)
    out = np.empty((N, m, n), np.int32)
    lib().or_residue_gemm(_ptr(a_res), _ptr(b_res), N, _ptr(moduli), m, n, k, _ptr(out))
    return out


def crt_reconstruct(residues: np.ndarray, moduli, bits: int, row_exp, col_exp) -> np.ndarray:
    residues = np.ascontiguousarray(residues, np.int32)
    N, rows, cols = residues.shape
    moduli = np.asarray(moduli, np.int32)
    re = np.ascontiguousarray(row_exp, np.int32)
    ce = np.ascontiguousarray(col_exp, np.int32)
    out = np.empty((rows, cols), np.float64)
    rc = lib().or_crt_reconstruct(_ptr(residues), N, _ptr(moduli), bits, _ptr(re), _ptr(ce),
                                  rows, cols, _ptr(out), cols)
    if rc != 0:
        raise ValueError("bad moduli")
    return out


def crt_matmul(A: np.ndarray, B: np.ndarray, bits: int = 53) -> np.ndarray:
    """Full CPU path for float64 A (m,k) and B (k,n), any strides."""
    A = np.asarray(A, dtype=np.float64)
    B = np.asarray(B, dtype=np.float64)
    m, k = A.shape
    k2, n = B.shape
    assert k == k2
    out = np.empty((m, n), np.float64)
    sa = [s // 8 for s in A.strides]
    sb = [s // 8 for s in B.strides]
    rc = lib().or_crt_matmul(_ptr(A), sa[0], sa[1], _ptr(B), sb[0], sb[1], m, n, k, bits,
                             _ptr(out), n)
    if rc == -1:
        raise ValueError(f"not enough primes for inner dim {k}, bits {bits}")
    if rc != 0:
        raise MemoryError("oracle allocation failed")
    return out


def set_threads(n: int) -> None:
    """Threads of the oracle's parallel loops, whatever OMP_NUM_THREADS says (a launcher such
    as torchrun sets it to 1 for every process)."""
    os.environ["OMP_NUM_THREADS"] = str(n)
    L = lib()
    L.or_set_threads.argtypes = [ctypes.c_int]
    L.or_set_threads.restype = None
    L.or_set_threads(int(n))


def crt_matmul_moduli(A: np.ndarray, B: np.ndarray, moduli, bits: int) -> np.ndarray:
    """The reference algorithm with an explicit moduli set (pairwise coprime, < 256) and
    precision ``bits`` in place of ``_PRIMES[:n]`` and ``_PRECISION_BITS[dtype]``."""
    A = np.asarray(A, dtype=np.float64)
    B = np.asarray(B, dtype=np.float64)
    m, k = A.shape
    n = B.shape[1]
    mods = np.asarray(moduli, np.int32)
    out = np.empty((m, n), np.float64)
    sa = [s // 8 for s in A.strides]
    sb = [s // 8 for s in B.strides]
    rc = lib().or_crt_matmul_moduli(_ptr(A), sa[0], sa[1], _ptr(B), sb[0], sb[1], m, n, k,
                                    _ptr(mods), len(mods), bits, _ptr(out), n)
    if rc != 0:
        raise ValueError(f"oracle failed ({rc})")
    return out


# ---------------------------------------------------------------------------------------
# The exactly rounded product (the accuracy reference; not part of the reference's path)
# ---------------------------------------------------------------------------------------
_SPLIT = 134217729.0  # 2^27 + 1: Veltkamp's splitter for binary64


def _two_product(a: np.ndarray, b: np.ndarray):
    """p + e == a * b exactly, elementwise (Dekker's product with Veltkamp's split), valid while
    nothing overflows or underflows: |a|, |b| < 2^995 and every partial product, down to
    2^-106 |a b|, above the normal range's floor (callers check |a b| >= 2^-900)."""
    c = _SPLIT * a
    ah = c - (c - a)
    al = a - ah
    c = _SPLIT * b
    bh = c - (c - b)
    bl = b - bh
    p = a * b
    e = ((ah * bh - p) + ah * bl + al * bh) + al * bl
    return p, e


def exact_rounded_matmul(A: np.ndarray, B: np.ndarray) -> np.ndarray:
    """float64 C[i, j] = the exact sum_k A[i, k] * B[k, j], rounded once to nearest-even.

    Every product is split exactly into two doubles (p + e), and math.fsum returns the
    correctly rounded sum of its (exact) inputs, so the result is the rounding of the exact
    rational dot product.  Entries whose products leave the range where the split is exact
    fall back to exact rational arithmetic (fractions.Fraction).  For the sizes of a sample
    (a few thousand entries at k = 8192) this takes seconds."""
    import math
    from fractions import Fraction

    A = np.ascontiguousarray(A, np.float64)
    B = np.ascontiguousarray(B, np.float64)
    m, k = A.shape
    k2, n = B.shape
    assert k == k2
    out = np.empty((m, n), np.float64)
    Bt = np.ascontiguousarray(B.T)
    for i in range(m):
        a = A[i]
        for j in range(n):
            b = Bt[j]
            prod = a * b
            mag = np.abs(prod)
            safe = (np.all(np.isfinite(prod)) and np.abs(a).max(initial=0.0) < 2.0**995
                    and np.abs(b).max(initial=0.0) < 2.0**995
                    and not np.any((mag > 0) & (mag < 2.0**-900)))
            if safe:
                p, e = _two_product(a, b)
                out[i, j] = math.fsum(np.concatenate([p, e]).tolist())
            else:
                out[i, j] = float(sum(Fraction(x) * Fraction(y) for x, y in
                                      zip(a.tolist(), b.tolist())))
    return out
