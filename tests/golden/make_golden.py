"""Generate golden fixtures from the reference implementation itself.

Run where the reference package is importable, with the reference's ``src`` directory on
the path::

    PYTHONPATH=<the reference's src> python tests/golden/make_golden.py

Each case runs the reference's own CPU path (``tensor_inv.crt_matmul``) stage by stage
and stores every intermediate in ``tests/golden/<case>.npz``:

``A``, ``B``      float64 inputs (exact images of the dtype the case names)
``bits``          precision bits the reference picked for that dtype
``moduli``        the moduli (``_PRIMES[:n]``)
``row_exp``,
``col_exp``       ``_scale_to_int`` exponents
``a_res``,
``b_res``         ``_residues`` of A (N,m,k) and B (N,k,n), int8
``c_res``         ``_matmul_residues`` on CPU, int32 (N,m,n)
``out``           ``crt_matmul(A, B)`` float64

plus ``n_moduli.npz`` with ``_n_moduli(k, bits)`` over a grid of k.  The fixtures are
small (a few hundred KB in total) and are committed; this script is how they were made.
"""

from __future__ import annotations

import importlib
import math
from pathlib import Path

import numpy as np
import torch

ref = importlib.import_module("tensor_inv.crt_matmul")  # the reference module

OUT = Path(__file__).resolve().parent


def _dump(name, A, B, dtype):
    A = A.to(dtype)
    B = B.to(dtype)
    bits = ref._PRECISION_BITS[A.dtype]
    Ad, Bd = A.double(), B.double()
    n_mod = ref._n_moduli(Ad.shape[-1], bits)
    moduli = ref._PRIMES[:n_mod]
    A_int, B_int, row_exp, col_exp = ref._scale_to_int(Ad, Bd, bits)
    a_res = ref._residues(A_int, moduli)
    b_res = ref._residues(B_int, moduli)
    c_res = torch.stack(ref._matmul_residues(a_res, b_res, moduli))
    out = ref.crt_matmul(A, B)
    np.savez_compressed(
        OUT / f"{name}.npz",
        A=Ad.numpy(), B=Bd.numpy(), bits=np.int32(bits), moduli=np.asarray(moduli, np.int32),
        row_exp=row_exp.numpy().astype(np.int32), col_exp=col_exp.numpy().astype(np.int32),
        a_res=a_res.numpy(), b_res=b_res.numpy(), c_res=c_res.numpy().astype(np.int32),
        out=out.numpy(), dtype=str(dtype).replace("torch.", ""),
    )
    print(f"{name}: {tuple(A.shape)} x {tuple(B.shape)} {dtype} N={n_mod}")


def main():
    # tests/test_crt.py:7-12 inputs
    torch.manual_seed(42)
    A = torch.randn(37, 51, dtype=torch.float64)
    B = torch.randn(51, 29, dtype=torch.float64)
    _dump("crt37x51x29_fp64", A, B, torch.float64)
    _dump("crt37x51x29_fp32", A, B, torch.float32)

    # wide exponent spread: (U(0,1) - 0.5) * exp(phi * N(0,1)), phi = 2
    g = torch.Generator().manual_seed(7)
    def spread(r, c, phi):
        u = torch.rand(r, c, generator=g, dtype=torch.float64) - 0.5
        return u * torch.exp(phi * torch.randn(r, c, generator=g, dtype=torch.float64))
    _dump("spread_phi2_32x300x40", spread(32, 300, 2.0), spread(300, 40, 2.0), torch.float64)
    _dump("spread_phi05_48x130x40", spread(48, 130, 0.5), spread(130, 40, 0.5), torch.float64)

    # zero rows/cols, huge and tiny rows, subnormal and signed-zero entries
    g.manual_seed(11)
    A = torch.randn(16, 40, generator=g, dtype=torch.float64)
    B = torch.randn(40, 12, generator=g, dtype=torch.float64)
    A[3] = 0.0
    A[5] *= 1e-200
    A[6] *= 1e200
    A[7, 2] = 5e-324
    A[8] = -0.0
    A[9, :] = 3e-310
    B[:, 4] = 0.0
    B[:, 7] *= 1e-250
    B[:, 9] *= 1e100  # 1e200 * 1e100 stays finite; an overflow raises in the reference
    _dump("edge_rows_16x40x12", A, B, torch.float64)

    # rounding ties in the scaling step: row max 1.0 -> scale 2^52, entries (2j+1)/2 ulp
    A = torch.zeros(6, 24, dtype=torch.float64)
    A[:, 0] = 1.0
    for j in range(1, 24):
        A[:, j] = (2 * j + 1) * 2.0**-53 * (1 if j % 2 else -1) + (j % 3) * 2.0**-51
    B = torch.randn(24, 5, generator=g, dtype=torch.float64)
    B[0] = 0.75
    _dump("ties_6x24x5", A, B, torch.float64)

    # subnormal outputs: the final ldexp rounds a second time
    A = torch.randn(24, 33, generator=g, dtype=torch.float64) * 1e-160
    B = torch.randn(33, 20, generator=g, dtype=torch.float64) * 1e-155
    B[:, 3] *= 1e-3
    _dump("subnormal_out_24x33x20", A, B, torch.float64)

    # reduced precision inputs
    A = torch.randn(20, 33, generator=g, dtype=torch.float64)
    B = torch.randn(33, 17, generator=g, dtype=torch.float64)
    _dump("bf16_20x33x17", A, B, torch.bfloat16)
    _dump("fp16_20x33x17", A, B, torch.float16)

    # degenerate shapes
    _dump("k1_5x1x6", torch.randn(5, 1, generator=g, dtype=torch.float64),
          torch.randn(1, 6, generator=g, dtype=torch.float64), torch.float64)
    _dump("one_1x7x1", torch.randn(1, 7, generator=g, dtype=torch.float64),
          torch.randn(7, 1, generator=g, dtype=torch.float64), torch.float64)

    # k > 1024: N = 24 moduli
    _dump("k1100_16x1100x12", torch.randn(16, 1100, generator=g, dtype=torch.float64),
          torch.randn(1100, 12, generator=g, dtype=torch.float64), torch.float64)

    ks = np.unique(np.concatenate([np.arange(0, 300), 2 ** np.arange(0, 18),
                                   2 ** np.arange(0, 18) - 1, 2 ** np.arange(0, 18) + 1,
                                   [7000, 7100, 7131, 7132, 7200, 8192, 65536, 135263]]))
    table = np.array([[k, b, ref._n_moduli(int(k), b)] for b in (8, 11, 24, 53) for k in ks],
                     np.int64)
    np.savez_compressed(OUT / "n_moduli.npz", table=table)
    print("n_moduli table", table.shape, "torch", torch.__version__, "python math", math.__name__)


if __name__ == "__main__":
    main()
