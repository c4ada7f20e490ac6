"""The reference's own GPU path, built from its source, for context timing only.

TEST INFRASTRUCTURE ONLY (like the rest of ``oracle/``): the product package never imports
it; ``bench.py --impl reference`` uses it to time the reference's CUDA branch on the B200
beside its CPU path.

``build()`` compiles the reference's ``src/tensor_inv/csrc/crt_kernel.cu`` -- the file its
``_cuda_crt.py`` JIT-compiles with ``torch.utils.cpp_extension.load`` (``_cuda_crt.py:12-20``)
-- unmodified, where it lies in the reference tree, into ``oracle/_ref/`` (git-ignored; the
built module travels with the repository to a GPU machine, where the reference tree is
absent).  It needs the reference tree, so it runs only where that tree is present.

``crt_matmul_ref_gpu(A, B)`` restates the reference's CUDA branch around that module, step
for step: the torch scaling and residues of ``_scale_to_int`` / ``_residues``
(``crt_matmul.py:32-46``), the padding to multiples of 4 and the cuBLASLt batched int8 GEMM
with its in-place mod reduce (``_cuda_crt.py:44-79``, ``crt_kernel.cu:17-91``), and the
double-double reconstruction with weights split into three doubles (``_cuda_crt.py:23-41,
82-109``, ``crt_kernel.cu:93-125``).  That reconstruction is approximate, unlike the CPU
path's exact one, which is why its error is reported beside this library's.
"""

from __future__ import annotations

import importlib.machinery
import importlib.util
import math
import os
from pathlib import Path

_HERE = Path(__file__).resolve().parent
REF_DIR = _HERE / "_ref"
MODULE = "crt_cuda"  # the name the reference loads its extension under
REFERENCE_SOURCE = Path("/root/reference/src/tensor_inv/csrc/crt_kernel.cu")

_PRIMES = [3, 5, 7, 11, 13, 17, 19, 23, 29, 31, 37, 41, 43, 47, 53,
           59, 61, 67, 71, 73, 79, 83, 89, 97, 101, 103, 107, 109, 113, 127]

_module = None


def built_path() -> Path | None:
    hits = sorted(REF_DIR.glob(f"{MODULE}*.so"))
    return hits[0] if hits else None


def build(verbose: bool = False) -> Path | None:
    """Compile the reference's extension for sm_100a into oracle/_ref (None when the reference
    tree is absent, as on a GPU machine, where the module built here is used)."""
    if not REFERENCE_SOURCE.exists():
        return built_path()
    so = built_path()
    if so is not None and so.stat().st_mtime >= REFERENCE_SOURCE.stat().st_mtime:
        return so
    REF_DIR.mkdir(exist_ok=True)
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
    from torch.utils.cpp_extension import load

    load(name=MODULE, sources=[str(REFERENCE_SOURCE)], build_directory=str(REF_DIR),
         extra_cuda_cflags=["-O3"], verbose=verbose)
    return built_path()


def module():
    """The compiled reference extension (torch must be imported first)."""
    global _module
    if _module is None:
        import torch  # noqa: F401 - the extension links against the loaded torch

        so = built_path()
        if so is None:
            raise RuntimeError("the reference's crt_kernel extension is not built "
                               "(oracle.ref_gpu.build() where the reference tree is present)")
        loader = importlib.machinery.ExtensionFileLoader(MODULE, str(so))
        spec = importlib.util.spec_from_file_location(MODULE, str(so), loader=loader)
        mod = importlib.util.module_from_spec(spec)
        loader.exec_module(mod)
        _module = mod
    return _module


def _n_moduli(k: int, bits: int) -> int:
    target = 2 * k * (1 << (2 * bits))
    prod = 1
    for i, p in enumerate(_PRIMES):
        prod *= p
        if prod > target:
            return i + 1
    raise ValueError(f"not enough primes for inner dim {k}, bits {bits}")


def _weights_three_doubles(moduli):
    """CRT weights W_i = M_i (M_i^-1 mod m_i) as hi + mid + lo doubles, and M as hi + lo."""
    big_m = math.prod(moduli)
    hi, mid, lo = [], [], []
    for p in moduli:
        mi = big_m // p
        w = mi * pow(mi, -1, p)
        h = float(w)
        rest = w - int(h)
        md = float(rest)
        hi.append(h)
        mid.append(md)
        lo.append(float(rest - int(md)))
    m_hi = float(big_m)
    return hi, mid, lo, m_hi, float(big_m - int(m_hi)), 1.0 / m_hi


def crt_matmul_ref_gpu(A, B, bits: int = 53):
    """C = A @ B through the reference's CUDA branch (float64 CUDA tensors in and out)."""
    import torch
    import torch.nn.functional as F

    mod = module()
    dev = A.device
    k = A.shape[1]
    moduli = _PRIMES[:_n_moduli(k, bits)]
    # scaling and residues, in torch, on the device
    row_e = A.abs().amax(dim=-1).clamp(min=1e-300).frexp()[1]
    col_e = B.abs().amax(dim=-2).clamp(min=1e-300).frexp()[1]
    a_int = torch.ldexp(A, bits - row_e.unsqueeze(-1)).round().to(torch.int64)
    b_int = torch.ldexp(B, bits - col_e.unsqueeze(-2)).round().to(torch.int64)
    mt = torch.tensor(moduli, dtype=torch.int64, device=dev)
    a_res = (a_int.unsqueeze(0) % mt.view(-1, 1, 1)).to(torch.int8)
    del a_int
    b_res = (b_int.unsqueeze(0) % mt.view(-1, 1, 1)).to(torch.int8)
    del b_int
    m, n = a_res.shape[-2], b_res.shape[-1]

    def pad4(x):
        pr, pc = (-x.shape[-2]) % 4, (-x.shape[-1]) % 4
        return x if pr == pc == 0 else F.pad(x, (0, pc, 0, pr))

    c = mod.batched_int8_gemm_mod(pad4(a_res).contiguous(), pad4(b_res).contiguous(),
                                  torch.tensor(moduli, dtype=torch.int32, device=dev))
    del a_res, b_res
    residues = [c[i, :m, :n] for i in range(len(moduli))]
    stack = torch.stack(residues).contiguous()
    del c, residues
    hi, mid, lo, m_hi, m_lo, inv_m = _weights_three_doubles(moduli)
    f64 = dict(dtype=torch.float64, device=dev)
    return mod.crt_reconstruct(stack, torch.tensor(hi, **f64), torch.tensor(mid, **f64),
                               torch.tensor(lo, **f64), m_hi, m_lo, inv_m,
                               row_e.int().contiguous(), col_e.int().contiguous(), 2 * bits,
                               m, n, len(moduli))
