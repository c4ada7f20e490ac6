"""ctypes binding of ``libtensor_inv_crt.so`` (the C ABI in ``include/tensor_inv_crt.h``).

The library is the only compute path: there is no CPU or PyTorch fallback.  Loading it
needs no GPU (so the CPU test suite can check its exports); every compute entry point
returns ``TI_ERR_NO_DEVICE`` unless an sm_100 device is current.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libtensor_inv_crt.so"

TI_OK = 0
TI_ERR_INVALID_ARGUMENT = 1
TI_ERR_UNSUPPORTED = 2
TI_ERR_WORKSPACE = 3
TI_ERR_CUDA = 4
TI_ERR_DEVICE_TIMEOUT = 5
TI_ERR_NO_DEVICE = 6
TI_ERR_SCRATCH_LIMIT = 7

TI_OUT_STORE = 0
TI_OUT_SUBTRACT = 1
TI_OUT_ADD = 2

TI_MODULI_PRIMES = 0
TI_MODULI_WIDE = 1

TI_NONFINITE_EXP = -(2**31)
TI_MAX_K = 135263
TI_MAX_K_WIDE = 133144

# name -> (restype, argtypes); mirrors include/tensor_inv_crt.h
_i64, _int, _p, _sz = ctypes.c_int64, ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t


class CrtOptions(ctypes.Structure):
    """ti_crt_options_t."""

    _fields_ = [("moduli", ctypes.c_int), ("n_moduli", ctypes.c_int),
                ("stage_events", ctypes.c_void_p * 4), ("bands", ctypes.c_int),
                ("lower", ctypes.c_int)]


_opt = ctypes.POINTER(CrtOptions)
SIGNATURES = {
    "ti_status_string": (ctypes.c_char_p, [_int]),
    "ti_version": (ctypes.c_char_p, []),
    "ti_n_moduli": (_int, [_i64, _int, ctypes.POINTER(_int)]),
    "ti_primes": (ctypes.POINTER(ctypes.c_int32), []),
    "ti_crt_workspace_size": (_int, [_i64, _i64, _i64, _int, ctypes.POINTER(_sz)]),
    "ti_crt_split": (_int, [_p, _i64, _i64, _i64, _i64, _int, _int, _p, _p, _i64, _p]),
    "ti_batched_gemm_workspace_size": (_int, [_i64, _i64, _i64, _i64, ctypes.POINTER(_sz)]),
    "ti_batched_int8_gemm_mod": (_int, [_p, _p, _p, _i64, _i64, _i64, _i64, _p, _p, _sz, _p]),
    "ti_crt_reconstruct": (_int, [_p, _p, _int, _int, _p, _p, _i64, _i64, _p, _i64, _p]),
    "ti_crt_matmul": (_int, [_p, _i64, _i64, _p, _i64, _i64, _p, _i64, _i64, _i64, _i64, _int,
                             _int, _p, _sz, _p]),
    "ti_crt_matmul_events": (_int, [_p, _i64, _i64, _p, _i64, _i64, _p, _i64, _i64, _i64, _i64,
                                    _int, _int, _p, _sz, _p, _p]),
    "ti_crt_matmul_noalloc": (_int, [_p, _i64, _i64, _p, _i64, _i64, _p, _i64, _i64, _i64,
                                     _i64, _int, _int, _p]),
    "ti_crt_plan": (_int, [_i64, _int, _opt, ctypes.POINTER(_int), ctypes.POINTER(_int),
                           ctypes.POINTER(ctypes.c_int32)]),
    "ti_crt_workspace_size_ex": (_int, [_i64, _i64, _i64, _int, _opt, ctypes.POINTER(_sz)]),
    "ti_crt_matmul_ex": (_int, [_p, _i64, _i64, _p, _i64, _i64, _p, _i64, _i64, _i64, _i64, _int,
                                _int, _p, _sz, _p, _opt]),
    "ti_crt_host_workspace_size": (_int, [_i64, _i64, _i64, _int, _opt, ctypes.POINTER(_sz)]),
    "ti_crt_matmul_host": (_int, [_p, _i64, _i64, _p, _i64, _i64, _p, _i64, _i64, _i64, _i64,
                                  _int, _p, _sz, _p, _opt]),
    "ti_device_error": (_int, [ctypes.POINTER(_int), _int]),
    "ti_selftest_bounded_wait": (_int, [_int, ctypes.c_longlong, _p]),
    "ti_crt_residue_partial_workspace_size": (_int, [_i64, _i64, _i64, _int,
                                                     ctypes.POINTER(_sz)]),
    "ti_crt_residue_partial": (_int, [_p, _i64, _i64, _p, _i64, _i64, _i64, _i64, _i64, _int,
                                      _int, _p, _p, _p, _p, _sz, _p]),
    "ti_lu_panel_workspace_size": (_int, [ctypes.POINTER(_sz)]),
    "ti_lu_panel": (_int, [_p, _i64, _i64, _i64, _i64, _p, _p, _sz, _p]),
    "ti_lu_panel_ex": (_int, [_p, _i64, _i64, _i64, _i64, _i64, _i64, _p, _p, _sz, _p]),
}

_lib = None


class NativeError(RuntimeError):
    """A non-zero ti_status_t from the library."""

    def __init__(self, fn: str, status: int):
        self.status = status
        super().__init__(f"{fn} failed: {status_string(status)} (status {status})")


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH.name} is not built; run `python -m tensor_inv_b200._build` "
                "(nvcc for sm_100a). tensor_inv_b200 has no CPU fallback.")
        L = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def status_string(status: int) -> str:
    return lib().ti_status_string(int(status)).decode()


def check(fn: str, status: int) -> None:
    if status != TI_OK:
        raise NativeError(fn, status)


def n_moduli(k: int, bits: int) -> int:
    out = ctypes.c_int(0)
    st = lib().ti_n_moduli(int(k), int(bits), ctypes.byref(out))
    if st == TI_ERR_UNSUPPORTED:
        raise ValueError(f"not enough primes for inner dim {k}, bits {bits}")
    check("ti_n_moduli", st)
    return out.value


def primes() -> list[int]:
    p = lib().ti_primes()
    return [int(p[i]) for i in range(30)]


def crt_workspace_size(m: int, n: int, k: int, bits: int) -> int:
    out = ctypes.c_size_t(0)
    check("ti_crt_workspace_size", lib().ti_crt_workspace_size(m, n, k, bits, ctypes.byref(out)))
    return out.value


def options(moduli=None, n_moduli=None, events=None, bands=0, lower=False) -> CrtOptions:
    """ti_crt_options_t from Python values: moduli None/'primes' or 'wide'; bands 0 = auto;
    lower: only C[r][c] with r >= c is needed."""
    if moduli in (None, "primes"):
        kind = TI_MODULI_PRIMES
    elif moduli == "wide":
        kind = TI_MODULI_WIDE
    else:
        raise ValueError(f"moduli must be None, 'primes' or 'wide', got {moduli!r}")
    n = 0 if n_moduli is None else int(n_moduli)
    if n < 0:
        raise ValueError("n_moduli must be positive")
    o = CrtOptions(kind, n)
    o.bands = int(bands)
    o.lower = 1 if lower else 0
    if events is not None:
        for i, e in enumerate(events):
            o.stage_events[i] = e
    return o


def crt_plan(k: int, bits: int, moduli=None, n_moduli=None):
    """(n_moduli, bits kept, moduli list) that ti_crt_matmul_ex uses for inner dimension k."""
    o = options(moduli, n_moduli)
    n = ctypes.c_int(0)
    b = ctypes.c_int(0)
    mods = (ctypes.c_int32 * 32)()
    st = lib().ti_crt_plan(int(k), int(bits), ctypes.byref(o), ctypes.byref(n), ctypes.byref(b),
                           mods)
    if st == TI_ERR_UNSUPPORTED:
        limit = TI_MAX_K if moduli in (None, "primes") else TI_MAX_K_WIDE
        if k > limit:
            raise ValueError(f"inner dim {k} exceeds {limit}, the bound that keeps the int32 "
                             f"residue accumulators exact for moduli {moduli or 'primes'!r}")
        most = 16 if moduli == "wide" else 25
        if n_moduli is not None and n_moduli > most:
            raise ValueError(f"n_moduli {n_moduli} exceeds the {most} moduli of the "
                             f"{moduli or 'primes'!r} set that the reconstruction takes (the "
                             f"product of the moduli must stay below 2^128)")
        raise ValueError(f"no moduli plan for inner dim {k}, bits {bits}, moduli {moduli!r}, "
                         f"n_moduli {n_moduli!r}")
    check("ti_crt_plan", st)
    return n.value, b.value, [int(mods[i]) for i in range(n.value)]


def crt_workspace_size_ex(m: int, n: int, k: int, bits: int, opt: CrtOptions) -> int:
    out = ctypes.c_size_t(0)
    check("ti_crt_workspace_size_ex",
          lib().ti_crt_workspace_size_ex(m, n, k, bits, ctypes.byref(opt), ctypes.byref(out)))
    return out.value


def batched_gemm_workspace_size(batch: int, M: int, K: int, N: int) -> int:
    out = ctypes.c_size_t(0)
    check("ti_batched_gemm_workspace_size",
          lib().ti_batched_gemm_workspace_size(batch, M, K, N, ctypes.byref(out)))
    return out.value


def device_error(reset: bool = True) -> int:
    out = ctypes.c_int(0)
    check("ti_device_error", lib().ti_device_error(ctypes.byref(out), 1 if reset else 0))
    return out.value


def crt_host_workspace_size(m: int, n: int, k: int, bits: int, opt: CrtOptions) -> int:
    out = ctypes.c_size_t(0)
    check("ti_crt_host_workspace_size",
          lib().ti_crt_host_workspace_size(m, n, k, bits, ctypes.byref(opt), ctypes.byref(out)))
    return out.value


def lu_panel_workspace_size() -> int:
    out = ctypes.c_size_t(0)
    check("ti_lu_panel_workspace_size", lib().ti_lu_panel_workspace_size(ctypes.byref(out)))
    return out.value


def lu_panel(W, j: int, jb: int, piv, workspace, stream) -> None:
    """The unblocked LU panel on columns [j, jb) of the row-major float64 CUDA tensor W, with
    the int64 pivot vector piv, in one launch on `stream` (a torch.cuda.Stream)."""
    n = W.shape[0]
    check("ti_lu_panel", lib().ti_lu_panel(W.data_ptr(), W.stride(0), n, j, jb, piv.data_ptr(),
                                           workspace.data_ptr(), workspace.numel(),
                                           stream.cuda_stream))


def lu_panel_cols(W, j: int, jb: int, pc: int, piv, workspace, stream) -> None:
    """The LU panel of rows [j, n) held in columns [pc, pc + jb - j) of the row-major float64
    CUDA tensor W (n rows, any column count); row swaps exchange all of W's columns."""
    n, ncols = W.shape
    check("ti_lu_panel_ex", lib().ti_lu_panel_ex(W.data_ptr(), W.stride(0), n, ncols, j, jb, pc,
                                                 piv.data_ptr(), workspace.data_ptr(),
                                                 workspace.numel(), stream.cuda_stream))
