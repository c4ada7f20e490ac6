"""Drop-in ``crt_matmul`` module: the reference's Python API over the sm_100a kernels.

Mirrors ``src/tensor_inv/crt_matmul.py`` of the reference: the same public function
``crt_matmul(A, B)`` and the same module-level names (``_PRIMES``, ``_PRECISION_BITS``,
``_n_moduli``, ``_residues``-style stage helpers), the same argument meaning and the
same errors.  Every stage runs in ``libtensor_inv_crt.so``:

========================  =====================================  ==========================
reference                 here                                   C ABI
========================  =====================================  ==========================
crt_matmul.py:20-29       ``_n_moduli``                          ``ti_n_moduli``
crt_matmul.py:32-46       ``_split`` (scale + residues, fused)   ``ti_crt_split``
crt_matmul.py:49-59       ``_matmul_residues``                   ``ti_batched_int8_gemm_mod``
crt_matmul.py:73-92       ``_crt_reconstruct``                   ``ti_crt_reconstruct``
crt_matmul.py:95-120     ``crt_matmul``                         ``ti_crt_matmul``
========================  =====================================  ==========================

Results are bit-identical to the reference's CPU path for finite inputs.  CPU tensors are
copied to the current CUDA device and the result is copied back (a transfer, not a CPU
fallback); without an sm_100 GPU every call raises.
"""

from __future__ import annotations

import ctypes

import torch

from . import _native as nat

# crt_matmul.py:5-9 -- the moduli: the 30 odd primes below 128
# fmt: off
_PRIMES = [
    3, 5, 7, 11, 13, 17, 19, 23, 29, 31, 37, 41, 43, 47, 53,
    59, 61, 67, 71, 73, 79, 83, 89, 97, 101, 103, 107, 109, 113, 127,
]
# fmt: on

# crt_matmul.py:12-17 -- significand bits kept per input dtype
_PRECISION_BITS = {
    torch.float16: 11,
    torch.bfloat16: 8,
    torch.float32: 24,
    torch.float64: 53,
}


def _n_moduli(k, bits):
    """min primes whose product covers dot-product range (crt_matmul.py:20-29)"""
    return nat.n_moduli(int(k), int(bits))


def _stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _cuda_device(*tensors) -> torch.device:
    for t in tensors:
        if t.is_cuda:
            return t.device
    if not torch.cuda.is_available():
        raise RuntimeError(
            "tensor_inv_b200.crt_matmul needs a CUDA device (sm_100a); it has no CPU path")
    return torch.device("cuda", torch.cuda.current_device())


def _strides_2d(X: torch.Tensor):
    """Element strides with one of them 1, or None if X needs a copy."""
    s0, s1 = X.stride()
    if X.shape[1] <= 1:
        s1 = 1
    if X.shape[0] <= 1 and s1 != 1:
        s0 = 1
    if s1 == 1 or s0 == 1:
        return s0, s1
    return None


def _check_dtype(A):
    bits = _PRECISION_BITS.get(A.dtype)
    if bits is None:
        supported = ", ".join(str(d) for d in _PRECISION_BITS)
        raise TypeError(
            f"unsupported dtype {A.dtype}. "
            f"CRT matmul emulates floating-point precision via int8 arithmetic; "
            f"input must be a float type ({supported})"
        )
    return bits


def _launch_crt_matmul(A, B, C, bits, out_mode, opt=None):
    """C (op)= A @ B on the device of C; A, B float64 on the same device, C float64 with
    unit column stride; ``opt`` a ti_crt_options_t (None: the reference's moduli).  Returns C."""
    m, k = A.shape
    n = B.shape[1]
    dev = C.device
    sa = _strides_2d(A)
    if sa is None:
        A = A.contiguous()
        sa = A.stride()
    sb = _strides_2d(B)
    if sb is None:
        B = B.contiguous()
        sb = B.stride()
    if C.stride(1) != 1 and n > 1:
        raise ValueError("output must have unit column stride")
    ldc = C.stride(0) if m > 1 else max(n, 1)
    if opt is None:
        opt = nat.options()
    ws_bytes = nat.crt_workspace_size_ex(m, n, k, bits, opt)
    ws = torch.empty(max(ws_bytes, 256), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        st = nat.lib().ti_crt_matmul_ex(
            A.data_ptr(), sa[0], sa[1], B.data_ptr(), sb[0], sb[1], C.data_ptr(), ldc, m, n,
            k, bits, out_mode, ws.data_ptr(), ws.numel(), _stream_ptr(dev), ctypes.byref(opt))
    nat.check("ti_crt_matmul_ex", st)
    return C


def _options(k, bits, moduli, n_moduli):
    """Validated ti_crt_options_t; raises ValueError like _n_moduli when no plan exists."""
    if moduli in (None, "primes") and n_moduli is None:
        _n_moduli(k, bits)  # the reference's ValueError, unchanged
    nat.crt_plan(k, bits, moduli, n_moduli)
    return nat.options(moduli, n_moduli)


def crt_matmul(A, B, *, moduli=None, n_moduli=None):
    """FP-accurate matmul via int8 CRT. Precision matches input dtype.

    Same contract as the reference (crt_matmul.py:95-120): ``bits`` from ``A.dtype``,
    operands promoted to float64, result float64 on ``A``'s device.

    Keyword-only extensions (absent from the reference; the defaults are its scheme):
    ``moduli='wide'`` uses pairwise-coprime odd moduli up to 255 instead of the primes up
    to 127; with ``n_moduli=None`` it takes the fewest that keep every bit of the input
    precision, so the result is bit-identical with about a third fewer residue GEMMs.
    ``n_moduli=N`` fixes the count (a moduli-count sweep); if N moduli cannot hold
    the full precision, the scaling keeps the largest b with prod(moduli) > 2*k*2^(2b) bits.
    """
    bits = _check_dtype(A)
    if A.dim() != 2 or B.dim() != 2:
        raise ValueError(f"crt_matmul expects 2-D operands, got {tuple(A.shape)} and "
                         f"{tuple(B.shape)}")
    m, k = A.shape
    if k == 0:
        raise IndexError("amax(): Expected reduction dim -1 to have non-zero size.")
    if B.shape[0] != k:
        raise RuntimeError(f"crt_matmul: shapes {tuple(A.shape)} and {tuple(B.shape)} "
                           "cannot be multiplied")
    opt = _options(k, bits, moduli, n_moduli)  # ValueError as in the reference
    n = B.shape[1]
    home = A.device
    dev = _cuda_device(A, B)
    if home.type == "cpu" and B.device.type == "cpu":
        return _crt_matmul_host(A.to(torch.float64), B.to(torch.float64), bits, opt, dev)
    A = A.to(device=dev, dtype=torch.float64)
    B = B.to(device=dev, dtype=torch.float64)
    C = torch.empty((m, n), dtype=torch.float64, device=dev)
    if m and n:
        _launch_crt_matmul(A, B, C, bits, nat.TI_OUT_STORE, opt)
    if home == dev:
        return C
    if home.type == "cpu":
        # device -> pinned host copy (cached pinned blocks, full-bandwidth transfer)
        out = torch.empty((m, n), dtype=torch.float64, pin_memory=True)
        out.copy_(C)
        return out
    return C.to(home)


class _PinnedPool:
    """Reusable page-locked host blocks for results returned on the CPU.

    A fresh 512 MiB pinned allocation costs ~64 ms on a B200 host (more than the product
    itself) whenever the previous result is still alive, which is the common loop
    ``C = crt_matmul(A, B)``.  Each result is a view of a pooled block; a block is handed
    out again only when no tensor, view or numpy array refers to its storage any more
    (storage use count back to the pool's own references), so a live result is never
    overwritten.  Blocks beyond ``max_bytes`` in total are not pooled.
    """

    def __init__(self, max_bytes=8 << 30):
        import threading

        self._lock = threading.Lock()
        self._blocks = []
        self._max = max_bytes
        self._count = getattr(torch._C, "_storage_Use_Count", None)

    def _free(self, base):
        # references: the pool's tensor plus the temporary storage wrapper of this call
        return self._count(base.untyped_storage()._cdata) <= 2

    def empty(self, m, n):
        nbytes = 8 * m * n
        if self._count is None or nbytes == 0:
            return torch.empty((m, n), dtype=torch.float64, pin_memory=True)
        with self._lock:
            best = None
            for base in self._blocks:
                if base.numel() >= nbytes and self._free(base):
                    if best is None or base.numel() < best.numel():
                        best = base
            if best is None:
                best = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
                if sum(b.numel() for b in self._blocks) + nbytes <= self._max:
                    self._blocks.append(best)
            return best[:nbytes].view(torch.float64).view(m, n)


_pinned_pool = _PinnedPool()


def _crt_matmul_host(A, B, bits, opt, dev):
    """CPU operands: copies and kernels pipelined in row bands (ti_crt_matmul_host); the
    result lands in pinned host memory.  Synchronous, like the reference's CPU call."""
    m, k = A.shape
    n = B.shape[1]
    sa = _strides_2d(A)
    if sa is None:
        A = A.contiguous()
        sa = A.stride()
    sb = _strides_2d(B)
    if sb is None:
        B = B.contiguous()
        sb = B.stride()
    out = _pinned_pool.empty(m, n)
    if m == 0 or n == 0:
        return out
    ws_bytes = nat.crt_host_workspace_size(m, n, k, bits, opt)
    ws = torch.empty(max(ws_bytes, 256), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev)
        st = nat.lib().ti_crt_matmul_host(
            A.data_ptr(), sa[0], sa[1], B.data_ptr(), sb[0], sb[1], out.data_ptr(), n, m, n, k,
            bits, ws.data_ptr(), ws.numel(), stream.cuda_stream, ctypes.byref(opt))
        nat.check("ti_crt_matmul_host", st)
        stream.synchronize()  # A, B and the workspace stay alive until the copies are done
    return out


def caller_moduli(k):
    """The moduli set the callers (lu, cholesky, rsvd) use for an inner dimension k: the wide
    set whenever it keeps every bit (outputs bit-identical to the reference's primes, with
    about a third fewer residue GEMMs), else the reference's primes."""
    return "wide" if 0 < k <= nat.TI_MAX_K_WIDE else None


def crt_matmul_update(C, A, B, alpha=-1, *, moduli=None, n_moduli=None, lower=False):
    """In-place ``C += alpha * crt_matmul(A, B)`` for alpha in {-1, +1}, C float64 CUDA.

    Bit-identical to ``C -= crt_matmul(A, B)`` (alpha=-1) or ``C += crt_matmul(A, B)``:
    the product is rounded to float64 first, then one IEEE subtraction/addition, fused
    into the reconstruction kernel so no temporary product is materialised.  ``lower=True``
    guarantees only the elements C[r, c] with r >= c (the others may be left unchanged):
    output tiles entirely above the diagonal are skipped, about half the work of a
    symmetric update.
    """
    bits = _check_dtype(A)
    if alpha not in (-1, 1):
        raise ValueError("alpha must be -1 or +1")
    if C.dtype != torch.float64 or not C.is_cuda:
        raise TypeError("C must be a float64 CUDA tensor")
    m, k = A.shape
    if B.shape[0] != k or C.shape != (m, B.shape[1]):
        raise RuntimeError("crt_matmul_update: shape mismatch")
    if m == 0 or B.shape[1] == 0 or k == 0:
        return C
    opt = _options(k, bits, moduli, n_moduli)
    opt.lower = 1 if lower else 0
    A = A.to(device=C.device, dtype=torch.float64)
    B = B.to(device=C.device, dtype=torch.float64)
    return _launch_crt_matmul(A, B, C, bits,
                              nat.TI_OUT_SUBTRACT if alpha == -1 else nat.TI_OUT_ADD, opt)


# ---------------------------------------------------------------------------------------
# stage functions (for stage-by-stage parity with the reference)
# ---------------------------------------------------------------------------------------
def _split(X, bits, n_mod, axis_k):
    """Exponents and int8 residues of one float64 CUDA operand.

    Fuses the reference's ``_scale_to_int`` and ``_residues`` (crt_matmul.py:32-46).
    ``axis_k`` is the reduction axis (1 for A, 0 for B).  Returns ``(exp int32[outer],
    res int8[n_mod, outer, k])``, the residues of the rows of A or of the columns of B.
    """
    X = X.to(torch.float64)
    outer_axis = 1 - axis_k
    outer, kdim = X.shape[outer_axis], X.shape[axis_k]
    s = X.stride()
    s_outer, s_k = s[outer_axis], s[axis_k]
    if kdim <= 1:
        s_k = 1
    if not (s_k == 1 or s_outer == 1):
        X = X.contiguous()
        s = X.stride()
        s_outer, s_k = s[outer_axis], s[axis_k]
    ld = (max(kdim, 1) + 15) // 16 * 16
    exp = torch.empty(outer, dtype=torch.int32, device=X.device)
    res = torch.empty((n_mod, outer, ld), dtype=torch.int8, device=X.device)
    with torch.cuda.device(X.device):
        st = nat.lib().ti_crt_split(X.data_ptr(), outer, kdim, s_outer, s_k, bits, n_mod,
                                    exp.data_ptr(), res.data_ptr(), ld, _stream_ptr(X.device))
    nat.check("ti_crt_split", st)
    return exp, res[:, :, :kdim]


def _scale_to_int_exponents(A, B, bits):
    """The exponents of the reference's ``_scale_to_int`` (crt_matmul.py:32-38)."""
    n_mod = 1
    re, _ = _split(A, bits, n_mod, axis_k=1)
    ce, _ = _split(B, bits, n_mod, axis_k=0)
    return re, ce


def _matmul_residues(a_res, b_res, moduli):
    """per-prime int8 matmul + modular reduction (crt_matmul.py:49-59), on tcgen05.

    a_res (N, m, k) and b_res (N, k, n) int8 CUDA tensors; returns a list of N int32
    (m, n) tensors with values in [0, p).
    """
    a_res = a_res.contiguous()
    b_res = b_res.contiguous()
    N, m, k = a_res.shape
    n = b_res.shape[2]
    dev = a_res.device
    c = torch.empty((N, m, n), dtype=torch.int32, device=dev)
    mod_t = (ctypes.c_int32 * N)(*[int(p) for p in moduli])
    ws = torch.empty(max(nat.batched_gemm_workspace_size(N, m, k, n), 256), dtype=torch.uint8,
                     device=dev)
    with torch.cuda.device(dev):
        st = nat.lib().ti_batched_int8_gemm_mod(
            a_res.data_ptr(), b_res.data_ptr(), ctypes.cast(mod_t, ctypes.c_void_p), N, m, k, n,
            c.data_ptr(), ws.data_ptr(), ws.numel(), _stream_ptr(dev))
    nat.check("ti_batched_int8_gemm_mod", st)
    return list(c)


def _crt_reconstruct(residues, moduli, bits, row_exp, col_exp):
    """Exact CRT reconstruction (crt_matmul.py:73-92) of N int32 (rows, cols) residues."""
    res = torch.stack(list(residues)).to(torch.int32).contiguous()
    N, rows, cols = res.shape
    dev = res.device
    out = torch.empty((rows, cols), dtype=torch.float64, device=dev)
    mod_t = (ctypes.c_int32 * N)(*[int(p) for p in moduli])
    re = row_exp.to(device=dev, dtype=torch.int32).contiguous()
    ce = col_exp.to(device=dev, dtype=torch.int32).contiguous()
    with torch.cuda.device(dev):
        st = nat.lib().ti_crt_reconstruct(
            res.data_ptr(), ctypes.cast(mod_t, ctypes.c_void_p), N, bits, re.data_ptr(),
            ce.data_ptr(), rows, cols, out.data_ptr(), max(cols, 1), _stream_ptr(dev))
    nat.check("ti_crt_reconstruct", st)
    return out
