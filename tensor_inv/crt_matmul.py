"""``tensor_inv.crt_matmul`` (src/tensor_inv/crt_matmul.py): the names the reference module
exports, including the private ones its notebooks import, bound to tensor_inv_b200's."""

from tensor_inv_b200.crt_matmul import (  # noqa: F401
    _PRECISION_BITS,
    _PRIMES,
    _crt_reconstruct,
    _matmul_residues,
    _n_moduli,
    crt_matmul,
)
