"""``tensor_inv.cholesky`` (src/tensor_inv/cholesky.py), bound to tensor_inv_b200's."""

from tensor_inv_b200.cholesky import cholesky  # noqa: F401
