"""``tensor_inv.lu`` (src/tensor_inv/lu.py), bound to tensor_inv_b200's."""

from tensor_inv_b200.lu import lu  # noqa: F401
