"""``tensor_inv.rsvd`` (src/tensor_inv/rsvd.py), bound to tensor_inv_b200's."""

from tensor_inv_b200.rsvd import rsvd  # noqa: F401
