"""The reference's import name, ``tensor_inv``, served by tensor_inv_b200.

Code written against the reference package (``from tensor_inv.crt_matmul import crt_matmul``,
``from tensor_inv.lu import lu``, ...) runs unchanged on the sm_100a path: every module here
re-exports the tensor_inv_b200 object of the same name (src/tensor_inv/__init__.py:1-6).
"""

from tensor_inv.cholesky import cholesky
from tensor_inv.crt_matmul import crt_matmul
from tensor_inv.lu import lu
from tensor_inv.rsvd import rsvd

__all__ = ["cholesky", "crt_matmul", "lu", "rsvd"]
