"""tensor_inv_b200: B200-native (sm_100a) CRT-emulated float64 matmul for tensor_inv.

Drop-in for the reference package's public API (src/tensor_inv/__init__.py:1-6):
``crt_matmul``, ``lu``, ``cholesky``, ``rsvd``.  The compute path is the C-ABI library
``libtensor_inv_crt.so`` (hand-written CUDA for sm_100a); there is no CPU fallback.
"""

from tensor_inv_b200.cholesky import cholesky
from tensor_inv_b200.crt_matmul import crt_matmul, crt_matmul_update
from tensor_inv_b200.lu import lu
from tensor_inv_b200.rsvd import rsvd

__all__ = ["cholesky", "crt_matmul", "crt_matmul_update", "lu", "rsvd"]
