"""The kernels' bounded waits, made to run out on purpose.

Every wait in the library's kernels (mbarrier phases of the TMA/MMA/epilogue pipelines, the
LU panel's grid barrier) gives up after a time limit, records a code in the device error
word and lets the kernel return, instead of hanging the GPU.  Here a wait that nothing will
ever complete runs with a 1 ms limit: the call must come back with TI_ERR_DEVICE_TIMEOUT and
the matching code, and the context must stay usable (the next product bit-exact against the
oracle).
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

K_ERR_TIMEOUT_MMA = 0x102
K_ERR_TIMEOUT_GRID_BARRIER = 0x105


@pytest.mark.parametrize("which,code", [(0, K_ERR_TIMEOUT_MMA), (1, K_ERR_TIMEOUT_GRID_BARRIER)])
def test_wait_runs_out_and_context_survives(oracle, which, code):
    import tensor_inv_b200 as ti
    from tensor_inv_b200 import _native as nat

    assert nat.device_error(reset=True) == 0
    stream = torch.cuda.current_stream().cuda_stream
    st = nat.lib().ti_selftest_bounded_wait(which, 1_000_000, stream)
    assert st == nat.TI_ERR_DEVICE_TIMEOUT, nat.lib().ti_status_string(st)
    assert nat.device_error(reset=True) == code
    assert nat.device_error(reset=False) == 0

    g = torch.Generator().manual_seed(which)
    A = torch.randn(200, 300, generator=g, dtype=torch.float64)
    B = torch.randn(300, 150, generator=g, dtype=torch.float64)
    C = ti.crt_matmul(A.cuda(), B.cuda()).cpu().numpy()
    want = oracle.crt_matmul(A.numpy(), B.numpy(), 53)
    assert np.array_equal(C.view(np.uint64), want.view(np.uint64))
    torch.cuda.synchronize()
    assert nat.device_error(reset=True) == 0


def test_selftest_rejects_bad_arguments():
    from tensor_inv_b200 import _native as nat

    assert nat.lib().ti_selftest_bounded_wait(2, 1_000_000, None) == nat.TI_ERR_INVALID_ARGUMENT
    assert nat.lib().ti_selftest_bounded_wait(0, 10, None) == nat.TI_ERR_INVALID_ARGUMENT
