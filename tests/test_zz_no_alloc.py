"""ti_crt_matmul_noalloc: the CRT matmul for callers that cannot allocate device memory.

Callers such as a host program whose own allocator already owns the GPU's memory pool, or a
latency-critical caller that cannot pay for cudaMalloc's implicit device synchronisation,
use this entry point: it takes no workspace and runs on the library's static 64 MiB device
scratch.  These tests call it through the C ABI and require its output to equal, bit for
bit (the tolerance of every parity test here), the output of ti_crt_matmul with a caller
workspace, on two calls in a row with different shapes, so the second call runs on the
scratch the first one left behind.  This file is collected last on purpose and passes both
on its own in a fresh process and after the rest of the suite.
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def nat():
    from tensor_inv_b200 import _native

    assert torch.cuda.is_available()
    return _native


def _inputs(m, n, k, seed):
    g = torch.Generator().manual_seed(seed)
    u = torch.rand(m, k, generator=g, dtype=torch.float64) - 0.5
    A = u * torch.exp(torch.randn(m, k, generator=g, dtype=torch.float64))
    u = torch.rand(k, n, generator=g, dtype=torch.float64) - 0.5
    B = u * torch.exp(torch.randn(k, n, generator=g, dtype=torch.float64))
    return A.cuda(), B.cuda()


def _with_workspace(nat, A, B):
    m, k = A.shape
    n = B.shape[1]
    C = torch.empty((m, n), dtype=torch.float64, device="cuda")
    ws_bytes = nat.crt_workspace_size(m, n, k, 53)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    st = nat.lib().ti_crt_matmul(A.data_ptr(), k, 1, B.data_ptr(), n, 1, C.data_ptr(), n, m, n, k,
                                 53, nat.TI_OUT_STORE, ws.data_ptr(), ws_bytes,
                                 torch.cuda.current_stream().cuda_stream)
    nat.check("ti_crt_matmul", st)
    return C


def _no_alloc(nat, A, B):
    m, k = A.shape
    n = B.shape[1]
    C = torch.empty((m, n), dtype=torch.float64, device="cuda")
    st = nat.lib().ti_crt_matmul_noalloc(A.data_ptr(), k, 1, B.data_ptr(), n, 1, C.data_ptr(), n,
                                         m, n, k, 53, nat.TI_OUT_STORE,
                                         torch.cuda.current_stream().cuda_stream)
    nat.check("ti_crt_matmul_noalloc", st)
    return C


def _same_bits(x, y):
    a = x.cpu().numpy().view(np.uint64)
    b = y.cpu().numpy().view(np.uint64)
    return int((a != b).sum())


def test_no_alloc_matches_workspace_entry_point_twice(nat):
    # first call: 512^3 (24 moduli, 18 MiB of scratch); second call: a ragged 100 x 90 x 7200
    # product (25 moduli, 33 MiB) laid over what the first call left in the shared scratch
    for (m, n, k, seed) in [(512, 512, 512, 1), (100, 90, 7200, 2)]:
        A, B = _inputs(m, n, k, seed)
        want = _with_workspace(nat, A, B)
        got = _no_alloc(nat, A, B)
        torch.cuda.synchronize()
        assert _same_bits(got, want) == 0, (m, n, k)
    assert nat.device_error(reset=True) == 0


def test_no_alloc_rejects_problems_beyond_the_scratch(nat):
    m = n = k = 1024  # needs about 75 MB of scratch at float64
    assert nat.crt_workspace_size(m, n, k, 53) > 64 << 20
    A, B = _inputs(8, 8, 8, 3)  # never read: the size check comes first
    st = nat.lib().ti_crt_matmul_noalloc(A.data_ptr(), k, 1, B.data_ptr(), n, 1, A.data_ptr(), n,
                                         m, n, k, 53, nat.TI_OUT_STORE,
                                         torch.cuda.current_stream().cuda_stream)
    assert st == nat.TI_ERR_SCRATCH_LIMIT
    assert "scratch" in nat.status_string(st)
