"""Products over a sharded inner dimension and row-sharded rSVD: two ranks (gloo) on one GPU,
checked bit for bit against the single-process results."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _same(a, b):
    return torch.equal(a.contiguous().view(torch.int64), b.contiguous().view(torch.int64))


def _worker(rank, world, port, case):
    import torch.distributed as dist

    import tensor_inv_b200 as ti
    from tensor_inv_b200 import distributed as D

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.cuda.set_device(0)
        if case == "sharded_k":
            g = torch.Generator().manual_seed(21)
            m, k, n = 150, 777, 90
            A = torch.randn(m, k, generator=g, dtype=torch.float64)
            B = torch.randn(k, n, generator=g, dtype=torch.float64)
            A[:, 5] *= 1e200   # a huge column that only rank 0 holds
            cuts = [0, 300, k]  # uneven split of the inner dimension
            k0, k1 = cuts[rank], cuts[rank + 1]
            got = D.crt_matmul_sharded_k(A[:, k0:k1].cuda(), B[k0:k1].cuda())
            want = ti.crt_matmul(A.cuda(), B.cuda())
            assert _same(got, want), "sharded-k product differs"
            # an empty slice on one rank (all of k on the other)
            A_e = A[:, :0] if rank == 0 else A
            B_e = B[:0] if rank == 0 else B
            got_e = D.crt_matmul_sharded_k(A_e.cuda(), B_e.cuda())
            assert _same(got_e, want), "sharded-k product with an empty slice differs"
            # a transposed view on the left (the rSVD shapes: Q^T B with Q's rows sharded)
            Q = torch.randn(k, 12, generator=g, dtype=torch.float64)
            got2 = D.crt_matmul_sharded_k(Q[k0:k1].cuda().T, B[k0:k1].cuda())
            assert _same(got2, ti.crt_matmul(Q.cuda().T, B.cuda())), "Q^T B differs"
        else:
            g = torch.Generator().manual_seed(22)
            m, n = 1001, 300
            A = torch.randn(m, n, generator=g, dtype=torch.float64).cuda()
            cuts = [0, 600, m]
            torch.manual_seed(5)
            U, S, Vt = D.rsvd_rows(A[cuts[rank]:cuts[rank + 1]], rank=16, n_power_iter=2)
            torch.manual_seed(5)
            U1, S1, Vt1 = ti.rsvd(A, rank=16, n_power_iter=2)
            assert _same(S, S1) and _same(Vt, Vt1), "S or Vt differs"
            assert _same(U, U1[cuts[rank]:cuts[rank + 1]]), "U rows differ"
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("case", ["sharded_k", "rsvd"])
def test_two_ranks_bit_identical(case):
    mp.spawn(_worker, args=(2, _free_port(), case), nprocs=2, join=True)
