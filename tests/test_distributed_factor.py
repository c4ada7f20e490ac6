"""Block-cyclic LU and Cholesky (tensor_inv_b200.distributed) against one process.

CPU tests: world sizes 2 and 3 on gloo, trailing products through the CPU oracle (an exact
CRT product, so each output depends only on its own row and column, as on the GPU); every
rank compares the distributed P, L, U (or L) with a world-size-1 run of the same code.
GPU tests: two gloo ranks on one GPU against ``lu`` / ``cholesky`` of the whole matrix.
"""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _same(a, b):
    return torch.equal(a.contiguous().view(torch.int64), b.contiguous().view(torch.int64))


def _matrix(kind, n, seed, device="cpu"):
    g = torch.Generator().manual_seed(seed)
    X = torch.randn(n, n, generator=g, dtype=torch.float64)
    if kind == "spd":
        X = X @ X.T / n + 1e-3 * torch.eye(n, dtype=torch.float64)
    elif kind == "ties":
        X = torch.randint(-3, 4, (n, n), generator=g).to(torch.float64)
    return X.to(device)


def _cpu_worker(rank, world, port, kind, n, block, errs):
    import torch.distributed as dist

    from oracle import oracle
    from tensor_inv_b200 import distributed as D

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        def mm(a, b):
            return torch.from_numpy(oracle.crt_matmul(a.contiguous().numpy(),
                                                      b.contiguous().numpy(), 53))

        singles = [dist.new_group([r]) for r in range(world)]  # collective: every rank
        A = _matrix(kind, n, 40 + n)
        if kind == "spd":
            got = D.cholesky_distributed(A, block, matmul=mm)
            want = D.cholesky_distributed(A, block, group=singles[rank], matmul=mm)
            ok = _same(got, want)
        else:
            P, L, U = D.lu_distributed(A, block, matmul=mm)
            P1, L1, U1 = D.lu_distributed(A, block, group=singles[rank], matmul=mm)
            ok = _same(P, P1) and _same(L, L1) and _same(U, U1)
            if kind == "randn":
                ok = ok and float((P @ A - L @ U).abs().max()) < 1e-10 * float(A.abs().max())
        if not ok:
            errs.put(f"rank {rank}: {kind} n={n} b={block} differs")
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
@pytest.mark.parametrize("kind,n,block", [("randn", 50, 8), ("ties", 40, 8), ("spd", 45, 8),
                                          ("randn", 16, 32)])
def test_cyclic_factorizations_match_one_process(oracle, world, kind, n, block):
    ctx = mp.get_context("spawn")
    errs = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_cpu_worker, args=(r, world, port, kind, n, block, errs))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert errs.empty(), errs.get()


def test_cyclic_columns_partition():
    from tensor_inv_b200 import distributed as D

    n, b = 70, 8
    for world in (1, 2, 3, 4):
        cols = torch.cat([D.cyclic_columns(n, b, r, world) for r in range(world)])
        assert sorted(cols.tolist()) == list(range(n))
        for r in range(world):
            assert all((c // b) % world == r for c in D.cyclic_columns(n, b, r, world).tolist())


def _gpu_worker(rank, world, port, kind, n, block):
    import torch.distributed as dist

    import tensor_inv_b200 as ti
    from tensor_inv_b200 import distributed as D

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.cuda.set_device(0)
        A = _matrix(kind, n, 70 + n, "cuda")
        if kind == "spd":
            got = D.cholesky_distributed(A, block)
            assert _same(got, ti.cholesky(A, block_size=block)), "cholesky differs"
        else:
            P, L, U = D.lu_distributed(A, block)
            P1, L1, U1 = ti.lu(A, block_size=block)
            assert _same(P, P1) and _same(L, L1) and _same(U, U1), "lu differs"
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.parametrize("kind,n,block,world", [("randn", 700, 64, 2), ("ties", 300, 64, 2),
                                                ("spd", 650, 64, 2), ("randn", 1300, 256, 2),
                                                ("randn", 1100, 128, 3), ("spd", 1500, 128, 3)])
def test_cyclic_factorizations_gpu_match_one_gpu(kind, n, block, world):
    mp.spawn(_gpu_worker, args=(world, _free_port(), kind, n, block), nprocs=world, join=True)


def _cpu_fail_worker(rank, world, port, errs):
    import torch.distributed as dist

    from tensor_inv_b200 import distributed as D

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        A = -torch.eye(24, dtype=torch.float64)  # not positive definite
        try:
            D.cholesky_distributed(A, 8, matmul=lambda a, b: a @ b)
            errs.put(f"rank {rank}: no error raised")
        except RuntimeError:
            pass
    finally:
        dist.destroy_process_group()


def test_cyclic_cholesky_failure_reaches_every_rank():
    """A panel that fails on its owner raises on every rank instead of leaving the others
    waiting in the next broadcast."""
    ctx = mp.get_context("spawn")
    errs = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_cpu_fail_worker, args=(r, 2, port, errs)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert errs.empty(), errs.get()


def test_row_permutation_moves_only_changed_rows():
    """The non-owners' row swaps: applying the owner's pivot vector by moving only the rows
    whose position changed equals the full permutation gather."""
    from tensor_inv_b200 import distributed as D

    g = torch.Generator().manual_seed(3)
    n, j, b = 40, 8, 6
    W = torch.randn(n, 5, generator=g, dtype=torch.float64)
    piv = torch.randperm(n, generator=g)
    new_piv = piv.clone()
    for k in range(j, j + b):  # the panel's swaps: row k with some row at or below it
        p = int(torch.randint(k, n, (1,), generator=g))
        new_piv[[k, p]] = new_piv[[p, k]]
    pos = D._inverse_perm(piv)
    want = W[pos[new_piv]]
    got = W.clone()
    D._apply_row_perm_(got, piv, new_piv, j, 2 * b)
    assert torch.equal(got, want)


def test_contiguous_runs():
    from tensor_inv_b200 import distributed as D

    assert D._contiguous_runs([], 4) == []
    assert D._contiguous_runs([3, 5, 7], 4) == [[3], [5], [7]]
    assert D._contiguous_runs(list(range(10)), 4) == [[0, 1, 2], [3, 4, 5], [6, 7, 8], [9]]
    assert sum(D._contiguous_runs(list(range(10)), 1), []) == list(range(10))
