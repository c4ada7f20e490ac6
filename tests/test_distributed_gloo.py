"""2-D sharded CRT matmul on world_size 2 and 4 gloo ranks (CPU, no GPU).

The block compute is the CPU oracle here (the product itself needs a B200); what is under
test is the sharding: block ranges, the panel broadcasts from one rank, the no-collective
block product, and the all-gather of C, which must reproduce the single-process result
bit for bit.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, m, n, k, out_q):
    import torch.distributed as dist

    from oracle import oracle
    from tensor_inv_b200 import distributed as D

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        A = B = None
        if rank == 0:
            g = torch.Generator().manual_seed(5)
            A = torch.randn(m, k, generator=g, dtype=torch.float64)
            B = torch.randn(k, n, generator=g, dtype=torch.float64) * 1e3
        Ap, Bp = D.scatter_panels(A, B, m, n, k, src=0)
        (r0, r1), (c0, c1) = D.my_ranges(m, n, rank, world)
        assert Ap.shape == (r1 - r0, k) and Bp.shape == (k, c1 - c0)
        Cb = D.crt_matmul_2d(Ap, Bp, matmul=lambda a, b: torch.from_numpy(
            oracle.crt_matmul(a.numpy(), b.numpy(), 53)))
        C = D.gather_blocks(Cb, m, n)
        if rank == 0:
            out_q.put(C.numpy().copy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_matches_single_process(oracle, world):
    m, n, k = 300, 270, 90
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, m, n, k, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        C = q.get(timeout=120)  # read before joining: a child that queued data exits only
    finally:                    # once its data has been read
        for p in procs:
            p.join(timeout=60)
        codes = [p.exitcode for p in procs]
        for p in procs:
            if p.is_alive():
                p.kill()
    assert codes == [0] * world, codes
    g = torch.Generator().manual_seed(5)
    A = torch.randn(m, k, generator=g, dtype=torch.float64)
    B = torch.randn(k, n, generator=g, dtype=torch.float64) * 1e3
    want = oracle.crt_matmul(A.numpy(), B.numpy(), 53)
    assert np.array_equal(C.view(np.uint64), want.view(np.uint64))


def test_grid_and_ranges():
    from tensor_inv_b200 import distributed as D

    assert [D.grid_shape(w) for w in (1, 2, 4, 8, 6, 9)] == [(1, 1), (1, 2), (2, 2), (2, 4),
                                                            (2, 3), (3, 3)]
    for size, parts in [(8192, 2), (8192, 4), (1000, 3), (100, 4), (5, 8)]:
        cuts = [D.block_range(size, parts, i) for i in range(parts)]
        assert cuts[0][0] == 0 and cuts[-1][1] == size
        assert all(a[1] == b[0] for a, b in zip(cuts, cuts[1:]))
        assert all(c[0] % 128 == 0 for c in cuts if c[0] < size)
    covered = np.zeros((1000, 700), int)
    for r in range(8):
        (r0, r1), (c0, c1) = D.my_ranges(1000, 700, r, 8)
        covered[r0:r1, c0:c1] += 1
    assert (covered == 1).all()


def _sharded_k_worker(rank, world, port, k_local, out_q):
    import torch.distributed as dist

    from tensor_inv_b200 import distributed as D

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        A = torch.ones(2, k_local, dtype=torch.float64)
        B = torch.ones(k_local, 3, dtype=torch.float64)
        try:
            D.crt_matmul_sharded_k(A, B)
            out_q.put((rank, "no error"))
        except ValueError as e:
            out_q.put((rank, f"ValueError: {e}"))
        except Exception as e:  # noqa: BLE001 - reported to the parent
            out_q.put((rank, f"{type(e).__name__}: {e}"))
    finally:
        dist.destroy_process_group()


def test_sharded_k_total_inner_dim_bound():
    """Each rank's slice (70000) is within the accumulator bound, but the whole inner dimension
    (140000) is not: every rank raises the single-GPU crt_matmul's ValueError, before any
    device work."""
    world, k_local = 2, 70000
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_sharded_k_worker, args=(r, world, port, k_local, q))
             for r in range(world)]
    for p in procs:
        p.start()
    try:
        got = dict(q.get(timeout=120) for _ in range(world))
    finally:
        for p in procs:
            p.join(timeout=60)
        for p in procs:
            if p.is_alive():
                p.kill()
    assert sorted(got) == [0, 1]
    for msg in got.values():
        assert msg.startswith("ValueError") and "140000 exceeds 135263" in msg, msg


def _grid_host_worker(rank, world, port, bands, out_q):
    import torch.distributed as dist

    from oracle import oracle
    from tensor_inv_b200 import distributed as D

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        pr, pc = D.grid_shape(world)
        i, j = D.grid_coords(rank, world)
        rows_g, cols_g = D.grid_groups()
        mb, nb, k = 96, 70, 60          # one rank's C block, the inner dimension
        g = torch.Generator().manual_seed(9)
        A = torch.randn(pr * mb, k, generator=g, dtype=torch.float64)  # the whole operands,
        B = torch.randn(k, pc * nb, generator=g, dtype=torch.float64)  # rebuilt on every rank
        Ap = A[i * mb:(i + 1) * mb]                      # this rank's A row panel
        Bp = B[:, j * nb:(j + 1) * nb]                   # and B column panel
        r = mb // bands // pc
        A_slices = torch.stack([Ap[b * pc * r + j * r: b * pc * r + (j + 1) * r]
                                for b in range(bands)])
        B_slice = Bp[i * (k // pr):(i + 1) * (k // pr)]
        C = D.crt_matmul_grid_host(A_slices, B_slice, row_group=rows_g[i], col_group=cols_g[j],
                                   matmul=lambda a, b: torch.from_numpy(
                                       oracle.crt_matmul(a.numpy(), b.numpy(), 53)),
                                   device="cpu")
        want = oracle.crt_matmul(Ap.numpy(), Bp.numpy(), 53)
        out_q.put((rank, bool(np.array_equal(C.numpy().view(np.uint64), want.view(np.uint64)))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,bands", [(2, 4), (4, 2)])
def test_grid_host_product_matches_the_blocks(oracle, world, bands):
    """Host-resident operands, each byte on one rank: every rank's C block, assembled from band
    gathers over its grid row and a B gather over its grid column, equals the oracle's product
    of the rank's panels bit for bit."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_grid_host_worker, args=(r, world, port, bands, q))
             for r in range(world)]
    for p in procs:
        p.start()
    try:
        got = dict(q.get(timeout=120) for _ in range(world))
    finally:
        for p in procs:
            p.join(timeout=60)
        for p in procs:
            if p.is_alive():
                p.kill()
    assert got == {r: True for r in range(world)}, got
