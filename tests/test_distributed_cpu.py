"""Multi-rank host logic on CPU (gloo, world_size 2): row partitioning, the
root broadcast and the row gather the row-sharded matmul uses.  The per-rank
compute is stood in by NumPy here; the GPU path is tested in
test_gpu_distributed.py."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, n, k, m, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from ozaki_jax_b200.distributed import broadcast_, gather_rows, row_range
        rng = np.random.RandomState(0)
        A = rng.randn(n, k)
        B = rng.randn(k, m)
        r0, r1 = row_range(n, rank, world)
        # B given on the root only: broadcast it
        Bt = torch.as_tensor(B if rank == 0 else np.zeros_like(B))
        broadcast_(Bt, src=0)
        C_local = torch.as_tensor(A[r0:r1] @ Bt.numpy())
        C_all = gather_rows(C_local, n)
        C_root = gather_rows(C_local, n, dst=0)
        ok = np.allclose(C_all.numpy(), A @ B, rtol=0, atol=1e-12)
        ok_root = (C_root is None) if rank != 0 else np.allclose(C_root.numpy(), A @ B, atol=1e-12)
        q.put((rank, bool(ok), bool(ok_root), r0, r1))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n", [10, 7, 1])
def test_rowsharded_logic_gloo_world2(n):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, n, 5, 3, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    res.sort()
    assert all(ok and okr for _, ok, okr, _, _ in res)
    # the blocks tile [0, n) without overlap
    assert res[0][3] == 0 and res[0][4] == res[1][3] and res[1][4] == n


def test_row_range_partition():
    from ozaki_jax_b200.distributed import row_range
    for n in (0, 1, 7, 8192, 8193):
        for world in (1, 2, 3, 8):
            blocks = [row_range(n, r, world) for r in range(world)]
            assert blocks[0][0] == 0 and blocks[-1][1] == n
            assert all(b[1] == c[0] for b, c in zip(blocks, blocks[1:]))
            sizes = [b[1] - b[0] for b in blocks]
            assert max(sizes) - min(sizes) <= 1
