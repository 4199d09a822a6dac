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


def _bad_args_worker(rank, world, port, q):
    """Rank 1 passes operands whose K does not match; every rank must raise
    ValueError before any data collective (none may hang in one)."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    out = {}
    try:
        from ozaki_jax_b200.distributed import (_or_status, gram_rowsharded, matmul_rowsharded,
                                                matmul_rowsharded_host)
        k_a = 8 if rank == 0 else 9
        A = torch.zeros((4, k_a), dtype=torch.float64)
        B = torch.zeros((8, 5), dtype=torch.float64)
        for name, call in (
                ("replicated", lambda: matmul_rowsharded(A, B, b_source="replicated")),
                ("root", lambda: matmul_rowsharded(A, B if rank == 0 else None, b_source="root")),
                ("root_missing_B", lambda: matmul_rowsharded(torch.zeros((4, 8), dtype=torch.float64),
                                                             None if rank == 0 else B,
                                                             b_source="root")),
                ("host", lambda: matmul_rowsharded_host(A.numpy(), B.numpy())),
                ("gram", lambda: gram_rowsharded(torch.zeros((4, 3 + rank), dtype=torch.float64)))):
            try:
                call()
                out[name] = "returned"
            except ValueError as e:
                out[name] = "ValueError: " + str(e)
        # status words are OR-ed over the ranks
        st = torch.tensor([1 if rank == 0 else 4], dtype=torch.int32)
        out["or"] = _or_status(st, None)
        out["or_inplace"] = int(st.item())
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


def test_bad_arguments_on_one_rank_raise_on_every_rank_gloo_world2():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_bad_args_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=180) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank in (0, 1):
        out = res[rank]
        for name in ("replicated", "root", "root_missing_B", "host", "gram"):
            assert out[name].startswith("ValueError"), (rank, name, out[name])
        assert out["or"] == 5 and out["or_inplace"] == 5
