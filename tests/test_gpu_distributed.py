"""Row-sharded matmul on two GPUs over NCCL (skipped with fewer GPUs): each
rank's rows of C equal the single-GPU result bit for bit, for B replicated
and for B's slices broadcast from the root."""

import os
import queue
import socket
import time

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    from datetime import timedelta
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=timedelta(seconds=120))
    try:
        import ozaki_jax_b200 as oz
        from ozaki_jax_b200.distributed import (gather_rows, gram_rowsharded, matmul_rowsharded,
                                                matmul_rowsharded_host, residual_rowsharded,
                                                row_range)
        rng = np.random.RandomState(0)
        out = {}
        # K = 700: BF16 slices; K = 5000 (rho 19, 600 rows per rank): int8 codes
        for n, k, m in ((600, 700, 500), (1200, 5000, 600)):
            A, B = rng.randn(n, k), rng.randn(k, m)
            ref = oz.matmul(A, B, pipeline="ondevice")  # single-GPU result on this device
            r0, r1 = row_range(n, rank, world)
            Ad = torch.as_tensor(A[r0:r1]).to(dev)
            for src in ("replicated", "root"):
                Bd = torch.as_tensor(B).to(dev) if (src == "replicated" or rank == 0) else None
                C = matmul_rowsharded(Ad, Bd, b_source=src)
                full = gather_rows(C, n)
                out[(k, src)] = bool(np.array_equal(full.cpu().numpy(), ref))
            # host arrays, B uploaded in shares and all-gathered over NCCL
            Ch = matmul_rowsharded_host(A[r0:r1], B)
            out[(k, "host")] = bool(np.array_equal(Ch, ref[r0:r1]))
        # residual rows: no collective, the single-GPU rows bit for bit
        A = rng.randn(1000, 5000)
        X, Bv = rng.randn(5000, 16), rng.randn(1000, 16)
        ref = oz.residual(A, X, Bv, mode="ozaki")
        r0, r1 = row_range(1000, rank, world)
        out["residual"] = bool(np.array_equal(residual_rowsharded(A[r0:r1], X, Bv[r0:r1]),
                                              ref[r0:r1]))
        # gram with A's rows split: N = 3000 (BF16 slices), N = 6000 (int8 codes);
        # this rank's rows of G equal the single-GPU gram's bit for bit
        for n, k in ((3000, 300), (6000, 700)):
            A = rng.randn(n, k) * np.exp(rng.randn(1, k))
            ref = oz.gram(A, mode="ozaki")
            r0, r1 = row_range(n, rank, world)
            Gr = gram_rowsharded(torch.as_tensor(A[r0:r1]).to(dev))
            c0, c1 = row_range(k, rank, world)
            out[("gram", n)] = bool(np.array_equal(Gr.cpu().numpy(), ref[c0:c1]))
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_rowsharded_matmul_two_gpus():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = []
    deadline = time.monotonic() + 300
    while len(res) < len(procs):
        try:
            res.append(q.get(timeout=5))
        except queue.Empty:
            dead = [p.exitcode for p in procs if p.exitcode not in (None, 0)]
            assert not dead, f"a rank exited with {dead}"
            assert time.monotonic() < deadline, "ranks did not finish"
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for _, out in res:
        assert len(out) == 9 and all(out.values()), out
