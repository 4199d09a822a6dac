"""Row-sharded matmul on two GPUs over NCCL (skipped with fewer GPUs): each
rank's rows of C equal the single-GPU result bit for bit, for B replicated
and for B's slices broadcast from the root."""

import os
import socket

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
        from ozaki_jax_b200.distributed import gather_rows, matmul_rowsharded, row_range
        rng = np.random.RandomState(0)
        A, B = rng.randn(600, 700), rng.randn(700, 500)
        ref = oz.matmul(A, B, pipeline="ondevice")  # single-GPU result on this device
        r0, r1 = row_range(600, rank, world)
        Ad = torch.as_tensor(A[r0:r1]).to(dev)
        out = {}
        for src in ("replicated", "root"):
            Bd = torch.as_tensor(B).to(dev) if (src == "replicated" or rank == 0) else None
            C = matmul_rowsharded(Ad, Bd, b_source=src)
            full = gather_rows(C, 600)
            out[src] = bool(np.array_equal(full.cpu().numpy(), ref))
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
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for _, out in res:
        assert out == {"replicated": True, "root": True}
