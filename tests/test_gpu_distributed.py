"""Row-sharded matmul on two GPUs over NCCL (skipped with fewer GPUs): each
rank's rows of C equal the single-GPU result bit for bit, for B replicated,
B's slices broadcast from the root and B's column blocks all-gathered (also
with a ragged column split); a NaN in B on the root makes every rank raise;
and one process can drive both GPUs through one context."""

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
        from ozaki_jax_b200.distributed import (close_contexts, column_range, gather_rows,
                                                gram_rowsharded, matmul_rowsharded,
                                                matmul_rowsharded_host, residual_rowsharded,
                                                row_range)
        rng = np.random.RandomState(0)
        out = {}
        # K = 700: BF16 slices; K = 5000 (rho 19, 600 rows per rank): int8 codes
        for n, k, m in ((600, 700, 500), (1200, 5000, 601)):
            A, B = rng.randn(n, k), rng.randn(k, m)
            ref = oz.matmul(A, B, pipeline="ondevice")  # single-GPU result on this device
            r0, r1 = row_range(n, rank, world)
            Ad = torch.as_tensor(A[r0:r1]).to(dev)
            for src in ("replicated", "root", "columns"):
                if src == "columns":
                    c0, c1 = column_range(m, rank, world)  # 601 columns: 301 + 300
                    Bd = torch.as_tensor(np.ascontiguousarray(B[:, c0:c1])).to(dev)
                else:
                    Bd = torch.as_tensor(B).to(dev) if (src == "replicated" or rank == 0) else None
                C = matmul_rowsharded(Ad, Bd, b_source=src)
                full = gather_rows(C, n)
                out[(k, src)] = bool(np.array_equal(full.cpu().numpy(), ref))
            # host arrays, B uploaded in shares and all-gathered over NCCL
            Ch = matmul_rowsharded_host(A[r0:r1], B)
            out[(k, "host")] = bool(np.array_equal(Ch, ref[r0:r1]))
        # a NaN in B, held by the root only: every rank raises, as one GPU would
        A, B = rng.randn(600, 5000), rng.randn(5000, 300)
        B[17, 5] = np.nan
        r0, r1 = row_range(600, rank, world)
        try:
            matmul_rowsharded(torch.as_tensor(A[r0:r1]).to(dev),
                              torch.as_tensor(B).to(dev) if rank == 0 else None, b_source="root")
            out["nan_root_raises"] = False
        except ValueError as e:
            out["nan_root_raises"] = "NaN" in str(e)
        # residual rows: no collective, the single-GPU rows bit for bit
        A = rng.randn(1000, 5000)
        X, Bv = rng.randn(5000, 16), rng.randn(1000, 16)
        ref = oz.residual(A, X, Bv, mode="ozaki")
        r0, r1 = row_range(1000, rank, world)
        out["residual"] = bool(np.array_equal(residual_rowsharded(A[r0:r1], X, Bv[r0:r1]),
                                              ref[r0:r1]))
        # gram with A's rows split: N = 3000 (BF16 slices), N = 6000 (int8 codes);
        # this rank's rows of G equal the single-GPU gram's bit for bit
        # N = 3000 (BF16 slices): A's columns travel, bit for bit; N = 6000 (int8
        # codes): partial int64 Gram sums reduced over the ranks, each pair's term
        # rounded on each rank's part -- within FP64 rounding of the single-GPU gram
        for n, k in ((3000, 300), (6000, 700)):
            A = rng.randn(n, k) * np.exp(rng.randn(1, k))
            ref = oz.gram(A, mode="ozaki")
            r0, r1 = row_range(n, rank, world)
            Gr = gram_rowsharded(torch.as_tensor(A[r0:r1]).to(dev)).cpu().numpy()
            c0, c1 = row_range(k, rank, world)
            if n == 3000:
                out[("gram", n)] = bool(np.array_equal(Gr, ref[c0:c1]))
            else:
                bound = 4 * 2.0 ** -52 * (np.abs(A).T @ np.abs(A))[c0:c1]
                out[("gram", n)] = bool(np.all(np.abs(Gr - ref[c0:c1]) <= bound))
        q.put((rank, out))
    finally:
        close_contexts()
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
        assert len(out) == 12 and all(out.values()), out


def _local_worker(q):
    """One process, two GPUs, one context (ozk_context_create_local): the
    column-block mode through the C ABI, each GPU's rows against the
    single-GPU result."""
    import ctypes
    import ozaki_jax_b200 as oz
    from ozaki_jax_b200 import _lib as L
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    lib = L.load()
    rng = np.random.RandomState(3)
    n, k, m = 1024, 5000, 700
    A, B = rng.randn(n, k), rng.randn(k, m)
    ref = oz.matmul(A, B, pipeline="ondevice")
    ctx = ctypes.c_void_p()
    L.check(lib.ozk_context_create_local(ctypes.byref(ctx), 2, (ctypes.c_int * 2)(0, 1)))
    try:
        P = ctypes.c_void_p
        I64 = ctypes.c_int64
        mc = (m + 1) // 2
        As, Bs, Cs, sts = [], [], [], []
        for g in range(2):
            dev = torch.device("cuda", g)
            As.append(torch.as_tensor(A[g * n // 2:(g + 1) * n // 2]).to(dev))
            Bs.append(torch.as_tensor(np.ascontiguousarray(B[:, g * mc:min(m, (g + 1) * mc)]))
                      .to(dev))
            Cs.append(torch.empty((n // 2, m), dtype=torch.float64, device=dev))
            sts.append(torch.zeros(1, dtype=torch.int32, device=dev))
        streams = [torch.cuda.current_stream(torch.device("cuda", g)).cuda_stream
                   for g in range(2)]
        L.check(lib.ozk_matmul_f64_multi(
            ctx, (P * 2)(*[a.data_ptr() for a in As]), (I64 * 2)(k, k),
            (P * 2)(*[b.data_ptr() for b in Bs]), (I64 * 2)(*[b.shape[1] for b in Bs]),
            (P * 2)(*[c.data_ptr() for c in Cs]), (I64 * 2)(m, m), n, k, m, 4, 1,
            L.OZK_B_COLUMNS, 0, (P * 2)(*streams), (P * 2)(*[t.data_ptr() for t in sts])))
        full = np.concatenate([c.cpu().numpy() for c in Cs])
        q.put(bool(np.array_equal(full, ref)) and all(int(t.item()) == 0 for t in sts))
    finally:
        lib.ozk_context_destroy(ctx)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_one_process_two_gpus_local_context():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_local_worker, args=(q,))
    p.start()
    ok = q.get(timeout=300)
    p.join(timeout=120)
    assert p.exitcode == 0 and ok
