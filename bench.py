"""Benchmark of the on-device Ozaki matmul, headline configuration (c2):
C = A @ B, A, B 8192 x 8192 FP64 N(0,1) (RandomState(0): A then B),
precision='high' (n_hi=4, n_lo=1, 24 slice GEMMs), accumulation='fused'.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...   (one rank per GPU)

A step is one pass of the pipeline over one batch: split + slice extraction
of A (row block) and B, then the persistent slice-pair GEMM with the FP64
epilogue.  Multi-GPU: rank r owns rows [r N/P, (r+1) N/P) of A and C (the
row extraction is row-local, so sharded slices are identical), B is given to
every rank; total work is fixed (strong scaling), no collective sits in the
data path; timing is the max over ranks.  Inputs (1 GiB) exceed L2, so no
flush is needed between steps.

Rank 0 prints one JSON line.  `value` is FP64-equivalent TFLOP/s (2NKM/t)
with inputs resident in HBM; `e2e` is the same metric through the public
API (ozaki_jax_b200.matmul on pinned host NumPy arrays -> the C entry point
ozk_matmul_f64_hostbuf, which overlaps the PCIe copies with the compute in
row blocks), every copy inside the timed region;
`cpu_baseline` times the NumPy oracle (the reference's
matmul_numpy(pipeline='ondevice') restated) on a row sample on the host
cores.  --impl reference runs only that CPU reference arm.
"""

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "FP64-equiv TFLOP/s (2MNK/t) at 8192^3 high + normwise rel err"
PRESETS = {"high": (4, 1), "medium": (3, 1), "max": (5, 4)}


# DRAM bytes (read + write) of one slice-GEMM launch of the default workload,
# from one capture of this command on a B200:
#   ncu --metrics dram__bytes_read.sum,dram__bytes_write.sum --clock-control none \
#       -k regex:k_slice_gemm -c 1 python bench.py --steps 2 --warmup 1
# (11.90 GB read + 0.70 GB written).  Other workloads report null.
GEMM_TRAFFIC_BYTES = {(8192, "high", "int8"): 12.60e9}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d.get("bf16_tflops_sustained", 1413.4), d.get("hbm_gbs", 6449.7), "measured"
    return 1400.0, 6650.0, "fallback"


def int8_peak(dev, seconds=1.5):
    """Sustained int8 x int8 -> int32 GEMM rate of cuBLASLt (torch._int_mm) on
    this GPU: 8192^3 looped for about `seconds`, so under the same power cap as
    the slice GEMM -- the int8 counterpart of the measured BF16 peak, which
    MEASURED_PEAKS.json does not have.  Returns (TOP/s or None, source text)."""
    import torch

    try:
        n = 8192
        g = torch.Generator(device=dev)
        g.manual_seed(1)
        a = torch.randint(-64, 64, (n, n), dtype=torch.int8, device=dev, generator=g)
        b = torch.randint(-64, 64, (n, n), dtype=torch.int8, device=dev, generator=g).t()
        for _ in range(3):
            torch._int_mm(a, b)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(10):
            torch._int_mm(a, b)
        e1.record()
        torch.cuda.synchronize(dev)
        iters = max(10, int(seconds * 1e3 / (e0.elapsed_time(e1) / 10)))
        e0.record()
        for _ in range(iters):
            torch._int_mm(a, b)
        e1.record()
        torch.cuda.synchronize(dev)
        ms = e0.elapsed_time(e1) / iters
        return (2.0 * n ** 3 / (ms * 1e-3) / 1e12,
                f"cuBLASLt int8 GEMM (torch._int_mm) {n}^3, {iters} calls "
                f"({iters * ms / 1e3:.1f} s sustained), measured in this run")
    except Exception as e:  # noqa: BLE001 -- report, fall back to the BF16-derived figure
        return None, f"int8 GEMM unavailable ({type(e).__name__})"


def tensor_peak(s8, dev):
    """(peak, unit, source, extra fields) for the slice GEMM's roofline.  The
    int8 peak is 2x the BF16 one (NVIDIA's dense int8 rate is twice its BF16
    rate); cuBLASLt's own int8 GEMM, timed here as well, reaches less than
    that on B200, so it is reported beside it as context only."""
    bf16_peak, _, src = peaks()
    if not s8:
        return bf16_peak, "TFLOP/s", f"{src} sustained bf16", {}
    p, why = int8_peak(dev)
    return 2.0 * bf16_peak, "TOP/s", f"2x {src} sustained bf16 (int8 dense rate)", {
        "int8_library_gemm": p, "int8_library_gemm_source": why}


def make_inputs(n, k, m):
    rng = np.random.RandomState(0)
    A = rng.randn(n, k)
    B = rng.randn(k, m)
    return A, B


class Clocks:
    """Samples the SM clock and the clock-event reasons of one GPU during the
    timed region: NVML polled every few milliseconds (so short regions still
    get samples), nvidia-smi at 200 ms when NVML is unavailable.  Read only."""

    REASONS = {"hw_slowdown": "HwSlowdown", "hw_thermal_slowdown": "HwThermalSlowdown",
               "sw_thermal_slowdown": "SwThermalSlowdown", "sw_power_cap": "SwPowerCap",
               "hw_power_brake_slowdown": "HwPowerBrakeSlowdown"}
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []
        self.samples = []
        self.mx = None
        self.reasons = set()
        self.stop_flag = threading.Event()
        self.nvml = None
        try:
            import pynvml
            import torch
            pynvml.nvmlInit()
            self.nvml = pynvml
            # the CUDA device's own GPU (NVML numbers GPUs ignoring CUDA_VISIBLE_DEVICES)
            uuid = str(torch.cuda.get_device_properties(index).uuid)
            self.handle = pynvml.nvmlDeviceGetHandleByUUID(
                uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
            self.mx = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
            self.bits = {}
            for name, suffix in self.REASONS.items():
                v = getattr(pynvml, "nvmlClocksEventReason" + suffix,
                            getattr(pynvml, "nvmlClocksThrottleReason" + suffix, None))
                if v is not None:
                    self.bits[name] = v
        except Exception:
            self.nvml = None
        self.smi_id = str(index)
        try:
            import torch
            u = str(torch.cuda.get_device_properties(index).uuid)
            self.smi_id = u if u.startswith("GPU-") else "GPU-" + u
        except Exception:
            pass

    def _poll(self):
        nv = self.nvml
        get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons",
                              getattr(nv, "nvmlDeviceGetCurrentClocksThrottleReasons", None))
        while not self.stop_flag.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.handle, nv.NVML_CLOCK_SM))
                r = get_reasons(self.handle) if get_reasons else 0
                for name, bit in self.bits.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.005)

    def start(self):
        if self.nvml is not None:
            self.t = threading.Thread(target=self._poll, daemon=True)
            self.t.start()
            return
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.smi_id}", f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except FileNotFoundError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.nvml is not None:
            self.stop_flag.set()
            self.t.join(timeout=2)
            sm = self.samples
            return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.mx,
                    "reasons": sorted(self.reasons), "samples": len(sm), "source": "nvml"}
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 8:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for nm, v in zip(names, f[4:8]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm), "source": "nvidia-smi"}


def cpu_oracle_sample(A, B, n_hi, n_lo, budget_s=12.0, max_rows=1024):
    """Times the NumPy oracle on the first rows of A (row-local extraction
    makes those rows exact oracle rows) and returns (FP64-equiv TFLOP/s,
    rows, seconds)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import ozaki_oracle as O
    rows = 32
    while True:
        t0 = time.perf_counter()
        O.ondevice_numpy(A[:rows], B, n_hi, n_lo)
        dt = time.perf_counter() - t0
        if dt >= budget_s / 3 or rows >= max_rows:
            break
        rows *= 2
    k, m = B.shape
    return 2.0 * rows * k * m / dt / 1e12, rows, dt


def reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    n = k = m = args.size
    n_hi, n_lo = PRESETS[args.precision]
    A, B = make_inputs(n, k, m)
    vals = []
    for i in range(args.warmup + args.steps):
        v, rows, dt = cpu_oracle_sample(A, B, n_hi, n_lo, budget_s=6.0, max_rows=256)
        if i >= args.warmup:
            vals.append((v, rows, dt))
    v = statistics.median(x[0] for x in vals)
    rows = vals[-1][1]
    cores = os.cpu_count()
    out = {
        "metric": METRIC, "value": v, "unit": "TFLOP/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 2.0 * n * k * m / (v * 1e12) * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
        "impl": "reference",
        "config": {"workload": f"matmul {n}x{k}x{m} precision={args.precision} "
                               f"pipeline=ondevice (NumPy restatement of matmul_numpy)",
                   "N": n, "K": k, "M": m, "precision": args.precision},
        "cpu_baseline": {"value": v, "unit": "TFLOP/s", "cores": cores, "kind": "port",
                         "sample": f"first {rows} rows of A x full B per step, "
                                   f"extrapolated by FLOPs"},
        "e2e": {"value": v, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(out), flush=True)


def ours(args):
    import torch
    import torch.distributed as dist

    import ozaki_jax_b200 as oz
    from ozaki_jax_b200 import _lib

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=300))
    lib = _lib.load()
    if args.l2_persist_mb > 0:
        _lib.check(lib.ozk_set_l2_persisting(int(args.l2_persist_mb) << 20, None))

    n = k = m = args.size
    n_hi, n_lo = PRESETS[args.precision]
    nS = n_hi + n_lo
    A, B = make_inputs(n, k, m)
    r0, r1 = rank * n // world, (rank + 1) * n // world
    A_blk = np.ascontiguousarray(A[r0:r1])
    nb = r1 - r0
    Ad = torch.as_tensor(A_blk).to(dev)
    Bd = torch.as_tensor(B).to(dev)
    C = torch.empty((nb, m), dtype=torch.float64, device=dev)
    rho = lib.ozk_compute_rho_f32(k)
    # int8 slice codes where exact (rho >= 19: K > 4096), else BF16 slices
    s8 = rho >= 19 and nb >= 256 and m >= 256 and not args.bf16
    k_pad = (k + 127) // 128 * 128 if s8 else (k + 63) // 64 * 64
    SA = torch.empty((nS, nb, k_pad), dtype=torch.int8 if s8 else torch.int16, device=dev)
    SB = torch.empty((nS, m, k_pad), dtype=torch.int8 if s8 else torch.int16, device=dev)
    fail = torch.zeros(1, dtype=torch.int32, device=dev)
    eA = torch.empty((nS, nb), dtype=torch.int32, device=dev)
    eB = torch.empty((nS, m), dtype=torch.int32, device=dev)
    BT = torch.empty((m, k), dtype=torch.float64, device=dev)  # transposed-B scratch
    GW = torch.empty(lib.ozk_slice_gemm_workspace_bytes(), dtype=torch.uint8, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    pa = (ctypes.c_uint8 * 256)()
    pb = (ctypes.c_uint8 * 256)()
    # the pipeline's order for accumulation='fused' (order-independent sums)
    npairs = lib.ozk_pair_schedule_snake(n_hi, n_lo, pa, pb, 256)
    stream = torch.cuda.current_stream(dev)
    sh = stream.cuda_stream

    ACC = _lib.OZK_ACC_FIXED  # accumulation='fused

    def step(evs=None):
        if evs:
            evs[0].record(stream)
        if s8:
            _lib.check(lib.ozk_extract_rows_s8_f64(Ad.data_ptr(), k, nb, k, rho, n_hi, n_lo,
                                                   SA.data_ptr(), k_pad, eA.data_ptr(),
                                                   fail.data_ptr(), status.data_ptr(), sh))
            _lib.check(lib.ozk_extract_cols_s8_f64(Bd.data_ptr(), m, k, m, rho, n_hi, n_lo,
                                                   SB.data_ptr(), k_pad, eB.data_ptr(),
                                                   BT.data_ptr(), BT.numel() * 8, fail.data_ptr(),
                                                   status.data_ptr(), sh))
        else:
            _lib.check(lib.ozk_extract_rows_f64(Ad.data_ptr(), k, nb, k, rho, n_hi, n_lo,
                                                SA.data_ptr(), k_pad, eA.data_ptr(),
                                                status.data_ptr(), sh))
            _lib.check(lib.ozk_extract_cols_f64(Bd.data_ptr(), m, k, m, rho, n_hi, n_lo,
                                                SB.data_ptr(), k_pad, eB.data_ptr(),
                                                BT.data_ptr(), BT.numel() * 8,
                                                status.data_ptr(), sh))
        if evs:
            evs[1].record(stream)
        if s8:
            _lib.check(lib.ozk_slice_gemm_s8(SA.data_ptr(), eA.data_ptr(), nS, SB.data_ptr(),
                                             eB.data_ptr(), nS, nb, m, k_pad, pa, pb, npairs, 0,
                                             1.0, 0.0, None, 0, C.data_ptr(), m, GW.data_ptr(),
                                             GW.numel(), rho, fail.data_ptr(), status.data_ptr(),
                                             sh))
        else:
            _lib.check(lib.ozk_slice_gemm(SA.data_ptr(), eA.data_ptr(), nS, SB.data_ptr(),
                                          eB.data_ptr(), nS, nb, m, k_pad, pa, pb, npairs,
                                          ACC, 0, 1.0, 0.0, None, 0, C.data_ptr(), m,
                                          None, GW.data_ptr(), GW.numel(), rho,
                                          status.data_ptr(), sh))
        if evs:
            evs[2].record(stream)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    for _ in range(args.warmup):
        step()
    barrier()
    assert status.item() == 0, f"device status {status.item()}"
    assert fail.item() == 0, "a slice had no int8 code (inputs far outside the FP32 range)"

    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    clocks = Clocks(local)
    clocks.start()
    barrier()
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    t_start.record(stream)
    for i in range(args.steps):
        step(ev[i])
    t_end.record(stream)
    barrier()
    clk = clocks.stop()
    total_ms = t_start.elapsed_time(t_end)
    gemm_ms = sum(e[1].elapsed_time(e[2]) for e in ev) / args.steps
    extract_ms = sum(e[0].elapsed_time(e[1]) for e in ev) / args.steps
    if world > 1:
        t = torch.tensor([total_ms, gemm_ms, extract_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms, gemm_ms, extract_ms = t.tolist()
    gemm_waits = None
    if os.environ.get("OZK_GEMM_STATS") == "1":
        w = (ctypes.c_ulonglong * 8)()
        n_ctas = lib.ozk_gemm_stats(w)
        if n_ctas > 0 and w[3]:
            gemm_waits = {"mma_wait_accumulator": w[0] / w[3], "mma_wait_loads": w[1] / w[3],
                          "producer_wait_free_stage_cycles_per_cta": w[2] / n_ctas,
                          "mma_total_cycles_per_cta": w[3] / n_ctas,
                          "epilogue_wait_cycles_per_pair": w[4] / max(w[6], 1),
                          "epilogue_busy_cycles_per_pair": w[5] / max(w[6], 1),
                          "mma_wait_loads_pair_head": w[7] / w[3]}
    ms_step = total_ms / args.steps
    flops_fp64eq = 2.0 * n * k * m
    value = flops_fp64eq / (ms_step * 1e-3) / 1e12

    # accuracy of this rank's block against native FP64 (cuBLAS DGEMM)
    R = torch.matmul(Ad, Bd)
    rel_err = float(torch.linalg.norm(C - R) / torch.linalg.norm(R))
    # native FP64 DGEMM throughput on the same block, for comparison
    for _ in range(2):
        torch.matmul(Ad, Bd, out=R)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(3):
        torch.matmul(Ad, Bd, out=R)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    dgemm_tflops_rank = 2.0 * nb * k * m / (e0.elapsed_time(e1) / 3 * 1e-3) / 1e12
    del R

    # end to end through the public API from pinned host memory
    pinA = torch.empty(A_blk.shape, dtype=torch.float64, pin_memory=True)
    pinA.numpy()[...] = A_blk
    pinB = torch.empty(B.shape, dtype=torch.float64, pin_memory=True)
    pinB.numpy()[...] = B
    hA, hB = pinA.numpy(), pinB.numpy()
    if world == 1:
        e2e_call = lambda: oz.matmul(hA, hB, pipeline="ondevice", precision=args.precision)
    else:
        # each rank uploads its rows of A and 1/P of B; B is all-gathered over NCCL
        from ozaki_jax_b200.distributed import matmul_rowsharded_host
        e2e_call = lambda: matmul_rowsharded_host(hA, hB, precision=args.precision)
    # two warm-up calls: the result of one call is still alive while the next
    # runs, so torch's pinned-host pool needs two output buffers
    Ch = e2e_call()
    Ch = e2e_call()
    barrier()
    e2e_steps = max(1, min(args.steps, 3))
    e0.record(stream)
    for _ in range(e2e_steps):
        Ch = e2e_call()
    e1.record(stream)
    barrier()
    e2e_ms = e0.elapsed_time(e1) / e2e_steps
    if world > 1:
        t = torch.tensor([e2e_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = t.item()
    assert Ch.shape == (nb, m)

    l2_prev = ctypes.c_size_t(0)
    _lib.check(lib.ozk_set_l2_persisting(ctypes.c_size_t(-1).value, ctypes.byref(l2_prev)))
    if rank == 0:
        bf16_peak, hbm_peak, src = peaks()
        gemm_tflops = npairs * 2.0 * nb * k * m / (gemm_ms * 1e-3) / 1e12
        mma_peak, mma_unit, peak_src, peak_extra = tensor_peak(s8, dev)
        ext_bytes = (8.0 * (nb * k + k * m) + (1.0 if s8 else 2.0) * nS * (nb + m) * k_pad
                     + 4.0 * nS * (nb + m))
        cpu_v, cpu_rows, cpu_dt = cpu_oracle_sample(A, B, n_hi, n_lo)
        out = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f64",
            "data": "synthetic",
            "config": {"workload": f"matmul {n}x{k}x{m} pipeline=ondevice accumulation=fused "
                                   f"precision={args.precision} ({npairs} slice GEMMs)",
                       "N": n, "K": k, "M": m, "precision": args.precision,
                       "slices": "int8 codes" if s8 else "bf16",
                       "parallelism": f"row-blocks x{world}", "l2": "inputs 1 GiB > L2, no flush",
                       "l2_persisting_mb": round(l2_prev.value / 2**20, 1)},
            "rel_err": rel_err,
            "dgemm_fp64_tflops": dgemm_tflops_rank * world,
            "breakdown_ms": {"extract": extract_ms, "slice_gemm": gemm_ms},
            "gemm_wait_fractions": gemm_waits,
            "roofline": {"bound": "tensor", "kernel": "k_slice_gemm",
                         "mma": "int8 x int8 -> int32" if s8 else "bf16 x bf16 -> fp32",
                         "achieved": gemm_tflops, "peak": mma_peak, "unit": mma_unit,
                         "frac": gemm_tflops / mma_peak, "peak_source": peak_src, **peak_extra,
                         "frac_of_int8_library_gemm": (gemm_tflops / peak_extra["int8_library_gemm"]
                                                       if peak_extra.get("int8_library_gemm")
                                                       else None),
                         "traffic": GEMM_TRAFFIC_BYTES.get(
                             (n, args.precision, "int8" if s8 else "bf16")) if world == 1 else None,
                         "traffic_unit": "bytes per launch (ncu dram__bytes_read+write)",
                         "extract": {"bound": "hbm", "achieved_gbs": ext_bytes / (extract_ms * 1e-3) / 1e9,
                                     "peak_gbs": hbm_peak,
                                     "frac": ext_bytes / (extract_ms * 1e-3) / 1e9 / hbm_peak}},
            "cpu_baseline": {"value": cpu_v, "unit": "TFLOP/s", "cores": os.cpu_count(),
                             "kind": "port",
                             "sample": f"first {cpu_rows} rows of A x full B ({cpu_dt:.1f} s), "
                                       f"NumPy oracle, OpenBLAS threads = cores"},
            # copies of the whole job (all ranks): A and C once, B once in total
            # (world == 1) or in per-rank shares padded to ceil(K/P) rows
            "e2e": {"value": flops_fp64eq / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                    "h2d_bytes_per_step": int(8 * (n * k + (k * m if world == 1 else
                                                            world * ((k + world - 1) // world) * m))),
                    "d2h_bytes_per_step": int(8 * n * m)},
            "clocks": clk,
            "gpu_launches": 4 * args.steps,
        }
        print(json.dumps(out), flush=True)
    if world > 1:
        dist.destroy_process_group()


WORKLOADS = {
    # name: (description, precision)
    "c3": ("matmul 4096x8192x4096 precision=max, (U(0,1)-0.5)*exp(10*N(0,1)) entries", "max"),
    "c4": ("gram A^T A, A 65536x4096 N(0,1), column j scaled by 10^(-6j/4095)", "high"),
    "c5a": ("matmul 32768^3 precision=medium, N(0,1)", "medium"),
    "c5b": ("residual b - A x, A 32768^2 N(0,1) + 32768 I, x, b 32768x16", "high"),
}


def other_workload(args):
    """The other benchmark configurations (c3 'max' on wide-range entries, c4
    gram, c5a 'medium' 32768^3, c5b residual) on one GPU, through the C entry
    points on device arrays (inputs drawn on the device from a seeded torch
    generator with each configuration's distribution).  Prints one JSON line."""
    import torch
    from ozaki_jax_b200 import _lib

    lib = _lib.load()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    desc, precision = WORKLOADS[args.workload]
    n_hi, n_lo = PRESETS[precision]
    n_pairs = n_hi * n_hi + 2 * n_hi * n_lo
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    randn = lambda *shape: torch.randn(*shape, generator=g, device=dev, dtype=torch.float64)
    st = torch.zeros(1, dtype=torch.int32, device=dev)
    sh = torch.cuda.current_stream(dev).cuda_stream
    w = args.workload
    if w in ("c3", "c5a"):
        n, k, m = (4096, 8192, 4096) if w == "c3" else (32768, 32768, 32768)
        if w == "c3":
            A = (torch.rand(n, k, generator=g, device=dev, dtype=torch.float64) - 0.5) * torch.exp(10 * randn(n, k))
            B = (torch.rand(k, m, generator=g, device=dev, dtype=torch.float64) - 0.5) * torch.exp(10 * randn(k, m))
        else:
            A, B = randn(n, k), randn(k, m)
        C = torch.empty((n, m), dtype=torch.float64, device=dev)
        ws = torch.empty(lib.ozk_matmul_workspace_bytes(n, k, m, n_hi, n_lo), dtype=torch.uint8, device=dev)
        call = lambda: _lib.check(lib.ozk_matmul_f64(
            A.data_ptr(), k, B.data_ptr(), m, C.data_ptr(), m, n, k, m, -1, n_hi, n_lo,
            _lib.OZK_ACC_FIXED, ws.data_ptr(), ws.numel(), st.data_ptr(), sh))
        flops, contraction, ref = 2.0 * n * k * m, k, (lambda: torch.matmul(A, B))
    elif w == "c4":
        n, k = 65536, 4096
        A = randn(n, k) * torch.pow(10.0, -6.0 * torch.arange(k, device=dev, dtype=torch.float64) / 4095)
        C = torch.empty((k, k), dtype=torch.float64, device=dev)
        ws = torch.empty(lib.ozk_gram_workspace_bytes(n, k, n_hi, n_lo), dtype=torch.uint8, device=dev)
        call = lambda: _lib.check(lib.ozk_gram_f64(
            A.data_ptr(), k, C.data_ptr(), k, n, k, -1, n_hi, n_lo, ws.data_ptr(), ws.numel(),
            st.data_ptr(), sh))
        flops, contraction, ref = 2.0 * n * k * k, n, (lambda: torch.matmul(A.T, A))
    else:
        n, m = 32768, 16
        k = n
        A = randn(n, n)
        A.diagonal().add_(float(n))
        X, Bv = randn(n, m), randn(n, m)
        C = torch.empty((n, m), dtype=torch.float64, device=dev)
        ws = torch.empty(lib.ozk_residual_workspace_bytes(n, n, m, n_hi, n_lo), dtype=torch.uint8, device=dev)
        call = lambda: _lib.check(lib.ozk_residual_f64(
            A.data_ptr(), n, X.data_ptr(), m, Bv.data_ptr(), m, C.data_ptr(), m, n, n, m, -1,
            n_hi, n_lo, ws.data_ptr(), ws.numel(), st.data_ptr(), sh))
        flops, contraction, ref = 2.0 * n * n * m, n, (lambda: Bv - torch.matmul(A, X))
    for _ in range(args.warmup):
        call()
    torch.cuda.synchronize(dev)
    assert st.item() == 0, f"device status {st.item()}"
    clocks = Clocks(0)
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        call()
    e1.record()
    torch.cuda.synchronize(dev)
    clk = clocks.stop()
    ms = e0.elapsed_time(e1) / args.steps
    R = ref()
    rel_err = float(torch.linalg.norm(C - R) / torch.linalg.norm(R))
    del R
    rho = lib.ozk_compute_rho_f32(contraction)
    s8 = rho >= 19
    bf16_peak, hbm_peak, src = peaks()
    out = {"metric": "FP64-equiv TFLOP/s (2MNK/t)" if w != "c4" else "FP64-equiv TFLOP/s (2NK^2/t)",
           "value": flops / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "n_gpus": 1,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
           "higher_is_better": True, "dtype": "f64", "data": "synthetic (torch CUDA generator, seed 0)",
           "config": {"workload": f"{w}: {desc}", "precision": precision,
                      "slices": "int8 codes" if s8 else "bf16", "rho": rho},
           "rel_err_vs_cublas_dgemm": rel_err, "clocks": clk}
    if w == "c5b":
        a_bytes = 8.0 * n * n
        out["roofline"] = {"bound": "hbm", "achieved": a_bytes / (ms * 1e-3) / 1e9,
                           "peak": hbm_peak, "unit": "GB/s", "frac": a_bytes / (ms * 1e-3) / 1e9 / hbm_peak,
                           "note": "algorithmic bytes = one read of A", "peak_source": src}
    else:
        tensor = n_pairs * flops
        if w == "c4":
            # only the tiles on or above the diagonal are computed
            tiles = (k // 256) * (k // 256 + 1) / 2 / (k // 256) ** 2
            tensor *= tiles
        peak, unit, psrc, extra = tensor_peak(s8, dev)
        ach = tensor / (ms * 1e-3) / 1e12
        out["roofline"] = {"bound": "tensor", "achieved": ach, "peak": peak, "unit": unit,
                           "frac": ach / peak, "peak_source": psrc, **extra}
        if extra.get("int8_library_gemm"):
            out["roofline"]["frac_of_int8_library_gemm"] = ach / extra["int8_library_gemm"]
    print(json.dumps(out), flush=True)


def kernel_case(spec, steps):
    """One small case of a single hot kernel, for profiling (the ncu captures
    summarised under profiles/ run these): 'extract:ROWSxK' runs the int8 row
    extraction (ozk_extract_rows_s8_f64, preset high) on N(0,1) rows,
    'cols:KxCOLS' runs the int8 column extraction (ozk_extract_cols_s8_f64,
    preset high) of a K x COLS operand, 'residual:ROWSxK' runs
    residual(mode='ozaki') with 16 right-hand sides.  Prints one JSON line with
    the mean time of `steps` calls after one."""
    import torch

    import ozaki_jax_b200 as oz
    from ozaki_jax_b200 import _lib

    kind, shape = spec.split(":")
    n, k = (int(v) for v in shape.lower().split("x"))
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    A = torch.randn(n, k, generator=g, device=dev, dtype=torch.float64)
    if kind == "extract":
        lib = _lib.load()
        k8 = (k + 127) // 128 * 128
        SA = torch.empty((5, n, k8), dtype=torch.int8, device=dev)
        eA = torch.empty((5, n), dtype=torch.int32, device=dev)
        fail = torch.zeros(1, dtype=torch.int32, device=dev)
        st = torch.zeros(1, dtype=torch.int32, device=dev)
        rho = lib.ozk_compute_rho_f32(k)

        def call():
            _lib.check(lib.ozk_extract_rows_s8_f64(
                A.data_ptr(), k, n, k, rho, 4, 1, SA.data_ptr(), k8, eA.data_ptr(),
                fail.data_ptr(), st.data_ptr(), torch.cuda.current_stream().cuda_stream))
    elif kind == "cols":
        # A is K x COLS here: n = K, k = COLS
        lib = _lib.load()
        k8 = (n + 127) // 128 * 128
        SB = torch.empty((5, k, k8), dtype=torch.int8, device=dev)
        eB = torch.empty((5, k), dtype=torch.int32, device=dev)
        BT = torch.empty((k, n), dtype=torch.float64, device=dev)  # transposed-operand scratch
        fail = torch.zeros(1, dtype=torch.int32, device=dev)
        st = torch.zeros(1, dtype=torch.int32, device=dev)
        rho = lib.ozk_compute_rho_f32(n)

        def call():
            _lib.check(lib.ozk_extract_cols_s8_f64(
                A.data_ptr(), k, n, k, rho, 4, 1, SB.data_ptr(), k8, eB.data_ptr(),
                BT.data_ptr(), BT.numel() * 8, fail.data_ptr(), st.data_ptr(),
                torch.cuda.current_stream().cuda_stream))
    elif kind == "residual":
        x = torch.randn(k, 16, generator=g, device=dev, dtype=torch.float64)
        b = torch.randn(n, 16, generator=g, device=dev, dtype=torch.float64)

        def call():
            oz.residual(A, x, b, mode="ozaki")
    else:
        raise SystemExit(f"unknown case {spec!r}")
    call()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        call()
    e1.record()
    torch.cuda.synchronize(dev)
    print(json.dumps({"case": spec, "ms": e0.elapsed_time(e1) / steps, "steps": steps}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--size", type=int, default=8192)
    ap.add_argument("--precision", choices=sorted(PRESETS), default="high")
    ap.add_argument("--bf16", action="store_true",
                    help="BF16 slices even where int8 codes are exact (comparison)")
    ap.add_argument("--l2-persist-mb", type=int, default=0,
                    help="persisting-L2 set-aside for the GEMM's running sums in MB "
                         "(0: the library's own choice)")
    ap.add_argument("--workload", choices=["c2"] + sorted(WORKLOADS), default="c2",
                    help="c2 (default): the headline 8192^3 line; others: the remaining "
                         "benchmark configurations on one GPU")
    ap.add_argument("--case", default=None,
                    help="profiling aid, not a bench line: one small single-kernel case, "
                         "extract:ROWSxK, cols:KxCOLS or residual:ROWSxK (--steps calls "
                         "after one)")
    args = ap.parse_args()
    if args.case:
        kernel_case(args.case, args.steps)
    elif args.workload != "c2" and args.impl == "ours":
        other_workload(args)
    elif args.impl == "reference":
        reference_arm(args)
    else:
        ours(args)


if __name__ == "__main__":
    main()
