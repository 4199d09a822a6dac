"""Benchmark of the on-device Ozaki matmul, headline configuration (c2):
C = A @ B, A, B 8192 x 8192 FP64 N(0,1) (RandomState(0): A then B),
precision='high' (n_hi=4, n_lo=1, 24 slice GEMMs), accumulation='fused'.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload c2|c3|c4|c5a|c5b]
    torchrun --nproc-per-node N bench.py --gpus N ...   (one rank per GPU)

A step is one call of the C-ABI operator a caller runs (ozk_matmul_f64 for
matmul, ozk_gram_f64, ozk_residual_f64) on inputs resident in HBM: split and
slice extraction of A and B, then the persistent slice-pair GEMM with the
exact fixed-point epilogue, and every other launch the operator makes (the
gated BF16 recomputation, which exits at once when the int8 codes were exact).
The operator's kernels are also launched one by one in a second timed loop,
for the per-kernel split and the roofline of the slice GEMM.  Multi-GPU
(torchrun, one rank per GPU): the step is the multi-GPU C-ABI operator
ozk_matmul_f64_multi; rank r owns rows [r N/P, (r+1) N/P) of A and C and, by
default (--b-source columns), columns [r mc, (r+1) mc) of B, mc = ceil(M/P):
each rank extracts its columns and the int8 slice stacks are all-gathered over
NCCL inside every step (the root broadcast and the replicated extraction are
timed too and reported under b_source_modes); timing is the max over ranks.
Inputs exceed L2 (126 MB), so no flush is needed between steps.

Rank 0 prints one JSON line.  `value` is FP64-equivalent TFLOP/s (2NKM/t)
of the operator; `parity` compares blocks of the full-size result with the
reference's result on the same blocks of the same input (the NumPy oracle;
rows of A and columns of B are extracted independently, so a block of the
oracle's output is that block of the full reference result), both against the
exact product; `e2e` is the same metric through the public API
(ozaki_jax_b200.matmul / gram / residual) on ordinary pageable NumPy arrays,
every copy inside the timed region (`pinned_value`: the same with page-locked
inputs); `cpu_baseline` times the NumPy oracle (the reference's
matmul_numpy(pipeline='ondevice') restated) on a block of the result with all
host cores.  --impl reference runs only that CPU reference arm.
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


# ---------------------------------------------------------------------------
# Workloads: BASELINE's configurations, drawn on the host from
# np.random.RandomState(0) in the order written next to each
# ---------------------------------------------------------------------------

WORKLOADS = {
    # name: (description, precision, kind)
    "c2": ("matmul 8192^3 precision=high, N(0,1)", "high", "matmul"),
    "c3": ("matmul 4096x8192x4096 precision=max, (U(0,1)-0.5)*exp(10*N(0,1)) entries", "max",
           "matmul"),
    "c4": ("gram A^T A, A 65536x4096 N(0,1), column j scaled by 10^(-6j/4095)", "high", "gram"),
    "c5a": ("matmul 32768^3 precision=medium, N(0,1)", "medium", "matmul"),
    "c5b": ("residual b - A x, A 32768^2 N(0,1) + 32768 I, x, b 32768x16", "high", "residual"),
}


def workload_config(name, desc, n_pairs, kind, n, k, m, precision, rho, inputs):
    """The part of `config` that names the workload, the same on both arms."""
    return {"workload": f"{name}: {desc} ({n_pairs} slice GEMMs), "
                        f"accumulation={'bf16_interleaved' if kind != 'matmul' else 'fused'}",
            "N": n, "K": k, "M": m, "precision": precision, "rho": rho, "inputs": inputs}


def make_inputs(n, k, m):
    """c2 (and --size): A (n x k) then B (k x m), i.i.d. N(0,1) from RandomState(0)."""
    rng = np.random.RandomState(0)
    A = rng.randn(n, k)
    B = rng.randn(k, m)
    return A, B


def make_workload(name, size=8192, rank=0, world=1):
    """Host arrays of a configuration, drawn from RandomState(0):
    c2  A then B, N(0,1)                                   (size^3)
    c3  A's U(0,1), A's N(0,1), B's U(0,1), B's N(0,1); entry (U-0.5)*exp(10 N)
    c4  A N(0,1) (65536 x 4096), then column j scaled by 10^(-6j/4095)
    c5a A then B, N(0,1) (32768^2)
    c5b A N(0,1) (32768^2) + 32768 I, then x, then b (32768 x 16 each)
    With world > 1, c5a and c5b give each rank only its rows of A (and of b):
    a full-size draw on every rank would hold 8 x 17 GB of host memory.  Rank
    r's rows then come from RandomState(1 + r) (N(0,1), plus the diagonal for
    c5b); B (c5a) and x (c5b) still come from RandomState(0).  Such a dict
    carries the global row count "n_total" and the rank's first row "row0".
    Returns a dict with the operands and the shapes."""
    rng = np.random.RandomState(0)
    if world > 1 and name in ("c5a", "c5b"):
        n = 32768
        r0, r1 = rank * n // world, (rank + 1) * n // world
        rr = np.random.RandomState(1 + rank)
        A = rr.randn(r1 - r0, n)
        if name == "c5a":
            return {"A": A, "B": rng.randn(n, n), "n_total": n, "row0": r0}
        A[np.arange(r1 - r0), r0 + np.arange(r1 - r0)] += n
        return {"A": A, "x": rng.randn(n, 16), "b": rr.randn(r1 - r0, 16), "n_total": n,
                "row0": r0}
    if name == "c2":
        A, B = make_inputs(size, size, size)
        return {"A": A, "B": B}
    if name == "c3":
        n, k, m = 4096, 8192, 4096
        A = (rng.rand(n, k) - 0.5) * np.exp(10 * rng.randn(n, k))
        B = (rng.rand(k, m) - 0.5) * np.exp(10 * rng.randn(k, m))
        return {"A": A, "B": B}
    if name == "c4":
        n, k = 65536, 4096
        A = rng.randn(n, k)
        A *= 10.0 ** (-6.0 * np.arange(k) / 4095)
        return {"A": A}
    if name == "c5a":
        n = 32768
        A = rng.randn(n, n)
        B = rng.randn(n, n)
        return {"A": A, "B": B}
    if name == "c5b":
        n = 32768
        A = rng.randn(n, n)
        A[np.arange(n), np.arange(n)] += n
        x = rng.randn(n, 16)
        b = rng.randn(n, 16)
        return {"A": A, "x": x, "b": b}
    raise SystemExit(f"unknown workload {name!r}")


# ---------------------------------------------------------------------------
# Parity on the full-size inputs: blocks of the result against the oracle
# ---------------------------------------------------------------------------

def _oracle():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import ozaki_oracle as O
    return O


def sample_blocks(n_rows, n_cols, rows=64, cols=256):
    """The first and the last block of an n_rows x n_cols result: the last one
    lies in the GEMM's last wave of tiles (the pair-split tiles, where a wave
    is ragged)."""
    r, c = min(rows, n_rows), min(cols, n_cols)
    blocks = [(0, r, 0, c)]
    last = (n_rows - r, n_rows, n_cols - c, n_cols)
    if last != blocks[0]:
        blocks.append(last)
    return blocks


def reference_blocks(kind, W, blocks, n_hi, n_lo):
    """The reference's results on blocks of the identical input, and the exact
    product there.  Rows of A and columns of B (lines of A for gram) are
    extracted independently of each other, so the oracle on a block's rows and
    columns gives exactly that block of the full-size reference result.
    Returns three lists of blocks: the reference's fused result (FP32 2Sum, the
    configuration's accumulation), its matmul_numpy(pipeline='ondevice')
    result (FP64 sums), and the correctly rounded exact result."""
    O = _oracle()
    fused, numpy_, exact = [], [], []
    for r0, r1, c0, c1 in blocks:
        if kind == "matmul":
            A, B = W["A"][r0:r1], W["B"][:, c0:c1]
            fused.append(O.fused_ondevice(A, B, n_hi, n_lo)[2])
            numpy_.append(O.ondevice_numpy(A, B, n_hi, n_lo))
            exact.append(O.exact_product(A, B))
        elif kind == "gram":
            # G = (P + P^T)/2 with P = ozaki(A^T, A), rho from the row count
            A = W["A"]
            rho = O.compute_rho_f32(A.shape[0])
            L, R = A[:, r0:r1].T, A[:, c0:c1]
            p1 = O.fused_ondevice(L, R, n_hi, n_lo, rho)[2]
            p2 = O.fused_ondevice(R.T, L.T, n_hi, n_lo, rho)[2]
            fused.append((p1 + p2.T) * 0.5)
            q1 = O.ondevice_numpy(L, R, n_hi, n_lo)
            q2 = O.ondevice_numpy(R.T, L.T, n_hi, n_lo)
            numpy_.append((q1 + q2.T) * 0.5)
            exact.append(O.exact_product(L, R))
        else:  # residual: b - A x, all columns of x
            A, x, b = W["A"][r0:r1], W["x"], W["b"][r0:r1]
            fused.append(b - O.fused_ondevice(A, x, n_hi, n_lo)[2])
            numpy_.append(b - O.ondevice_numpy(A, x, n_hi, n_lo))
            exact.append(b - O.exact_product(A, x))
    return fused, numpy_, exact


def parity_report(kind, W, ours_blocks, blocks, n_hi, n_lo):
    """Normwise relative errors, against the exact product, of this build's
    result and of the reference's on the same blocks of the same input; the
    north star's bar is ours <= 1.5x the reference's."""
    O = _oracle()
    t0 = time.perf_counter()
    fused, numpy_, exact = reference_blocks(kind, W, blocks, n_hi, n_lo)
    cat = lambda xs: np.concatenate([x.ravel() for x in xs])
    E = cat(exact)
    e_ours = O.rel_err(cat(ours_blocks), E)
    e_fused = O.rel_err(cat(fused), E)
    e_numpy = O.rel_err(cat(numpy_), E)
    finite = [e for e in (e_fused, e_numpy) if np.isfinite(e)]
    e_ref = min(finite) if finite else float("inf")
    floor = 32 * 2.0 ** -52
    return {
        "sample": "blocks [r0,r1)x[c0,c1) of the result: " + ", ".join(
            f"[{r0},{r1})x[{c0},{c1})" for r0, r1, c0, c1 in blocks),
        "exact": "correctly rounded FP64 result of the block (error-free split, math.fsum)",
        "rel_err_ours": e_ours,
        "rel_err_ref_fused": e_fused,
        "rel_err_ref_numpy": e_numpy,
        "ratio_to_ref": e_ours / e_ref if e_ref > 0 else None,
        "within_1p5x_ref": bool(e_ours <= max(1.5 * e_ref, floor)),
        "oracle_s": round(time.perf_counter() - t0, 1),
    }


# ---------------------------------------------------------------------------
# CPU baseline and the reference arm
# ---------------------------------------------------------------------------

def cpu_oracle_sample(A, B, n_hi, n_lo, budget_s=12.0, max_side=2048):
    """Times the NumPy oracle (the reference's matmul_numpy(pipeline='ondevice')
    restated) on the block C[0:s, 0:s] = A[0:s] @ B[:, 0:s] with all host
    cores; rows of A and columns of B are extracted independently, so the
    block is exactly that block of the full reference result and its work has
    the full job's mix (GEMM-dominated).  The side s doubles from 256 until a
    call takes budget_s / 3.  Returns (FP64-equiv TFLOP/s, s, seconds)."""
    O = _oracle()
    s = 256
    k = A.shape[1]
    while True:
        t0 = time.perf_counter()
        O.ondevice_numpy(A[:s], B[:, :s], n_hi, n_lo)
        dt = time.perf_counter() - t0
        if dt >= budget_s / 3 or s >= max_side:
            break
        s *= 2
    return 2.0 * s * k * s / dt / 1e12, s, dt


def reference_arm(args):
    """--impl reference: the reference's own CPU implementation of the path,
    the oracle port of matmul_numpy(pipeline='ondevice') (the reference is
    Python and cannot travel to the GPU box; the port is pinned bit for bit to
    the reference's own outputs).  Each step computes one bounded block of the
    workload, C[0:s, 0:s] (s fixed in the first warm-up step), and the line
    reports the measured rate on it; ms_per_step is that step's real time."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    O = _oracle()
    n = k = m = args.size
    n_hi, n_lo = PRESETS[args.precision]
    A, B = make_inputs(n, k, m)
    _, side, _ = cpu_oracle_sample(A, B, n_hi, n_lo, budget_s=9.0, max_side=2048)
    times = []
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        O.ondevice_numpy(A[:side], B[:, :side], n_hi, n_lo)
        dt = time.perf_counter() - t0
        if i >= args.warmup:
            times.append(dt)
    ms = statistics.mean(times) * 1e3
    v = 2.0 * side * k * side / (ms * 1e-3) / 1e12
    cores = os.cpu_count()
    out = {
        "metric": METRIC, "value": v, "unit": "TFLOP/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f64",
        "data": "synthetic (seeded; config.inputs says how)", "impl": "reference",
        "config": dict(workload_config(
            "c2", f"matmul {n}^3 precision={args.precision}, N(0,1)",
            n_hi * n_hi + 2 * n_hi * n_lo, "matmul", n, k, m, args.precision,
            O.compute_rho_f32(k), "RandomState(0), BASELINE's recipe"),
            parallelism="host cores (the reference's CPU path)"),
        "cpu_baseline": {"value": v, "unit": "TFLOP/s", "cores": cores, "kind": "port",
                         "sample": f"one step = the block C[0:{side}, 0:{side}] (A[0:{side}] x "
                                   f"B[:, 0:{side}], K={k}) by the NumPy port of matmul_numpy"
                                   f"(pipeline='ondevice'), OpenBLAS threads = cores; measured "
                                   f"rate, not extrapolated"},
        "e2e": {"value": v, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(out), flush=True)



# ---------------------------------------------------------------------------
# This build's arm
# ---------------------------------------------------------------------------

def _timed(call, steps, stream):
    """Mean milliseconds of `steps` calls, CUDA events on the launching stream."""
    import torch
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        call()
    e1.record(stream)
    e1.synchronize()
    return e0.elapsed_time(e1) / steps


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
    name = args.workload
    desc, precision, kind = WORKLOADS[name]
    if name == "c2":
        precision = args.precision
        desc = f"matmul {args.size}^3 precision={precision}, N(0,1)"
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=300))
    lib = _lib.load()
    if args.l2_persist_mb > 0:
        _lib.check(lib.ozk_set_l2_persisting(int(args.l2_persist_mb) << 20, None))
    n_hi, n_lo = PRESETS[precision]
    nS = n_hi + n_lo
    n_pairs = n_hi * n_hi + 2 * n_hi * n_lo

    W = make_workload(name, args.size, rank, world)
    stream = torch.cuda.current_stream(dev)
    sh = stream.cuda_stream
    st = torch.zeros(1, dtype=torch.int32, device=dev)
    res = {}  # results of the multi-GPU Python operators
    if kind == "matmul":
        A, B = W["A"], W["B"]
        n, k = W.get("n_total", A.shape[0]), A.shape[1]
        m = B.shape[1]
        r0, r1 = rank * n // world, (rank + 1) * n // world
        A_blk = np.ascontiguousarray(A if "n_total" in W else A[r0:r1])
        nb = r1 - r0
        Ad = torch.as_tensor(A_blk).to(dev)
        Bd = torch.as_tensor(B).to(dev)
        C = torch.empty((nb, m), dtype=torch.float64, device=dev)
        ws = torch.empty(lib.ozk_matmul_workspace_bytes(nb, k, m, n_hi, n_lo), dtype=torch.uint8,
                         device=dev)
        contraction = k
        flops = 2.0 * n * k * m

        def op():
            _lib.check(lib.ozk_matmul_f64(Ad.data_ptr(), k, Bd.data_ptr(), m, C.data_ptr(), m, nb,
                                          k, m, -1, n_hi, n_lo, _lib.OZK_ACC_FIXED, ws.data_ptr(),
                                          ws.numel(), st.data_ptr(), sh))
        if world > 1:
            # the multi-GPU operator: B's slices reach every rank inside the step
            from ozaki_jax_b200 import distributed as dd
            mctx = dd.context()
            c0, c1 = dd.column_range(m, rank, world)
            Bcols = Bd[:, c0:c1].contiguous()
            Pv, I64 = ctypes.c_void_p, ctypes.c_int64
            b_args = {"columns": (Bcols, c1 - c0), "root": (Bd if rank == 0 else None, m),
                      "replicated": (Bd, m)}

            def multi_op(mode):
                Bm, ldb = b_args[mode]
                args_ = (mctx.ptr, (Pv * 1)(Ad.data_ptr()), (I64 * 1)(k),
                         (Pv * 1)(Bm.data_ptr() if Bm is not None else None), (I64 * 1)(ldb),
                         (Pv * 1)(C.data_ptr()), (I64 * 1)(m), n, k, m, n_hi, n_lo,
                         dd._B_MODES[mode], _lib.OZK_MULTI_NOWAIT, (Pv * 1)(sh),
                         (Pv * 1)(st.data_ptr()))
                return lambda: _lib.check(lib.ozk_matmul_f64_multi(*args_))
            op = multi_op(args.b_source)
    elif kind == "gram":
        A = W["A"]
        n, k = A.shape
        m = k
        nb = k
        Ad = torch.as_tensor(A).to(dev)
        C = torch.empty((k, k), dtype=torch.float64, device=dev)
        ws = torch.empty(lib.ozk_gram_workspace_bytes(n, k, n_hi, n_lo), dtype=torch.uint8,
                         device=dev)
        contraction = n
        flops = 2.0 * n * k * k

        def op():
            _lib.check(lib.ozk_gram_f64(Ad.data_ptr(), k, C.data_ptr(), k, n, k, -1, n_hi, n_lo,
                                        ws.data_ptr(), ws.numel(), st.data_ptr(), sh))
        if world > 1:
            # rows of A split over the ranks; this rank's rows of G (gram_rowsharded)
            from ozaki_jax_b200.distributed import gram_rowsharded, row_range
            g0, g1 = row_range(n, rank, world)
            Ad_rows = Ad[g0:g1].contiguous()
            del Ad, C, ws
            Ad = Ad_rows
            c0g, c1g = row_range(k, rank, world)
            nb = c1g - c0g

            def op():
                res["C"] = gram_rowsharded(Ad_rows, precision=precision)
    else:
        A, x, b = W["A"], W["x"], W["b"]
        n, k = W.get("n_total", A.shape[0]), A.shape[1]
        m = x.shape[1]
        nb = A.shape[0]
        Ad, Xd, bd = (torch.as_tensor(v).to(dev) for v in (A, x, b))
        # at N > 1 every rank holds its rows of A and b and all of x, and runs the
        # operator on its rows (residual_rowsharded: rows are independent, no
        # collective in the data path)
        C = torch.empty((nb, m), dtype=torch.float64, device=dev)
        ws = torch.empty(lib.ozk_residual_workspace_bytes(nb, k, m, n_hi, n_lo), dtype=torch.uint8,
                         device=dev)
        contraction = k
        flops = 2.0 * n * k * m

        def op():
            _lib.check(lib.ozk_residual_f64(Ad.data_ptr(), k, Xd.data_ptr(), m, bd.data_ptr(), m,
                                            C.data_ptr(), m, nb, k, m, -1, n_hi, n_lo,
                                            ws.data_ptr(), ws.numel(), st.data_ptr(), sh))

    rho = lib.ozk_compute_rho_f32(contraction)
    s8 = rho >= 19 and os.environ.get("OZK_S8", "1") != "0"

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    # ---- value: the C-ABI operator, inputs resident in HBM
    for _ in range(args.warmup):
        op()
    barrier()
    assert st.item() == 0, f"device status {st.item()}"
    clocks = Clocks(local)
    clocks.start()
    barrier()
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    t_start.record(stream)
    for _ in range(args.steps):
        op()
    t_end.record(stream)
    barrier()
    op_ms = t_start.elapsed_time(t_end) / args.steps
    assert st.item() == 0, f"device status {st.item()}"
    b_modes = None
    if world > 1 and kind == "matmul":
        # the other ways of bringing B to every rank, each in its own timed loop
        b_modes = {}
        for mode in ("columns", "root", "replicated"):
            if mode == args.b_source:
                b_modes[mode] = op_ms
                continue
            f = multi_op(mode)
            for _ in range(2):
                f()
            barrier()
            b_modes[mode] = _timed(f, args.steps, stream)
        t = torch.tensor([b_modes[x] for x in ("columns", "root", "replicated")],
                         dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        b_modes = {x: {"ms_per_step": v, "value": flops / (v * 1e-3) / 1e12}
                   for x, v in zip(("columns", "root", "replicated"), t.tolist())}
        assert st.item() == 0, f"device status {st.item()}"

    # ---- the same kernels launched one by one, for the per-kernel split
    breakdown, gemm_ms, extract_ms, kernel_launches = None, None, None, 0
    if kind in ("matmul", "gram") and s8 and nb >= 256 and m >= 256 and (
            world == 1 or kind == "matmul"):
        k8 = (contraction + 127) // 128 * 128
        fail = torch.zeros(1, dtype=torch.int32, device=dev)
        pa = (ctypes.c_uint8 * 256)()
        pb = (ctypes.c_uint8 * 256)()
        npairs = lib.ozk_pair_schedule_snake(n_hi, n_lo, pa, pb, 256)
        GW = torch.empty(lib.ozk_slice_gemm_workspace_bytes(), dtype=torch.uint8, device=dev)
        if kind == "matmul":
            SA = torch.empty((nS, nb, k8), dtype=torch.int8, device=dev)
            SB = torch.empty((nS, m, k8), dtype=torch.int8, device=dev)
            eA = torch.empty((nS, nb), dtype=torch.int32, device=dev)
            eB = torch.empty((nS, m), dtype=torch.int32, device=dev)
            BT = torch.empty((m, k), dtype=torch.float64, device=dev)

            def extract():
                _lib.check(lib.ozk_extract_rows_s8_f64(Ad.data_ptr(), k, nb, k, rho, n_hi, n_lo,
                                                       SA.data_ptr(), k8, eA.data_ptr(),
                                                       fail.data_ptr(), st.data_ptr(), sh))
                _lib.check(lib.ozk_extract_cols_s8_f64(Bd.data_ptr(), m, k, m, rho, n_hi, n_lo,
                                                       SB.data_ptr(), k8, eB.data_ptr(),
                                                       BT.data_ptr(), BT.numel() * 8,
                                                       fail.data_ptr(), st.data_ptr(), sh))

            def gemm():
                _lib.check(lib.ozk_slice_gemm_s8(SA.data_ptr(), eA.data_ptr(), nS, SB.data_ptr(),
                                                 eB.data_ptr(), nS, nb, m, k8, pa, pb, npairs, 0,
                                                 1.0, 0.0, None, 0, C.data_ptr(), m, GW.data_ptr(),
                                                 GW.numel(), rho, fail.data_ptr(), st.data_ptr(),
                                                 sh))
            per_step = 4  # rows of A, transpose + rows of B, GEMM
        else:
            SA = torch.empty((nS, k, k8), dtype=torch.int8, device=dev)
            eA = torch.empty((nS, k), dtype=torch.int32, device=dev)
            BT = torch.empty((k, n), dtype=torch.float64, device=dev)

            def extract():
                _lib.check(lib.ozk_extract_cols_s8_f64(Ad.data_ptr(), k, n, k, rho, n_hi, n_lo,
                                                       SA.data_ptr(), k8, eA.data_ptr(),
                                                       BT.data_ptr(), BT.numel() * 8,
                                                       fail.data_ptr(), st.data_ptr(), sh))

            def gemm():
                _lib.check(lib.ozk_slice_gemm_s8(SA.data_ptr(), eA.data_ptr(), nS, SA.data_ptr(),
                                                 eA.data_ptr(), nS, k, k, k8, pa, pb, npairs, 1,
                                                 1.0, 0.0, None, 0, C.data_ptr(), k, GW.data_ptr(),
                                                 GW.numel(), rho, fail.data_ptr(), st.data_ptr(),
                                                 sh))
            per_step = 3
        for _ in range(args.warmup):
            extract()
            gemm()
        barrier()
        ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
        barrier()
        for i in range(args.steps):
            ev[i][0].record(stream)
            extract()
            ev[i][1].record(stream)
            gemm()
            ev[i][2].record(stream)
        barrier()
        assert fail.item() == 0 and st.item() == 0
        extract_ms = sum(e[0].elapsed_time(e[1]) for e in ev) / args.steps
        gemm_ms = sum(e[1].elapsed_time(e[2]) for e in ev) / args.steps
        kernel_launches = per_step * args.steps
        del SA, eA, BT
    clk = clocks.stop()
    if "C" in res:
        C = res["C"]
    if world > 1:
        t = torch.tensor([op_ms, gemm_ms or 0.0, extract_ms or 0.0], dtype=torch.float64,
                         device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        op_ms, g, e = t.tolist()
        gemm_ms, extract_ms = (g or None), (e or None)
    value = flops / (op_ms * 1e-3) / 1e12

    # ---- parity on the full-size input: blocks of this rank's result
    blocks = sample_blocks(nb, m)
    Ch = [C[r0_:r1_, c0_:c1_].cpu().numpy() for r0_, r1_, c0_, c1_ in blocks]
    if kind == "matmul":
        Wr = {"A": A_blk, "B": W["B"]}
    else:
        Wr = W
    parity = parity_report(kind, Wr, Ch, blocks, n_hi, n_lo) if rank == 0 else None

    # ---- native FP64 (cuBLAS DGEMM) on the same operands, for comparison
    rel_err_dgemm = dgemm_tflops = None
    if kind == "matmul":
        ref = lambda: torch.matmul(Ad, Bd)
    elif kind == "gram":
        ref = (lambda: torch.matmul(Ad.T, Ad)) if world == 1 else None
    else:
        ref = lambda: bd - torch.matmul(Ad, Xd)
    if ref is not None:
        R = ref()
        rel_err_dgemm = float(torch.linalg.norm(C - R) / torch.linalg.norm(R))
        del R
        dgemm_ms = _timed(lambda: ref(), 3, stream)
        dgemm_tflops = flops / (dgemm_ms * 1e-3) / 1e12  # every rank runs its share at once

    # ---- end to end through the public API, host arrays in and out
    def e2e_case(pinned):
        import torch as T
        host = {}
        srcs = {"matmul": ("A", "B"), "gram": ("A",), "residual": ("A", "x", "b")}[kind]
        for key in srcs:
            v = np.ascontiguousarray(A_blk if (kind == "matmul" and key == "A") else W[key])
            if pinned:
                p = T.empty(v.shape, dtype=T.float64, pin_memory=True)
                p.numpy()[...] = v
                v = p.numpy()
            host[key] = v
        if kind == "matmul" and world == 1:
            return lambda: oz.matmul(host["A"], host["B"], pipeline="ondevice", precision=precision)
        if kind == "matmul":
            from ozaki_jax_b200.distributed import matmul_rowsharded_host
            return lambda: matmul_rowsharded_host(host["A"], host["B"], precision=precision)
        if kind == "gram":
            return lambda: oz.gram(host["A"], precision=precision, mode="ozaki")
        return lambda: oz.residual(host["A"], host["x"], host["b"], precision=precision,
                                   mode="ozaki")

    def e2e_time(call):
        # two warm-up calls: one result is still alive while the next runs
        out = call()
        out = call()
        barrier()
        steps = max(1, min(args.steps, 3))
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for _ in range(steps):
            out = call()
        t1.record(stream)
        barrier()
        ms = t0.elapsed_time(t1) / steps
        if world > 1:
            t = torch.tensor([ms], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = t.item()
        assert out.shape == (nb, m)
        return ms
    # (at N > 1 the gram's and c5a's host copies would not fit eight ranks' host memory)
    e2e_ms = e2e_pinned_ms = None
    if world == 1 or name in ("c2", "c5b"):
        e2e_ms = e2e_time(e2e_case(pinned=False))
        e2e_pinned_ms = e2e_time(e2e_case(pinned=True))

    l2_prev = ctypes.c_size_t(0)
    _lib.check(lib.ozk_set_l2_persisting(ctypes.c_size_t(-1).value, ctypes.byref(l2_prev)))
    if world > 1:
        from ozaki_jax_b200.distributed import close_contexts
        close_contexts()
    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return
    bf16_peak, hbm_peak, src = peaks()
    # int8 path: extraction kernels (columns: transpose + rows), the slice GEMM
    # and the gated BF16 recomputation (two extractions and a GEMM), which
    # exits at once
    op_launches = {"matmul": 7, "gram": 5, "residual": 7}[kind] if s8 else 3
    if world > 1 and kind == "matmul":
        op_launches = 5  # A's rows, B's transpose + rows, flags, GEMM
    out = {
        "metric": METRIC if name == "c2" else (
            "FP64-equiv TFLOP/s (2NK^2/t)" if kind == "gram" else "FP64-equiv TFLOP/s (2MNK/t)"),
        "value": value, "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": op_ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f64",
        "data": "synthetic (seeded; config.inputs says how)",
        "config": {**workload_config(
                       name, desc, n_pairs, kind, n, k, m, precision, rho,
                       ("each rank's rows of A (and b) from RandomState(1 + rank); "
                        "B / x from RandomState(0)") if "n_total" in W else
                       "RandomState(0), BASELINE's recipe"),
                   "slices": "int8 codes" if s8 else "bf16",
                   "parallelism": f"row-blocks x{world}" if world > 1 else "1 GPU",
                   "timed": (f"ozk_matmul_f64_multi (the C-ABI multi-GPU operator), "
                             f"b_source={args.b_source}: B's int8 slices "
                             + {"columns": "all-gathered from per-rank column blocks",
                                "root": "broadcast from rank 0",
                                "replicated": "extracted on every rank (no exchange)"}[
                                 args.b_source] + " over NCCL inside every step"
                             if world > 1 else
                             "ozk_matmul_f64 (the C-ABI operator, all its launches)")
                            if kind == "matmul" else (
                                "gram_rowsharded -> ozk_gram_f64_multi (the C-ABI multi-GPU "
                                "operator): rows of A sharded, each slice pass's line maxima "
                                "all-reduced (NCCL), partial int64 Gram sums all-reduced, one "
                                "FP64 rounding" if (kind == "gram" and world > 1) else
                                f"ozk_{kind}_f64 (the C-ABI operator)"
                                + (" on each rank's rows (no collective)" if world > 1 else "")),
                   "l2": "inputs larger than L2 (126 MB), no flush",
                   "l2_persisting_mb_after": round(l2_prev.value / 2**20, 1)},
        "parity": parity,
        "b_source_modes": b_modes,
        "rel_err_vs_cublas_dgemm": rel_err_dgemm,
        "dgemm_fp64_tflops": dgemm_tflops,
        "breakdown_ms": {"operator": op_ms, "extract": extract_ms, "slice_gemm": gemm_ms,
                         "note": "extract / slice_gemm: the operator's kernels launched one by one "
                                 "in a second timed loop"},
        "clocks": clk,
        "gpu_launches": op_launches * args.steps + kernel_launches,
    }
    if kind in ("matmul", "gram") and gemm_ms:
        tensor = n_pairs * flops / world
        if kind == "gram":
            tiles = (k // 256) * (k // 256 + 1) / 2 / (k // 256) ** 2
            tensor *= tiles
        mma_peak, mma_unit, peak_src, peak_extra = tensor_peak(s8, dev)
        ach = tensor / (gemm_ms * 1e-3) / 1e12
        ext_bytes = (8.0 * (nb * k + k * m) + 1.0 * nS * (nb + m) * k8 + 4.0 * nS * (nb + m)
                     if kind == "matmul" else 8.0 * n * k + nS * k * k8 + 4.0 * nS * k)
        out["roofline"] = {
            "bound": "tensor", "kernel": "k_slice_gemm", "mma": "int8 x int8 -> int32",
            "achieved": ach, "peak": mma_peak, "unit": mma_unit, "frac": ach / mma_peak,
            "peak_source": peak_src, **peak_extra,
            "frac_of_int8_library_gemm": (ach / peak_extra["int8_library_gemm"]
                                          if peak_extra.get("int8_library_gemm") else None),
            "traffic": GEMM_TRAFFIC_BYTES.get((n, precision, "int8")) if world == 1 else None,
            "traffic_unit": "bytes per launch (ncu dram__bytes_read+write)",
            "extract": {"bound": "hbm", "achieved_gbs": ext_bytes / (extract_ms * 1e-3) / 1e9,
                        "peak_gbs": hbm_peak,
                        "frac": ext_bytes / (extract_ms * 1e-3) / 1e9 / hbm_peak}}
    elif kind == "residual":
        a_bytes = 8.0 * n * k
        out["roofline"] = {"bound": "hbm", "kernel": "the residual operator",
                           "achieved": a_bytes / (op_ms * 1e-3) / 1e9, "peak": hbm_peak,
                           "unit": "GB/s", "frac": a_bytes / (op_ms * 1e-3) / 1e9 / hbm_peak,
                           "peak_source": src, "traffic": None,
                           "note": "algorithmic bytes = one read of A"}
    # copies of the whole job (all ranks): A and C once, B once in total
    # (world == 1) or in per-rank shares padded to ceil(K/P) rows
    if kind == "matmul":
        h2d = 8 * (n * k + (k * m if world == 1 else world * ((k + world - 1) // world) * m))
        d2h = 8 * n * m
    elif kind == "gram":
        h2d, d2h = 8 * n * k, 8 * k * k
    else:
        h2d, d2h = 8 * (n * k + 2 * n * m), 8 * n * m
    if e2e_ms is not None:
        out["e2e"] = {"value": flops / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                      "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
                      "host_memory": "pageable NumPy arrays (what a drop-in caller passes)",
                      "pinned_value": flops / (e2e_pinned_ms * 1e-3) / 1e12}
    else:
        out["e2e"] = None
    # the CPU baseline runs on rank 0 at N = 1 only (torchrun limits a rank's
    # OpenBLAS threads, and the figure does not depend on N)
    if (name == "c2" or args.cpu_baseline) and world == 1:
        if kind == "matmul":
            cpu_v, side, cpu_dt = cpu_oracle_sample(W["A"], W["B"], n_hi, n_lo)
            out["cpu_baseline"] = {
                "value": cpu_v, "unit": "TFLOP/s", "cores": os.cpu_count(), "kind": "port",
                "sample": f"block C[0:{side}, 0:{side}] ({cpu_dt:.1f} s) by the NumPy port of "
                          f"matmul_numpy(pipeline='ondevice'), OpenBLAS threads = cores"}
    print(json.dumps(out), flush=True)
    if world > 1:
        dist.destroy_process_group()



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
    ap.add_argument("--size", type=int, default=8192, help="c2 only: N = K = M")
    ap.add_argument("--precision", choices=sorted(PRESETS), default="high", help="c2 only")
    ap.add_argument("--l2-persist-mb", type=int, default=0,
                    help="persisting-L2 set-aside for the GEMM's running sums in MB "
                         "(0: the library's own choice)")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="c2",
                    help="c2 (default): the headline 8192^3 line; others: the remaining "
                         "benchmark configurations on one GPU")
    ap.add_argument("--b-source", choices=["columns", "root", "replicated"], default="columns",
                    help="--gpus > 1: how B's slices reach every rank in the timed operator "
                         "(all three are timed and reported)")
    ap.add_argument("--cpu-baseline", action="store_true",
                    help="also time the CPU oracle for a workload other than c2")
    ap.add_argument("--case", default=None,
                    help="profiling aid, not a bench line: one small single-kernel case, "
                         "extract:ROWSxK, cols:KxCOLS or residual:ROWSxK (--steps calls "
                         "after one)")
    args = ap.parse_args()
    if args.case:
        kernel_case(args.case, args.steps)
    elif args.impl == "reference":
        reference_arm(args)
    else:
        ours(args)


if __name__ == "__main__":
    main()
