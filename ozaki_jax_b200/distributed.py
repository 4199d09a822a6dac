"""Row-sharded Ozaki matmul over the GPUs of one node (one process per GPU).

The reference has no multi-device code; this is the build's partitioning of
the on-device path.  Rank r owns rows [r*N/P, (r+1)*N/P) of A and of C.  Row
extraction is row-local, so each rank's slices of A are bit-identical to the
single-GPU ones and each rank's block of C equals the corresponding rows of
the single-GPU result.  B reaches every rank in one of two ways:

  b_source='replicated'  every rank was given B and extracts its column slices
                         locally (no collective in the data path);
  b_source='root'        rank 0 extracts B's slices once and broadcasts the slice
                         stack (int8 codes where exact, else BF16) and exponents
                         over NCCL (NVLink).

The collectives go through torch.distributed (NCCL for CUDA tensors, gloo on
CPU); the compute is libozaki_b200.
"""

import ctypes

import numpy as np
import torch
import torch.distributed as dist

from . import _device as D
from . import _lib as L
from .matmul import _resolve_precision, compute_rho_f32


def row_range(n, rank, world):
    """Rows [r0, r1) of an n-row matrix owned by `rank` of `world`."""
    return rank * n // world, (rank + 1) * n // world


def broadcast_(t, src=0, group=None):
    """In-place broadcast of a tensor from `src` (thin wrapper, kept for tests)."""
    dist.broadcast(t, src=src, group=group)
    return t


def gather_rows(C_local, n_total, dst=None, group=None):
    """Assemble the row blocks of C.  Blocks may differ in size by one row, so
    each is padded to the largest block for the collective.  dst=None gathers on
    every rank (all_gather); otherwise only rank `dst` returns the full C."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    sizes = [row_range(n_total, r, world) for r in range(world)]
    mx = max(r1 - r0 for r0, r1 in sizes)
    pad = torch.zeros((mx,) + tuple(C_local.shape[1:]), dtype=C_local.dtype,
                      device=C_local.device)
    pad[: C_local.shape[0]] = C_local
    if dst is None:
        parts = [torch.empty_like(pad) for _ in range(world)]
        dist.all_gather(parts, pad, group=group)
    else:
        parts = [torch.empty_like(pad) for _ in range(world)] if rank == dst else None
        dist.gather(pad, gather_list=parts, dst=dst, group=group)
        if rank != dst:
            return None
    return torch.cat([p[: r1 - r0] for p, (r0, r1) in zip(parts, sizes)], dim=0)


def _pairs(lib, n_hi, n_lo):
    pa = (ctypes.c_uint8 * 256)()
    pb = (ctypes.c_uint8 * 256)()
    n = L.check(lib.ozk_pair_schedule_snake(n_hi, n_lo, pa, pb, 256))
    return pa, pb, n


def matmul_rowsharded(A_local, B, K=None, precision="high", b_source="replicated", group=None):
    """C_local = (A @ B)[rows of this rank] with the Ozaki 'fused' accumulation.

    A_local: this rank's row block of A (CUDA float64, rows x K).
    B: the full K x M matrix on every rank ('replicated'), or a K x M tensor
       whose contents matter only on rank 0 ('root'; other ranks may pass a
       tensor of the right shape or None with K given through A_local).
    Returns this rank's rows of C (CUDA float64).  All ranks must call it.
    """
    lib = L.load()
    n_hi, n_lo = _resolve_precision(precision)
    nS = n_hi + n_lo
    dev = A_local.device
    rank = dist.get_rank(group)
    Ad = A_local.to(dtype=torch.float64).contiguous()
    nb, Kd = Ad.shape
    if b_source not in ("replicated", "root"):
        raise ValueError("b_source must be 'replicated' or 'root'")
    shape = torch.tensor(list(B.shape) if (B is not None and rank == 0) else [0, 0],
                         dtype=torch.int64, device=dev)
    if b_source == "root":
        dist.broadcast(shape, src=0, group=group)
        Kb, M = int(shape[0]), int(shape[1])
    else:
        Kb, M = B.shape
    if Kb != Kd:
        raise ValueError(f"Incompatible shapes for matmul: {tuple(Ad.shape)} and {(Kb, M)}.")
    rho = compute_rho_f32(Kd)
    sh = D.stream_handle(dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    C = torch.empty((nb, M), dtype=torch.float64, device=dev)
    pa, pb, npairs = _pairs(lib, n_hi, n_lo)
    GW = torch.empty(lib.ozk_slice_gemm_workspace_bytes(), dtype=torch.uint8, device=dev)
    have_b = b_source == "replicated" or rank == 0
    Bd = B.to(device=dev, dtype=torch.float64).contiguous() if have_b else None
    BT = torch.empty((M, Kd), dtype=torch.float64, device=dev) if have_b else None

    # int8 slice codes (exact for rho >= 19) when every rank's GEMM can take them;
    # the ranks agree on the format of B's slices before any is broadcast.
    use_s8 = rho >= 19 and M >= 256
    if use_s8:
        nbmin = torch.tensor([nb], dtype=torch.int64, device=dev)
        dist.all_reduce(nbmin, op=dist.ReduceOp.MIN, group=group)
        use_s8 = int(nbmin.item()) >= 256
    if use_s8:
        k8 = (Kd + 127) // 128 * 128
        fail = torch.zeros(1, dtype=torch.int32, device=dev)
        SB = torch.empty((nS, M, k8), dtype=torch.int8, device=dev)
        eB = torch.empty((nS, M), dtype=torch.int32, device=dev)
        if have_b:
            L.check(lib.ozk_extract_cols_s8_f64(Bd.data_ptr(), Bd.stride(0), Kd, M, rho, n_hi,
                                                n_lo, SB.data_ptr(), k8, eB.data_ptr(),
                                                BT.data_ptr(), BT.numel() * 8, fail.data_ptr(),
                                                status.data_ptr(), sh))
        if b_source == "root":
            dist.broadcast(SB, src=0, group=group)
            dist.broadcast(eB, src=0, group=group)
            dist.broadcast(fail, src=0, group=group)
        SA = torch.empty((nS, nb, k8), dtype=torch.int8, device=dev)
        eA = torch.empty((nS, nb), dtype=torch.int32, device=dev)
        L.check(lib.ozk_extract_rows_s8_f64(Ad.data_ptr(), Ad.stride(0), nb, Kd, rho, n_hi, n_lo,
                                            SA.data_ptr(), k8, eA.data_ptr(), fail.data_ptr(),
                                            status.data_ptr(), sh))
        # a code without an exact int8 value anywhere sends every rank to BF16
        dist.all_reduce(fail, op=dist.ReduceOp.MAX, group=group)
        if int(fail.item()) == 0:
            L.check(lib.ozk_slice_gemm_s8(SA.data_ptr(), eA.data_ptr(), nS, SB.data_ptr(),
                                          eB.data_ptr(), nS, nb, M, k8, pa, pb, npairs, 0, 1.0,
                                          0.0, None, 0, C.data_ptr(), M, GW.data_ptr(), GW.numel(),
                                          rho, None, status.data_ptr(), sh))
        else:
            use_s8 = False
        del SA, SB
    if not use_s8:
        k_pad = (max(Kd, 1) + 63) // 64 * 64
        SB = torch.empty((nS, M, k_pad), dtype=torch.int16, device=dev)
        eB = torch.empty((nS, M), dtype=torch.int32, device=dev)
        if have_b:
            L.check(lib.ozk_extract_cols_f64(Bd.data_ptr(), Bd.stride(0), Kd, M, rho, n_hi, n_lo,
                                             SB.data_ptr(), k_pad, eB.data_ptr(), BT.data_ptr(),
                                             BT.numel() * 8, status.data_ptr(), sh))
        if b_source == "root":
            # NCCL has no 16-bit integer type: move the BF16 bit patterns as bytes
            dist.broadcast(SB.view(torch.uint8), src=0, group=group)
            dist.broadcast(eB, src=0, group=group)
        SA = torch.empty((nS, nb, k_pad), dtype=torch.int16, device=dev)
        eA = torch.empty((nS, nb), dtype=torch.int32, device=dev)
        if nb > 0:
            L.check(lib.ozk_extract_rows_f64(Ad.data_ptr(), Ad.stride(0), nb, Kd, rho, n_hi, n_lo,
                                             SA.data_ptr(), k_pad, eA.data_ptr(), status.data_ptr(),
                                             sh))
            L.check(lib.ozk_slice_gemm(SA.data_ptr(), eA.data_ptr(), nS, SB.data_ptr(),
                                       eB.data_ptr(), nS, nb, M, k_pad, pa, pb, npairs,
                                       L.OZK_ACC_FIXED, 0, 1.0, 0.0, None, 0, C.data_ptr(), M,
                                       None, GW.data_ptr(), GW.numel(), rho, status.data_ptr(), sh))
    flags = int(status.item())
    if flags:
        raise ValueError("Ozaki preflight marked this input as unsafe: inputs contain NaN or Inf"
                         if flags & (L.OZK_FLAG_NONFINITE | L.OZK_FLAG_RANGE)
                         else f"device status {flags}")
    return C


def matmul_rowsharded_host(A_local, B, precision="high", group=None):
    """This rank's rows of C = A @ B from host arrays, with B's upload split over
    the ranks.

    A_local: this rank's row block of A (NumPy, host).  B: the K x M matrix as a
    host array on every rank; rank r uploads only its share of B's rows
    (rows [r*ceil(K/P), (r+1)*ceil(K/P)) ), the shares are all-gathered over
    NCCL (NVLink) into the full B on every GPU, and the on-device pipeline runs
    on this rank's rows.  Each rank moves its A rows, 1/P of B and its C rows
    over PCIe instead of all of B.  Returns this rank's rows of C as NumPy,
    bit-identical to the same rows of the single-GPU result.  All ranks must
    call it.
    """
    from .matmul import _flags_reasons, _PREFIX
    n_hi, n_lo = _resolve_precision(precision)
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    dev = torch.device("cuda", torch.cuda.current_device())
    A = np.ascontiguousarray(A_local, dtype=np.float64)
    Bh = np.asarray(B, dtype=np.float64)
    if A.ndim != 2 or Bh.ndim != 2 or A.shape[1] != Bh.shape[0]:
        raise ValueError(f"Incompatible shapes for matmul: {A.shape} and {Bh.shape}.")
    K, M = Bh.shape
    kc = (K + world - 1) // world
    k0, k1 = min(K, rank * kc), min(K, (rank + 1) * kc)
    share = torch.zeros((kc, M), dtype=torch.float64, device=dev)
    if k1 > k0:
        share[: k1 - k0].copy_(D.to_device_f64(Bh[k0:k1], dev))
    gathered = torch.empty((world * kc, M), dtype=torch.float64, device=dev)
    dist.all_gather_into_tensor(gathered, share, group=group)
    Bd = gathered[:K]
    nb = A.shape[0]
    if nb == 0 or M == 0:
        return np.zeros((nb, M))
    # A and C stay on the host: the host-buffer pipeline streams them in row
    # blocks over PCIe while the blocks before are computed; B is read from
    # this GPU's gathered copy.
    lib = L.load()
    Ch = D.host_empty_f64((nb, M))
    ws_bytes = lib.ozk_matmul_hostbuf_workspace_bytes(nb, K, M, n_hi, n_lo, L.OZK_ACC_FIXED, 0)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    flags = ctypes.c_int32(0)
    L.check(lib.ozk_matmul_f64_hostbuf(
        A.ctypes.data, K, Bd.data_ptr(), M, Ch.ctypes.data, M, nb, K, M, compute_rho_f32(K),
        n_hi, n_lo, L.OZK_ACC_FIXED, 0, ws.data_ptr(), ws_bytes, ctypes.byref(flags),
        D.stream_handle(dev)))
    if flags.value & L.OZK_FLAG_TIMEOUT:
        raise L.OzakiError(L.OZK_ERR_TIMEOUT, "a device-side wait exceeded its time budget")
    if flags.value:
        raise ValueError(_PREFIX + "; ".join(_flags_reasons(flags.value)))
    return Ch


def residual_rowsharded(A_local, x, b_local, precision="high", accumulation="bf16_interleaved"):
    """This rank's rows of r = b - A x (residual(mode='ozaki')): rows of A and b
    are independent and x is given to every rank, so there is no collective;
    the result equals the same rows of the single-GPU residual bit for bit."""
    from .solve import residual
    return residual(A_local, x, b_local, precision=precision, accumulation=accumulation,
                    mode="ozaki")


def gram_rowsharded(A_local, precision="high", group=None):
    """This rank's block of rows of G = A^T A (gram(mode='ozaki')) with A's rows
    split over the ranks.

    A_local: this rank's rows of A (CUDA float64, N_r x K).  Rank r owns columns
    [rK/P, (r+1)K/P) of A and rows [rK/P, (r+1)K/P) of G:
      1. an all-to-all over NCCL gives each rank every row of its columns, so it
         extracts their slices (lines of length N) itself, as the single-GPU
         gram does;
      2. the slice stacks and exponents are all-gathered;
      3. each rank multiplies its lines' slices by all of them: its rows of G.
    Pair (a, b) of element (j, i) is pair (b, a) of element (i, j), and the pair
    set and the fixed-point term scaling are symmetric under that swap, so the
    rows equal the single-GPU symmetric gram bit for bit.  Returns this rank's
    rows of G (CUDA float64, K_r x K).  All ranks must call it.
    """
    from .matmul import _flags_reasons, _PREFIX
    lib = L.load()
    n_hi, n_lo = _resolve_precision(precision)
    nS = n_hi + n_lo
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    Ad = A_local.to(dtype=torch.float64).contiguous()
    dev = Ad.device
    n_loc, K = Ad.shape
    counts = [torch.zeros(1, dtype=torch.int64, device=dev) for _ in range(world)]
    dist.all_gather(counts, torch.tensor([n_loc], dtype=torch.int64, device=dev), group=group)
    counts = [int(c.item()) for c in counts]
    N = sum(counts)
    cols = [row_range(K, r, world) for r in range(world)]
    c0, c1 = cols[rank]
    kr = c1 - c0
    # 1. columns of A to their owners
    send = torch.cat([Ad[:, a:b].reshape(-1) for a, b in cols])
    recv = torch.empty(N * kr, dtype=torch.float64, device=dev)
    dist.all_to_all_single(recv, send, output_split_sizes=[n * kr for n in counts],
                           input_split_sizes=[n_loc * (b - a) for a, b in cols], group=group)
    A_cols = torch.cat([blk.view(n, kr) for blk, n in zip(recv.split([n * kr for n in counts]),
                                                          counts)])  # N x kr
    rho = compute_rho_f32(N)
    kmax = max(b - a for a, b in cols)
    # the slice format is decided the same way on every rank
    use_s8 = rho >= 19 and min(b - a for a, b in cols) >= 256 and K >= 256 and N <= 65536
    sh = D.stream_handle(dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    pa = (ctypes.c_uint8 * 256)()
    pb = (ctypes.c_uint8 * 256)()
    npairs = L.check(lib.ozk_pair_schedule_snake(n_hi, n_lo, pa, pb, 256))
    GW = torch.empty(lib.ozk_slice_gemm_workspace_bytes(), dtype=torch.uint8, device=dev)
    BT = torch.empty(max(kr * N, 1), dtype=torch.float64, device=dev)
    G = torch.empty((kr, K), dtype=torch.float64, device=dev)

    def slices_and_gemm(s8):
        n_pad = (N + 127) // 128 * 128 if s8 else (N + 63) // 64 * 64
        dt = torch.int8 if s8 else torch.int16
        S = torch.zeros((nS, kmax, n_pad), dtype=dt, device=dev)
        E = torch.zeros((nS, kmax), dtype=torch.int32, device=dev)
        fail = torch.zeros(1, dtype=torch.int32, device=dev)
        # this rank's lines: slices [nS][kr][n_pad], padded to kmax lines for the gather
        Sk = torch.empty((nS, kr, n_pad), dtype=dt, device=dev)
        Ek = torch.empty((nS, kr), dtype=torch.int32, device=dev)
        if kr > 0:
            if s8:
                L.check(lib.ozk_extract_cols_s8_f64(
                    A_cols.data_ptr(), kr, N, kr, rho, n_hi, n_lo, Sk.data_ptr(), n_pad,
                    Ek.data_ptr(), BT.data_ptr(), BT.numel() * 8, fail.data_ptr(),
                    status.data_ptr(), sh))
            else:
                L.check(lib.ozk_extract_cols_f64(
                    A_cols.data_ptr(), kr, N, kr, rho, n_hi, n_lo, Sk.data_ptr(), n_pad,
                    Ek.data_ptr(), BT.data_ptr(), BT.numel() * 8, status.data_ptr(), sh))
            S[:, :kr] = Sk
            E[:, :kr] = Ek
        if s8:
            # a code without an exact int8 value on any rank sends every rank to BF16
            dist.all_reduce(fail, op=dist.ReduceOp.MAX, group=group)
            if int(fail.item()):
                return False
        # 2. every rank's slices: [P][nS][kmax][n_pad] -> [nS][K][n_pad]
        allS = torch.empty((world,) + tuple(S.shape), dtype=dt, device=dev)
        allE = torch.empty((world,) + tuple(E.shape), dtype=torch.int32, device=dev)
        dist.all_gather_into_tensor(allS.view(torch.uint8), S.view(torch.uint8), group=group)
        dist.all_gather_into_tensor(allE, E, group=group)
        SB = torch.cat([allS[r, :, : b - a] for r, (a, b) in enumerate(cols)], dim=1).contiguous()
        EB = torch.cat([allE[r, :, : b - a] for r, (a, b) in enumerate(cols)], dim=1).contiguous()
        if kr == 0:
            return True
        # 3. this rank's rows of G
        if s8:
            L.check(lib.ozk_slice_gemm_s8(Sk.data_ptr(), Ek.data_ptr(), nS, SB.data_ptr(),
                                          EB.data_ptr(), nS, kr, K, n_pad, pa, pb, npairs, 0, 1.0,
                                          0.0, None, 0, G.data_ptr(), K, GW.data_ptr(), GW.numel(),
                                          rho, None, status.data_ptr(), sh))
        else:
            L.check(lib.ozk_slice_gemm(Sk.data_ptr(), Ek.data_ptr(), nS, SB.data_ptr(),
                                       EB.data_ptr(), nS, kr, K, n_pad, pa, pb, npairs,
                                       L.OZK_ACC_FIXED, 0, 1.0, 0.0, None, 0, G.data_ptr(), K,
                                       None, GW.data_ptr(), GW.numel(), rho, status.data_ptr(),
                                       sh))
        return True

    if not (use_s8 and slices_and_gemm(True)):
        slices_and_gemm(False)
    flags = int(status.item())
    if flags:
        raise ValueError(_PREFIX + "; ".join(_flags_reasons(flags)))
    return G
