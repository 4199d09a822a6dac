"""Row-sharded Ozaki matmul over the GPUs of one node (one process per GPU).

The reference has no multi-device code; this is the build's partitioning of
the on-device path.  Rank r owns rows [r*N/P, (r+1)*N/P) of A and of C.  Row
extraction is row-local, so each rank's slices of A are bit-identical to the
single-GPU ones and each rank's block of C equals the corresponding rows of
the single-GPU result.  B reaches every rank in one of three ways:

  b_source='replicated'  every rank was given B and extracts its column slices
                         locally (no exchange of B);
  b_source='root'        rank 0 extracts B's slices once and broadcasts the slice
                         stack (int8 codes where exact, else BF16) and exponents
                         over NCCL (NVLink);
  b_source='columns'     rank r holds columns column_range(M, r, P) of B, extracts
                         them, and the slice stacks are all-gathered over NCCL.

matmul_rowsharded runs the library's multi-GPU operator (ozk_matmul_f64_multi
on an ozk_context with its own NCCL communicator); argument agreement and the
other helpers use torch.distributed (NCCL for CUDA tensors, gloo on CPU).
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


def _meta_device(dev, group):
    """Device for small host-logic collectives: the compute device under NCCL,
    the CPU under gloo."""
    return dev if dist.get_backend(group) == "nccl" else torch.device("cpu")


def _agree(err, values, dev, group):
    """Every rank contributes `err` (a message, or None when its arguments are
    valid) and a list of int64 `values`; one all_gather gives every rank all of
    them.  If any rank's arguments are invalid, every rank raises ValueError
    before the first data collective, so no rank is left waiting in one.
    Returns the gathered values, one list per rank."""
    world = dist.get_world_size(group)
    mdev = _meta_device(dev, group)
    mine = torch.tensor([1 if err else 0] + [int(v) for v in values], dtype=torch.int64,
                        device=mdev)
    parts = [torch.empty_like(mine) for _ in range(world)]
    dist.all_gather(parts, mine, group=group)
    rows = [p.tolist() for p in parts]
    bad = [r for r, row in enumerate(rows) if row[0]]
    if bad:
        raise ValueError(err if err else f"invalid arguments on rank(s) {bad}")
    return [row[1:] for row in rows]


_FLAG_BITS = 8


def _or_status(status, group):
    """Bitwise OR of the OZK_FLAG_* words of all ranks (collectives have no OR:
    the bits are spread into words and reduced with MAX), written back into
    `status` in place.  Every rank then raises for a bad value in any rank's
    operands, as the single-GPU call does."""
    mdev = _meta_device(status.device, group)
    bits = ((status.to(mdev).view(1) >> torch.arange(_FLAG_BITS, device=mdev)) & 1).to(torch.int32)
    dist.all_reduce(bits, op=dist.ReduceOp.MAX, group=group)
    word = int((bits.to(torch.int64) << torch.arange(_FLAG_BITS, device=mdev)).sum().item())
    status.fill_(word)
    return word


class MultiContext:
    """The library's multi-GPU context (ozk_context) for this process's GPU in a
    torch.distributed job: one NCCL communicator over the ranks of `group`,
    made from an id that rank 0 creates and the process group broadcasts."""

    def __init__(self, group=None):
        lib = L.load()
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = torch.cuda.current_device()
        idbuf = ctypes.create_string_buffer(L.OZK_NCCL_ID_BYTES)
        err = None
        if self.rank == 0:
            rc = lib.ozk_nccl_unique_id(idbuf, L.OZK_NCCL_ID_BYTES)
            err = None if rc == 0 else L.detail()
        box = [bytes(idbuf.raw) if err is None else None, err]
        dist.broadcast_object_list(box, src=dist.get_global_rank(group, 0) if group else 0,
                                   group=group)
        if box[1] is not None:
            raise L.OzakiError(L.OZK_ERR_NCCL, box[1])
        idbuf = ctypes.create_string_buffer(box[0], L.OZK_NCCL_ID_BYTES)
        self.ptr = ctypes.c_void_p()
        L.check(lib.ozk_context_create_rank(ctypes.byref(self.ptr), self.world, self.rank, idbuf,
                                            L.OZK_NCCL_ID_BYTES, self.device))

    def wait(self, dev):
        """Bounded wait for the work NOWAIT calls enqueued on the current stream
        of `dev` (ozk_context_wait): raises OzakiError (OZK_ERR_TIMEOUT or
        OZK_ERR_NCCL, the context then unusable) where a peer failed."""
        L.check(L.load().ozk_context_wait(
            self.ptr, (ctypes.c_void_p * 1)(D.stream_handle(dev))))

    def close(self):
        if self.ptr:
            L.check(L.load().ozk_context_destroy(self.ptr))
            self.ptr = ctypes.c_void_p()


_CONTEXTS = {}


def context(group=None):
    """The cached MultiContext of `group` on the current GPU (created by a
    collective call on first use: every rank must ask for it together)."""
    key = (id(group), torch.cuda.current_device())
    if key not in _CONTEXTS:
        _CONTEXTS[key] = MultiContext(group)
    return _CONTEXTS[key]


def close_contexts():
    """Destroys the cached contexts (call on every rank before
    destroy_process_group)."""
    for c in _CONTEXTS.values():
        c.close()
    _CONTEXTS.clear()


_B_MODES = {"replicated": L.OZK_B_REPLICATED, "root": L.OZK_B_ROOT, "columns": L.OZK_B_COLUMNS}


def column_range(m, rank, world):
    """Columns [c0, c1) of an m-column B held by `rank` with b_source='columns':
    blocks of ceil(m / world) columns, the last one shorter."""
    mc = (m + world - 1) // world
    return min(m, rank * mc), min(m, (rank + 1) * mc)


def matmul_rowsharded(A_local, B, precision="high", b_source="replicated", group=None):
    """C_local = (A @ B)[rows of this rank] with the Ozaki 'fused' accumulation,
    through the library's multi-GPU operator (ozk_matmul_f64_multi, NCCL).

    A_local: this rank's row block of A (CUDA float64), rows row_range(N, r, P).
    B: 'replicated': the full K x M matrix on every rank;
       'root': the full matrix on rank 0 (other ranks may pass None); its slice
               stack and exponents are broadcast;
       'columns': this rank's columns column_range(M, r, P) of B (K x m_r); the
               slice stacks are all-gathered.
    Returns this rank's rows of C (CUDA float64), bit-identical to the same rows
    of the single-GPU result.  All ranks must call it.
    """
    lib = L.load()
    n_hi, n_lo = _resolve_precision(precision)
    dev = A_local.device
    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    # arguments are checked on every rank and agreed on before any data moves
    err = None
    if b_source not in _B_MODES:
        err = f"b_source must be one of {sorted(_B_MODES)}"
    elif A_local.dim() != 2:
        err = f"A_local must be 2-D, got shape {tuple(A_local.shape)}"
    elif (b_source != "root" or rank == 0) and (B is None or B.dim() != 2):
        err = "B must be a 2-D tensor on " + ("rank 0" if b_source == "root" else "every rank")
    nb, Kd = tuple(A_local.shape) if A_local.dim() == 2 else (0, 0)
    Kb, Mb = tuple(B.shape) if (err is None and B is not None and B.dim() == 2) else (-1, -1)
    meta = _agree(err, [nb, Kd, Kb, Mb], dev, group)
    N = sum(row[0] for row in meta)
    if any(row[0] != row_range(N, r, world)[1] - row_range(N, r, world)[0]
           for r, row in enumerate(meta)):
        raise ValueError(f"A's row blocks must follow row_range({N}, rank, {world}); got "
                         f"{[row[0] for row in meta]}")
    if b_source == "columns":
        M = sum(row[3] for row in meta)
        want = [column_range(M, r, world)[1] - column_range(M, r, world)[0] for r in range(world)]
        if [row[3] for row in meta] != want:
            raise ValueError(f"B's column blocks must follow column_range({M}, rank, {world}): "
                             f"{want}; got {[row[3] for row in meta]}")
        holders = range(world)
    elif b_source == "root":
        M = meta[0][3]
        holders = [0]
    else:
        M = meta[0][3]
        if any(row[3] != M for row in meta):
            raise ValueError("B must have the same shape on every rank")
        holders = range(world)
    K = meta[0][1]
    bad = [r for r, row in enumerate(meta) if row[1] != K or (r in holders and row[2] != K)]
    if bad:
        raise ValueError(f"Incompatible shapes for matmul: A_local has {meta[bad[0]][1]} columns "
                         f"and B {meta[bad[0]][2]} rows on rank {bad[0]}.")
    if K < 1 or M < 1:
        raise ValueError(f"K and M must be >= 1 (got K={K}, M={M})")
    ctx = context(group)
    Ad = A_local.to(dtype=torch.float64).contiguous()
    Bd = (B.to(device=dev, dtype=torch.float64).contiguous()
          if (B is not None and rank in holders) else None)
    C = torch.empty((nb, M), dtype=torch.float64, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    P = ctypes.c_void_p
    I64 = ctypes.c_int64

    def call(flags):
        L.check(lib.ozk_matmul_f64_multi(
            ctx.ptr, (P * 1)(Ad.data_ptr()), (I64 * 1)(K),
            (P * 1)(Bd.data_ptr() if Bd is not None else None),
            (I64 * 1)(Bd.shape[1] if Bd is not None else 0), (P * 1)(C.data_ptr()), (I64 * 1)(M),
            N, K, M, n_hi, n_lo, _B_MODES[b_source], flags, (P * 1)(D.stream_handle(dev)),
            (P * 1)(status.data_ptr())))
        # a bounded wait: a peer that failed ends it with an error, not a hang
        ctx.wait(dev)

    call(L.OZK_MULTI_NOWAIT)
    flags = int(status.item())  # the OZK_FLAG_* bits of every rank
    if flags & L.OZK_FLAG_REDO:
        # a slice had no exact int8 code on some rank: every rank sees it and
        # repeats with BF16 slices
        status.zero_()
        call(L.OZK_MULTI_NOWAIT | L.OZK_MULTI_BF16)
        flags = int(status.item())
    if flags & L.OZK_FLAG_TIMEOUT:
        raise L.OzakiError(L.OZK_ERR_TIMEOUT, "a device-side wait exceeded its time budget")
    if flags:
        from .matmul import _flags_reasons, _PREFIX
        raise ValueError(_PREFIX + "; ".join(_flags_reasons(flags)))
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
    dev = (torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available()
           else torch.device("cpu"))
    A = np.ascontiguousarray(A_local, dtype=np.float64)
    Bh = np.asarray(B, dtype=np.float64)
    err = None
    if A.ndim != 2 or Bh.ndim != 2 or A.shape[1] != Bh.shape[0]:
        err = f"Incompatible shapes for matmul: {A.shape} and {Bh.shape}."
    K, M = Bh.shape if Bh.ndim == 2 else (-1, -1)
    meta = _agree(err, [K, M], dev, group)
    if any(row != [K, M] for row in meta):
        raise ValueError(f"B must have the same shape on every rank; got {[tuple(r) for r in meta]}")
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
        _or_status(torch.zeros(1, dtype=torch.int32, device=dev), group)  # same steps as the others
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
    # a bad value in any rank's rows makes every rank raise, as one GPU would
    word = _or_status(torch.tensor([flags.value], dtype=torch.int32, device=dev), group)
    if word & L.OZK_FLAG_TIMEOUT:
        raise L.OzakiError(L.OZK_ERR_TIMEOUT, "a device-side wait exceeded its time budget")
    if word:
        raise ValueError(_PREFIX + "; ".join(_flags_reasons(word)))
    return Ch


def residual_rowsharded(A_local, x, b_local, precision="high", accumulation="bf16_interleaved"):
    """This rank's rows of r = b - A x (residual(mode='ozaki')): rows of A and b
    are independent and x is given to every rank, so there is no collective;
    the result equals the same rows of the single-GPU residual bit for bit."""
    from .solve import residual
    return residual(A_local, x, b_local, precision=precision, accumulation=accumulation,
                    mode="ozaki")


def _gram_reduced(lib, Ad, N, K, n_hi, n_lo, group):
    """G = A^T A through ozk_gram_f64_multi (partial int64 Gram sums reduced over
    the ranks).  Returns (G on this rank, OZK_FLAG_* bits of all ranks), or
    None where the operator does not apply (the same decision on every rank)."""
    ctx = context(group)
    dev = Ad.device
    G = torch.empty((K, K), dtype=torch.float64, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    P, I64 = ctypes.c_void_p, ctypes.c_int64
    rc = lib.ozk_gram_f64_multi(ctx.ptr, (P * 1)(Ad.data_ptr() if Ad.numel() else None),
                                (I64 * 1)(K), (P * 1)(G.data_ptr()), (I64 * 1)(K), N, K, n_hi,
                                n_lo, L.OZK_MULTI_NOWAIT, (P * 1)(D.stream_handle(dev)),
                                (P * 1)(status.data_ptr()))
    if rc == L.OZK_ERR_UNSUPPORTED:
        return None
    L.check(rc)
    ctx.wait(dev)
    return G, int(status.item())


def gram_rowsharded(A_local, precision="high", group=None, full=False):
    """This rank's block of rows of G = A^T A (gram(mode='ozaki')) with A's rows
    split over the ranks (all of G with full=True).

    With int8 slice codes (N > 4096, K >= 256) and A's rows on row_range(N, r, P),
    this is ozk_gram_f64_multi, the reduction of partial Gram blocks: each slice
    pass takes the lines' maxima over all ranks, each rank's int8 GEMM adds up
    its rows' exact pair products in int64, the sums are all-reduced exactly and
    rounded to FP64 once.  Each pair's term is rounded at 2^-36 of the top
    product grid on each rank's part, so a rare element can differ from the
    single-GPU gram in its last bit (bit-identical with one rank).

    Otherwise (and if a slice has no exact int8 code on some rank) A's columns
    travel instead.  Rank r owns columns [rK/P, (r+1)K/P) of A and rows
    [rK/P, (r+1)K/P) of G:
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
    dev = A_local.device
    err = None if A_local.dim() == 2 else f"A_local must be 2-D, got shape {tuple(A_local.shape)}"
    n_loc, K = tuple(A_local.shape) if err is None else (0, -1)
    meta = _agree(err, [n_loc, K], dev, group)
    if any(row[1] != K for row in meta):
        raise ValueError(f"A_local must have the same column count on every rank; got "
                         f"{[row[1] for row in meta]}")
    Ad = A_local.to(dtype=torch.float64).contiguous()
    counts = [row[0] for row in meta]
    N = sum(counts)
    if N < 1:
        raise ValueError("gram needs at least one row")
    cols = [row_range(K, r, world) for r in range(world)]
    c0, c1 = cols[rank]
    kr = c1 - c0
    if all(n == row_range(N, r, world)[1] - row_range(N, r, world)[0]
           for r, n in enumerate(counts)):
        got = _gram_reduced(lib, Ad, N, K, n_hi, n_lo, group)
        if got is not None and not got[1] & L.OZK_FLAG_REDO:
            Gf, flags = got
            if flags & L.OZK_FLAG_TIMEOUT:
                raise L.OzakiError(L.OZK_ERR_TIMEOUT, "a device-side wait exceeded its time budget")
            if flags:
                raise ValueError(_PREFIX + "; ".join(_flags_reasons(flags)))
            return Gf if full else Gf[c0:c1]
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
    flags = _or_status(status, group)
    if flags & L.OZK_FLAG_TIMEOUT:
        raise L.OzakiError(L.OZK_ERR_TIMEOUT, "a device-side wait exceeded its time budget")
    if flags:
        raise ValueError(_PREFIX + "; ".join(_flags_reasons(flags)))
    if full:
        return gather_rows(G, K, group=group)
    return G
