/*
 * ozaki_b200.h -- C ABI of libozaki_b200.so, the B200 (sm_100a) kernels behind
 * the Ozaki FP64-emulation matmul path of Efithor/ozaki-jax.
 *
 * The reference runs this path as jitted JAX/XLA (or Pallas-TPU) operators
 * with static integer arguments and device FP64 arrays in and out.  Each entry
 * point below replaces one of them; the comment on each names the reference
 * function (file:line, paths inside the reference project) it stands in for.
 *
 * Conventions
 *   - All matrices are row-major (C order, as NumPy and JAX use); `ld*` are
 *     leading dimensions in elements.  Pointers to matrices are DEVICE pointers.
 *   - Calls are asynchronous and ordered on `stream` (a cudaStream_t passed as
 *     void*; NULL = legacy default stream).  Nothing is synchronised inside
 *     a call unless its comment says so.
 *   - Return value: OZK_OK (0) when the work was validated and enqueued, or a
 *     negative ozk_status.  Conditions found by a kernel (non-finite input, a
 *     device-side wait that ran out of time) are OR-ed as OZK_FLAG_* bits into
 *     the caller's device word `status_dev` (int32, may be NULL to skip); read
 *     it after the stream completes, or call ozk_check_status().
 *   - Slices are BF16 bit patterns (uint16); exponents are int32.
 *   - No C++ exceptions cross this boundary; no global mutable state other
 *     than per-device caches created on first use.
 */
#ifndef OZAKI_B200_H
#define OZAKI_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  OZK_OK = 0,
  OZK_ERR_ARG = -1,         /* invalid argument (shape, mode, pointer, size) */
  OZK_ERR_UNSAFE = -2,      /* preflight bound violated (bits <= 0, K bound) */
  OZK_ERR_NONFINITE = -3,   /* an input holds NaN/Inf or overflows FP32 */
  OZK_ERR_CUDA = -4,        /* a CUDA runtime/driver call failed */
  OZK_ERR_NCCL = -5,        /* a collective failed */
  OZK_ERR_TIMEOUT = -6,     /* a device-side wait exceeded its time budget */
  OZK_ERR_WORKSPACE = -7,   /* caller workspace too small */
  OZK_ERR_UNSUPPORTED = -8  /* valid request this build does not handle */
} ozk_status;

/* Bits OR-ed into *status_dev by kernels. */
#define OZK_FLAG_NONFINITE 0x1  /* non-finite value seen while splitting */
#define OZK_FLAG_TIMEOUT 0x2    /* a bounded device wait gave up */
#define OZK_FLAG_RANGE 0x4      /* a finite FP64 input overflows FP32 when split */

/* Accumulation modes of ozk_slice_gemm. */
#define OZK_ACC_F64 0       /* FP64 running sum in the GEMM epilogue -> C (double) */
#define OZK_ACC_PRODUCTS 1  /* write each pair's exact FP32 product -> products */
#define OZK_ACC_FIXED 2     /* exact int64 fixed-point sum (on-device slices) -> C */

/* ---------------------------------------------------------------- policies */

/* _compute_rho_f32 (ozaki_jax/extract.py:109-113). */
int ozk_compute_rho_f32(int64_t K);
/* _compute_rho (ozaki_jax/extract.py:12-18), FP64 host pipeline. */
int ozk_compute_rho_f64(int64_t K);
/* _make_pair_schedule (ozaki_jax/pallas_gemm_accum.py:26-87): writes the
 * slice-pair order (hi x hi, hi x lo, lo x hi) into pair_a/pair_b (capacity
 * `cap`) and returns the pair count, or OZK_ERR_ARG. */
int ozk_pair_schedule(int n_hi, int n_lo, uint8_t* pair_a, uint8_t* pair_b, int cap);
/* The same pairs in an L2-friendly order (consecutive pairs share an operand
 * slice), used with order-independent OZK_ACC_FIXED sums. */
int ozk_pair_schedule_snake(int n_hi, int n_lo, uint8_t* pair_a, uint8_t* pair_b, int cap);
/* Host-pipeline triangular schedule i + j <= n-1 (ozaki_jax/matmul.py:23-32). */
int ozk_triangular_schedule(int n_slices, uint8_t* pair_a, uint8_t* pair_b, int cap);

/* ---------------------------------------------------------------- kernels */

/* Row extraction of an FP64 matrix X (rows x K, ldx): double-FP32 split
 * (_jax_double_f32_split, ozaki_jax/matmul.py:204-213) followed by n_hi
 * sigma-trick slices of the hi part and n_lo of the lo part
 * (jax_extract_split_rows, ozaki_jax/extract.py:197-242), bit-identical to the
 * reference.  slices: [n_hi+n_lo][rows][k_pad] BF16 (k_pad >= K, multiple of
 * 64; columns K..k_pad-1 are written as zeros); exps: [n_hi+n_lo][rows]. */
int ozk_extract_rows_f64(const double* X, int64_t ldx, int64_t rows, int64_t K, int rho,
                         int n_hi, int n_lo, uint16_t* slices, int64_t k_pad, int32_t* exps,
                         int32_t* status_dev, void* stream);

/* Column extraction of X (K x cols, ldx) (jax_extract_split_cols,
 * ozaki_jax/extract.py:245-286), written transposed: slices
 * [n_hi+n_lo][cols][k_pad] (K contiguous), exps [n_hi+n_lo][cols].
 * scratch: optional device buffer of cols*K doubles for the transposed fast
 * path (NULL: taken from the stream-ordered pool). */
int ozk_extract_cols_f64(const double* X, int64_t ldx, int64_t K, int64_t cols, int rho,
                         int n_hi, int n_lo, uint16_t* slices, int64_t k_pad, int32_t* exps,
                         double* scratch, size_t scratch_bytes, int32_t* status_dev,
                         void* stream);

/* FP64 sigma-trick extraction of the host pipeline (extract_split_rows /
 * extract_split_cols, ozaki_jax/extract.py:21-103): n_slices slices of the
 * FP64 input itself, same layouts as above. */
int ozk_extract_rows_host_f64(const double* X, int64_t ldx, int64_t rows, int64_t K, int rho,
                              int n_slices, uint16_t* slices, int64_t k_pad, int32_t* exps,
                              int32_t* status_dev, void* stream);
int ozk_extract_cols_host_f64(const double* X, int64_t ldx, int64_t K, int64_t cols, int rho,
                              int n_slices, uint16_t* slices, int64_t k_pad, int32_t* exps,
                              int32_t* status_dev, void* stream);

/* Persistent tcgen05/TMEM slice-pair GEMM over a pair list, replacing the
 * slice GEMMs and the scaled 2Sum accumulation of the reference
 * (ozaki_jax/matmul.py:248-281, :418-488; ozaki_jax/pallas_ops.py:178-239;
 * the fused Pallas kernel ozaki_jax/pallas_gemm_accum.py:90-316).
 *   SA: [nA][N][k_pad] BF16 left slices, eA: [nA][N];
 *   SB: [nB][M][k_pad] BF16 right slices (K contiguous), eB: [nB][M].
 *   Pair p multiplies SA[pair_a[p]] by SB[pair_b[p]]^T; pair_a/pair_b are
 *   HOST arrays of n_pairs (<= 128) entries.
 * mode OZK_ACC_F64:  C[r][c] = beta*Cin[r][c] + alpha * sum_p P_p[r][c]
 *                    * 2^(eA[a][r] + eB[b][c]), summed in FP64 in pair order
 *                    (Cin may be NULL when beta == 0).
 * mode OZK_ACC_FIXED: the same sum computed exactly in an int64 per element whose
 *                    unit is 2^(2(rho-24) - 36 + eA[0][r] + eB[0][c]) (slice 0 must be
 *                    the top slice on both sides, rho the extraction's), rounded
 *                    to FP64 once: accuracy of an FP64 sum without FP64 work per pair.
 * mode OZK_ACC_PRODUCTS: products[p][r][c] = P_p[r][c] (FP32, exact), ld = M.
 * symmetric != 0 (gram): requires SA == SB, eA == eB, N == M; only tiles on
 * or above the diagonal are computed and each is also written mirrored, so C
 * is exactly symmetric.
 * workspace: optional device scratch of ozk_slice_gemm_workspace_bytes()
 * bytes (256-byte aligned). */
int ozk_slice_gemm(const uint16_t* SA, const int32_t* eA, int nA, const uint16_t* SB,
                   const int32_t* eB, int nB, int64_t N, int64_t M, int64_t k_pad,
                   const uint8_t* pair_a, const uint8_t* pair_b, int n_pairs, int mode,
                   int symmetric, double alpha, double beta, const double* Cin, int64_t ldcin,
                   double* C, int64_t ldc, float* products, void* workspace, size_t ws_bytes,
                   int rho, int32_t* status_dev, void* stream);
/* Scratch ozk_slice_gemm uses for its 256-wide tiles (per-CTA FP64 running
 * sums, L2-resident); with a smaller or NULL workspace it runs 128-wide tiles
 * that keep the sums in TMEM. */
size_t ozk_slice_gemm_workspace_bytes(void);

/* int8 slice codes (no counterpart in the reference: an exact re-encoding of
 * its BF16 slices for the tensor cores' integer path).  Every slice of the
 * on-device extraction is an integer multiple of 2^(rho-24) of magnitude at
 * most 2^(25-rho); for rho >= 19 (K > 4096 with the reference's rho) the code
 * q = slice * 2^(24-rho) is an exact int8 with |q| <= 64, and an int8 x int8
 * MMA with int32 accumulation gives exactly the per-pair products the BF16
 * slices give in FP32.  Same recurrence and exponents as
 * ozk_extract_rows_f64 / ozk_extract_cols_f64; slices [n_hi+n_lo][lines][k_pad]
 * int8 with k_pad a multiple of 128 (<= 65536).  A value without an exact code
 * (slices of lines whose magnitude leaves the FP32 range the recurrence needs)
 * sets *fail_dev = 1: the codes are then unusable and the BF16 entry points
 * must be used.  The column form needs cols*K doubles of scratch (NULL: taken
 * from the stream-ordered pool). */
int ozk_extract_rows_s8_f64(const double* X, int64_t ldx, int64_t rows, int64_t K, int rho,
                            int n_hi, int n_lo, int8_t* slices, int64_t k_pad, int32_t* exps,
                            int32_t* fail_dev, int32_t* status_dev, void* stream);
int ozk_extract_cols_s8_f64(const double* X, int64_t ldx, int64_t K, int64_t cols, int rho,
                            int n_hi, int n_lo, int8_t* slices, int64_t k_pad, int32_t* exps,
                            double* scratch, size_t scratch_bytes, int32_t* fail_dev,
                            int32_t* status_dev, void* stream);

/* ozk_slice_gemm in OZK_ACC_FIXED mode on int8 slice codes (kind::i8 MMAs,
 * int32 accumulators): the same C bit for bit as the BF16 slices give.  Needs
 * rho >= 19, N and M >= 256, k_pad a multiple of 128 and a workspace of
 * ozk_slice_gemm_workspace_bytes().  With skip_if_dev non-NULL the GEMM does
 * nothing when *skip_if_dev != 0 (pass the extraction's fail word to keep a
 * failed extraction from producing a result, without a host round trip). */
int ozk_slice_gemm_s8(const int8_t* SA, const int32_t* eA, int nA, const int8_t* SB,
                      const int32_t* eB, int nB, int64_t N, int64_t M, int64_t k_pad,
                      const uint8_t* pair_a, const uint8_t* pair_b, int n_pairs, int symmetric,
                      double alpha, double beta, const double* Cin, int64_t ldcin, double* C,
                      int64_t ldc, void* workspace, size_t ws_bytes, int rho,
                      const int32_t* skip_if_dev, int32_t* status_dev, void* stream);

/* Reference-order FP32 2Sum accumulation of materialised products
 * (accumulate_2sum / _accumulate_2sum_logic, ozaki_jax/pallas_ops.py:178-239,
 * :372-396, with the scales of _precompute_accumulation_scales, :107-175):
 * products [n_pairs][N][M] in ondevice_pairs(n_hi, n_lo) order; writes
 * C_hi, C_lo (FP32, may be NULL) and C = f64(C_hi) + f64(C_lo) (may be NULL).
 * Bit-identical to the reference's fused / ondevice accumulation. */
int ozk_accumulate_2sum(const float* products, const int32_t* eA, const int32_t* eB,
                        int64_t N, int64_t M, int n_hi, int n_lo, float* C_hi, float* C_lo,
                        double* C, int64_t ldc, void* stream);

/* The general accumulate_2sum of the reference (accumulate_2sum with
 * backend 'auto'/'jax'/'pallas', ozaki_jax/pallas_ops.py:372-396, arithmetic
 * :178-239): products [n_products][N][M] FP32, col_scales [n_products][M]
 * FP32, row_scales [n_groups][N] FP32, all on the device; the block structure
 * block_group_sizes as HOST arrays: group_sizes[g] products per group, and
 * block_ends[b] = one past the last group of block b (n_blocks <= 8).
 * Writes C_hi, C_lo (FP32 [N][M], either may be NULL), bit-identical to the
 * reference. */
int ozk_accumulate_2sum_scaled(const float* products, const float* col_scales,
                               const float* row_scales, const int32_t* group_sizes, int n_groups,
                               const int32_t* block_ends, int n_blocks, int64_t N, int64_t M,
                               float* C_hi, float* C_lo, void* stream);

/* ---------------------------------------------------------------- pipelines */

/* Workspace bytes ozk_matmul_f64 uses for an N x K by K x M product with
 * (n_hi, n_lo) slices on the current device.  A smaller workspace down to the
 * slices-only size is accepted and selects 128-wide GEMM tiles. */
size_t ozk_matmul_workspace_bytes(int64_t N, int64_t K, int64_t M, int n_hi, int n_lo);

/* The on-device pipeline (_matmul_ondevice accumulation='fused' /
 * 'bf16_interleaved' -> _fully_fused_f64_jit / _bf16_interleaved_f64_jit,
 * ozaki_jax/matmul.py:514-540, :641-686): C = A @ B with FP64 inputs and
 * output on the device.  rho < 0 selects _compute_rho_f32(K).  workspace may be
 * NULL (then it is taken from the stream-ordered pool and returned).
 * acc_mode: OZK_ACC_FIXED (exact int64 fixed-point sums, rounded to FP64 once:
 * the 'fused' / 'bf16_interleaved' default), OZK_ACC_F64 (FP64 sums in pair
 * order: the reference's FP64 'host' accumulation) or OZK_ACC_PRODUCTS
 * (materialised products + the reference's FP32 2Sum, bit-identical to the
 * reference's 'ondevice' / 'fused' result). */
int ozk_matmul_f64(const double* A, int64_t lda, const double* B, int64_t ldb, double* C,
                   int64_t ldc, int64_t N, int64_t K, int64_t M, int rho, int n_hi, int n_lo,
                   int acc_mode, void* workspace, size_t ws_bytes, int32_t* status_dev,
                   void* stream);

/* The on-device pipeline called with HOST arrays (ozaki_jax.matmul on NumPy
 * inputs with pipeline='ondevice', ozaki_jax/matmul.py:781-821 -> :641-686,
 * where the arrays are transferred to the device, the jitted pipeline runs and
 * the result comes back to the host): A, B, C are host pointers (pinned memory
 * copies at full DMA speed; pageable memory works through the driver's
 * staging); any of them may also be device memory of this GPU (unified
 * addressing picks the copy direction; pageable host arrays go through the
 * page-locked staging of ozk_memcpy_staged).  The copies overlap the compute: B is copied and column-extracted
 * first, then A and C move in row blocks of block_rows rows (0 = automatic) on
 * two internal copy streams while the previous block's slice GEMM runs on
 * `stream`.  Blocking: returns after C is written; *status_host receives the
 * OZK_FLAG_* bits of the run (0 = clean).  acc_mode as for ozk_matmul_f64;
 * workspace as sized by ozk_matmul_hostbuf_workspace_bytes, or NULL for the
 * stream-ordered pool. */
size_t ozk_matmul_hostbuf_workspace_bytes(int64_t N, int64_t K, int64_t M, int n_hi, int n_lo,
                                          int acc_mode, int64_t block_rows);
int ozk_matmul_f64_hostbuf(const double* A, int64_t lda, const double* B, int64_t ldb, double* C,
                           int64_t ldc, int64_t N, int64_t K, int64_t M, int rho, int n_hi,
                           int n_lo, int acc_mode, int64_t block_rows, void* workspace,
                           size_t ws_bytes, int32_t* status_host, void* stream);

/* Host <-> device copy of `bytes` (no counterpart in the reference: the
 * reference's jnp.asarray / np.asarray transfers, ozaki_jax/matmul.py:803-821).
 * One of dst, src is device memory of the current GPU, the other host memory.
 * Pageable host memory goes through the library's page-locked staging ring
 * with host memcpy threads (the driver's own staging of pageable memory is
 * several times slower than PCIe); page-locked host memory is copied
 * directly.  Blocking: returns when the copy is complete (after the work
 * already on `stream`). */
int ozk_memcpy_staged(void* dst, const void* src, size_t bytes, void* stream);

/* Allocation-free variant of ozk_matmul_f64 (acc_mode OZK_ACC_FIXED, rho from K).
 * It has no counterpart in the reference.  For callers that must not allocate
 * device memory during a call (a process whose framework owns the GPU's memory,
 * such as JAX/XLA reserving most of it for its own allocator, or a plugin
 * callback its host forbids from allocating): the slice workspace comes from a
 * fixed device array of OZK_NOALLOC_SCRATCH_BYTES compiled into the library,
 * held by every GPU that loads it until exit.  The bound is the slices-only
 * workspace (not ozk_matmul_workspace_bytes, which adds the GEMM state scratch
 * of about 38 MB): with nS = n_hi + n_lo and k_pad = K rounded up to 64,
 *   align256(2 nS N k_pad) + align256(2 nS M k_pad) + align256(4 nS N)
 *   + align256(4 nS M) + align256(8 K M) + 256 <= OZK_NOALLOC_SCRATCH_BYTES,
 * else OZK_ERR_WORKSPACE; 1024 x 1024 x 1024 at (4, 1) fits.  Without the
 * state scratch the slice GEMM runs its 128-wide BF16 tiles (running sums in
 * TMEM; at most 16 columns use the int8 skinny kernel); the sums are exact,
 * so C is bit-identical to ozk_matmul_f64 with OZK_ACC_FIXED.  Each call looks
 * up the array's address in the current context (cudaGetSymbolAddress); the
 * first call in a context also loads the module and should come before any
 * stream capture.  All calls share the array; calls that overlap on the GPU
 * race on it and must be serialised by the caller.  No cudaMalloc/cudaFree
 * (OZK_GEMM_STATS diagnostics record nothing for these calls). */
#define OZK_NOALLOC_SCRATCH_BYTES (32 * 1024 * 1024)
int ozk_matmul_f64_noalloc(const double* A, int64_t lda, const double* B, int64_t ldb, double* C,
                           int64_t ldc, int64_t N, int64_t K, int64_t M, int n_hi, int n_lo,
                           int32_t* status_dev, void* stream);

/* ---------------------------------------------------------------- multi-GPU */

/* A set of GPUs that compute one product together (no counterpart in the
 * reference, which has no multi-device code; this partitions the on-device
 * operators _fully_fused_f64_jit / _bf16_interleaved_f64_jit,
 * ozaki_jax/matmul.py:514-540, across the GPUs of one node).  It holds one
 * NCCL communicator per local GPU and per-GPU workspaces grown on demand;
 * NCCL (libnccl.so.2) is loaded at run time.  Two ways to make one:
 *   - one process per GPU: every rank calls ozk_context_create_rank with the
 *     same OZK_NCCL_ID_BYTES id, made by ozk_nccl_unique_id on one rank and
 *     passed to the others by the caller (an MPI broadcast, a torch.distributed
 *     store, a file, ...);
 *   - one process driving several GPUs (the JAX model): ozk_context_create_local
 *     with the device list; global rank i is devices[i]. */
#define OZK_NCCL_ID_BYTES 128
typedef struct ozk_context ozk_context;
int ozk_nccl_unique_id(void* id_out, size_t len);
int ozk_context_create_rank(ozk_context** ctx, int nranks, int rank, const void* nccl_id,
                            size_t id_len, int device);
int ozk_context_create_local(ozk_context** ctx, int ndev, const int* devices);
int ozk_context_destroy(ozk_context* ctx);
/* Global rank count, the global rank of the first local GPU, local GPU count. */
int ozk_context_info(const ozk_context* ctx, int* nranks, int* first_rank, int* nlocal);
/* Waits for the work that OZK_MULTI_NOWAIT calls enqueued on streams[i] (one
 * per local GPU, NULL: the legacy default streams) with the bound of the
 * blocking calls: NCCL's asynchronous errors are watched, and after
 * OZK_NCCL_TIMEOUT_MS (default 300 s) or an NCCL failure the communicators are
 * aborted, the context becomes unusable and OZK_ERR_TIMEOUT / OZK_ERR_NCCL is
 * returned.  A rank whose peer failed (or never made its call) therefore gets
 * an error instead of waiting forever, as a plain stream synchronisation
 * would. */
int ozk_context_wait(ozk_context* ctx, void* const* streams);

/* How B reaches every rank in ozk_matmul_f64_multi. */
#define OZK_B_REPLICATED 0 /* every rank holds all of B (K x M) and extracts it */
#define OZK_B_ROOT 1       /* rank 0 holds B; its slices are broadcast over NCCL */
#define OZK_B_COLUMNS 2    /* rank r holds columns [r mc, min(M, (r+1) mc)) of B,
                              mc = ceil(M / P), as a K x m_r matrix; slices all-gathered */
/* Flags of ozk_matmul_f64_multi. */
#define OZK_MULTI_NOWAIT 0x1 /* do not wait for the result (see below) */
#define OZK_MULTI_BF16 0x2   /* BF16 slices even where int8 codes are exact */
/* Status bit: the int8 pass of a NOWAIT call found a slice without an exact
 * int8 code on some rank, so C was not written; repeat the call with
 * OZK_MULTI_BF16 (every rank sees this bit, so all repeat together). */
#define OZK_FLAG_REDO 0x8

/* C = A @ B row-sharded over the context's P global ranks (matmul(...,
 * pipeline='ondevice', accumulation='fused') on the whole A): global rank r
 * holds rows [r N / P, (r+1) N / P) of A (lda) and of C (ldc).  Arrays are
 * indexed by local GPU (ozk_context_info's nlocal entries): A[i], B[i], C[i]
 * are device pointers on that GPU, streams[i] its stream (NULL array: the
 * legacy default streams), status_dev[i] a device word receiving the OZK_FLAG_*
 * bits of ALL ranks (NULL array or entry: not reported).  Each rank's rows of
 * C are bit-identical to the same rows of ozk_matmul_f64 with OZK_ACC_FIXED.
 * All ranks must make the same calls in the same order, on the same streams
 * from one call to the next (the workspace is reused).  Without
 * OZK_MULTI_NOWAIT the call waits for the result (watching NCCL; after
 * OZK_NCCL_TIMEOUT_MS, default 300 s, or an NCCL failure the communicators are
 * aborted and the context is unusable) and runs a BF16 pass itself if an
 * int8 code failed; with it, the call returns once everything is enqueued. */
int ozk_matmul_f64_multi(ozk_context* ctx, const double* const* A, const int64_t* lda,
                         const double* const* B, const int64_t* ldb, double* const* C,
                         const int64_t* ldc, int64_t N, int64_t K, int64_t M, int n_hi, int n_lo,
                         int b_mode, int flags, void* const* streams, int32_t* const* status_dev);

/* G = A^T A with A's rows sharded over the context's P ranks (gram(mode='ozaki')
 * on the whole A, _gram_ozaki_jit, ozaki_jax/gram.py:19-37, with the rows
 * split as BASELINE's multi-GPU gram asks: partial Gram blocks reduced).
 * Global rank r holds rows [r N / P, (r+1) N / P) of A (lda); every rank
 * receives all of G (K x K, ldg).  The lines of the gram are A's columns, split
 * by rows over the ranks: each slice pass takes the lines' maxima over all
 * ranks (an NCCL all-reduce of 2 K floats), so every rank's int8 codes are the
 * single-GPU codes of its rows; each rank's symmetric int8 GEMM writes its raw
 * int64 fixed-point sums, the sums are all-reduced exactly (NCCL int64 sum),
 * and one kernel rounds them to FP64 and mirrors them.  Per-pair terms are
 * rounded at 2^-36 of the top grid on each rank's partial products, so G can
 * differ from ozk_gram_f64 in the last bit of rare elements (it is identical
 * with one rank).  Int8 codes only (rho >= 19, N > 4096; K >= 256; at most
 * 65536 rows per rank), else OZK_ERR_UNSUPPORTED.  If some code has no exact
 * int8 value on any rank, G is not written and every rank's status gets
 * OZK_FLAG_REDO.  flags: OZK_MULTI_NOWAIT as for ozk_matmul_f64_multi. */
int ozk_gram_f64_multi(ozk_context* ctx, const double* const* A, const int64_t* lda,
                       double* const* G, const int64_t* ldg, int64_t N, int64_t K, int n_hi,
                       int n_lo, int flags, void* const* streams, int32_t* const* status_dev);

/* The FP64 host pipeline (matmul(pipeline='host'), ozaki_jax/matmul.py:823-851):
 * FP64 extraction into n_slices slices, triangular pairs, FP64 accumulation,
 * all on the device.  rho < 0 selects _compute_rho(K). */
size_t ozk_matmul_host_workspace_bytes(int64_t N, int64_t K, int64_t M, int n_slices);
int ozk_matmul_host_f64(const double* A, int64_t lda, const double* B, int64_t ldb, double* C,
                        int64_t ldc, int64_t N, int64_t K, int64_t M, int rho, int n_slices,
                        void* workspace, size_t ws_bytes, int32_t* status_dev, void* stream);

/* gram(mode='ozaki') (_gram_ozaki_jit, ozaki_jax/gram.py:19-37): G = A^T A for
 * A (N x K, lda), G (K x K, ldg), rho < 0 selects _compute_rho_f32(N).  The
 * slices of A are extracted once and serve both operands. */
size_t ozk_gram_workspace_bytes(int64_t N, int64_t K, int n_hi, int n_lo);
int ozk_gram_f64(const double* A, int64_t lda, double* G, int64_t ldg, int64_t N, int64_t K,
                 int rho, int n_hi, int n_lo, void* workspace, size_t ws_bytes,
                 int32_t* status_dev, void* stream);

/* residual(mode='ozaki') (_residual_ozaki_jit / _ozaki_matvec_f64,
 * ozaki_jax/solve.py:38-53, :78-82): R = Bv - A @ X for A (N x K), X (K x M),
 * Bv and R (N x M).  rho < 0 selects _compute_rho_f32(K). */
size_t ozk_residual_workspace_bytes(int64_t N, int64_t K, int64_t M, int n_hi, int n_lo);
int ozk_residual_f64(const double* A, int64_t lda, const double* X, int64_t ldx,
                     const double* Bv, int64_t ldb, double* R, int64_t ldr, int64_t N,
                     int64_t K, int64_t M, int rho, int n_hi, int n_lo, void* workspace,
                     size_t ws_bytes, int32_t* status_dev, void* stream);

/* ---------------------------------------------------------------- status */

/* Synchronises `stream`, reads *status_dev (device) and returns OZK_OK,
 * OZK_ERR_NONFINITE or OZK_ERR_TIMEOUT (timeout wins), or OZK_ERR_CUDA. */
int ozk_check_status(const int32_t* status_dev, void* stream);
/* Static text for a status code. */
const char* ozk_strerror(int status);
/* Copies the last error detail of the calling host thread into buf. */
int ozk_last_error_detail(char* buf, size_t len);
/* Diagnostics (no counterpart in the reference): with OZK_GEMM_STATS=1 in
 * the environment, sums over the CTAs of the last slice-GEMM launch of
 * {0: MMA-thread cycles waiting for a free accumulator, 1: MMA-thread cycles
 * waiting for loaded stages, 2: producer cycles waiting for free stages,
 * 3: MMA-thread total cycles, 4: epilogue cycles waiting for a finished
 * accumulator, 5: epilogue cycles processing, 6: epilogue pairs, 7: the part
 * of 1 spent in the first pipeline-depth k-blocks of each pair}
 * (epilogue figures from one warp per CTA); returns the CTA count
 * (synchronises the device).  The counters are allocated on the first
 * recorded launch; launches without the GEMM state scratch record none. */
int ozk_gemm_stats(unsigned long long* out8);
/* Failure-path self-test (no counterpart in the reference): one CTA waits on an
 * mbarrier nothing arrives at, through the bounded wait all kernels use; after
 * budget_ms the wait gives up, writes 0 to *ok_dev and raises
 * OZK_FLAG_TIMEOUT in *status_dev.  No fault, no hang. */
int ozk_selftest_timeout(int budget_ms, int32_t* status_dev, int32_t* ok_dev, void* stream);
/* L2 residency of the slice GEMM's running sums (no counterpart in the
 * reference).  The 256-wide GEMM tiles keep per-CTA running sums in a global
 * scratch (ozk_slice_gemm_workspace_bytes, about 38 MB) that it re-reads every
 * pair, and it marks those accesses evict_last, a priority that takes effect
 * inside the context's persisting-L2 set-aside.  The library does not change
 * that limit by default (the context's own set-aside, 23.7 MB on B200, keeps
 * the GEMM within 2.5% of one that holds all the sums).  Opt-ins:
 * OZK_L2_PERSIST=sticky in the environment raises it once per device to hold
 * the sums, OZK_L2_PERSIST=<MB> to that size; or this call sets it
 * explicitly: `bytes` (clamped to the device maximum; 0 turns it off;
 * (size_t)-1 only queries), the value in force before goes to *previous (may
 * be NULL).  The limit belongs to this process's CUDA context and ends with
 * it; lines not marked persisting may use the set-aside while no persisting
 * data holds it. */
int ozk_set_l2_persisting(size_t bytes, size_t* previous);
/* Library version string. */
const char* ozk_version(void);

#ifdef __cplusplus
}
#endif
#endif /* OZAKI_B200_H */
