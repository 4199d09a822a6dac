// extern "C" entry points of libozaki_b200.so (declared in ozaki_b200.h):
// argument validation, the reference's policies (rho, presets, pair
// schedules, preflight bounds), workspace layout and kernel sequencing.
#include <cuda_runtime.h>
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "ozaki_b200.h"
#include "ozk_internal.h"

namespace ozk {

static thread_local char t_detail[512] = "";

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_detail, sizeof(t_detail), fmt, ap);
  va_end(ap);
  return code;
}

int set_cuda_error(const char* what, cudaError_t e) {
  return set_error(OZK_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

int device_sm_count(int dev) {
  static int cache[64] = {0};
  if (dev < 0 || dev >= 64) return 148;
  if (!cache[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

// Time budget of every device-side wait (default 2 s; OZK_WAIT_BUDGET_MS
// overrides it).  A legitimate wait lasts microseconds.
uint64_t wait_budget_ns() {
  static uint64_t v = 0;
  if (!v) {
    const char* s = getenv("OZK_WAIT_BUDGET_MS");
    long ms = s ? atol(s) : 0;
    v = (uint64_t)(ms > 0 ? ms : 2000) * 1000000ull;
  }
  return v;
}

static int rho_f32(int64_t K) {  // extract.py:109-113
  int64_t k = K < 2 ? 2 : K;
  int lg = 0;
  while (((int64_t)1 << lg) < k) ++lg;  // ceil(log2 k)
  int gamma = (int)ceil(24.0 - (24.0 - lg) / 2.0);
  return gamma > 17 ? gamma : 17;
}

static int rho_f64(int64_t K) {  // extract.py:12-18
  int64_t k = K < 2 ? 2 : K;
  int lg = 0;
  while (((int64_t)1 << lg) < k) ++lg;
  int gamma = (int)ceil(53.0 - (24.0 - lg) / 2.0);
  return gamma > 46 ? gamma : 46;
}

// BF16 -> FP32 exact inner-product bound K * (2^bits - 1)^2 < 2^24
// (matmul.py:605-621 and :84-97).
int check_bound(int64_t K, int bits) {
  if (bits <= 0)
    return set_error(OZK_ERR_UNSAFE, "non-positive bits per slice (%d); K=%lld is too large", bits,
                     (long long)K);
  double m = (double)(((int64_t)1 << bits) - 1);
  if ((double)K * m * m >= 16777216.0)
    return set_error(OZK_ERR_UNSAFE, "K=%lld violates BF16->FP32 exact inner-product bound",
                     (long long)K);
  return OZK_OK;
}

static int ondevice_pairs(int n_hi, int n_lo, uint8_t* pa, uint8_t* pb, int cap) {
  if (n_hi < 1 || n_lo < 0 || n_hi > OZK_MAX_SIDE || n_lo > OZK_MAX_SIDE)
    return set_error(OZK_ERR_ARG, "n_hi must be in [1,%d] and n_lo in [0,%d]", OZK_MAX_SIDE,
                     OZK_MAX_SIDE);
  int n = n_hi * n_hi + 2 * n_hi * n_lo;
  if (n > cap) return set_error(OZK_ERR_ARG, "pair capacity too small");
  int k = 0;
  for (int i = 0; i < n_hi; ++i)
    for (int j = 0; j < n_hi; ++j) pa[k] = i, pb[k++] = j;
  for (int i = 0; i < n_hi; ++i)
    for (int j = 0; j < n_lo; ++j) pa[k] = i, pb[k++] = n_hi + j;
  for (int i = 0; i < n_lo; ++i)
    for (int j = 0; j < n_hi; ++j) pa[k] = n_hi + i, pb[k++] = j;
  return n;
}

// Pair order for order-independent (fixed-point) sums: the same pairs as
// ondevice_pairs, arranged so consecutive pairs share an operand slice (the
// hi x hi block row by row in alternating direction, then hi x lo walking back
// over the A slices, then lo x hi), which keeps one operand panel hot in L2
// at every pair boundary.
static int snake_pairs(int n_hi, int n_lo, uint8_t* pa, uint8_t* pb, int cap) {
  int n = ondevice_pairs(n_hi, n_lo, pa, pb, cap);
  if (n < 0) return n;
  int k = 0;
  int last_i = 0;
  for (int i = 0; i < n_hi; ++i) {
    for (int jj = 0; jj < n_hi; ++jj) {
      const int j = (i % 2 == 0) ? jj : n_hi - 1 - jj;
      pa[k] = (uint8_t)i, pb[k++] = (uint8_t)j;
    }
    last_i = i;
  }
  for (int j = 0; j < n_lo; ++j)
    for (int ii = 0; ii < n_hi; ++ii) {
      const int i = ((j % 2 == 0) == (last_i == n_hi - 1)) ? n_hi - 1 - ii : ii;
      pa[k] = (uint8_t)i, pb[k++] = (uint8_t)(n_hi + j);
    }
  for (int i = 0; i < n_lo; ++i)
    for (int jj = 0; jj < n_hi; ++jj) {
      const int j = (i % 2 == 0) ? jj : n_hi - 1 - jj;
      pa[k] = (uint8_t)(n_hi + i), pb[k++] = (uint8_t)j;
    }
  return k == n ? n : set_error(OZK_ERR_ARG, "pair schedule mismatch");
}

struct Workspace {
  uint16_t* SA;
  uint16_t* SB;
  int32_t* eA;
  int32_t* eB;
  double* BT;  // transposed FP64 copy of the column-extracted operand
  float* products;
  double* state;  // per-CTA FP64 running sums of the 256-wide GEMM tiles
  size_t state_bytes;
  int32_t* gate;  // set when an int8 slice code failed: the BF16 recomputation runs
  size_t bytes;
};

static size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

// Layout: SA [nS][N][k_pad] | SB [nS][M][k_pad] | eA [nS][N] | eB [nS][M] |
// BT [bt_elems] FP64 | products [n_pairs][N][M] (only when materialised) |
// state [state_bytes] (optional GEMM scratch) | gate word.  The slice areas
// are sized for BF16; int8 codes use the first half of each.
static Workspace layout(void* base, int64_t N, int64_t K, int64_t M, int nS, int n_prod,
                        int64_t bt_elems, size_t state_bytes = 0) {
  const int64_t k_pad = round_up(K < 1 ? 1 : K, OZK_KB);
  Workspace w;
  size_t off = 0;
  char* b = (char*)base;
  w.SA = (uint16_t*)(b + off);
  off += align256((size_t)nS * N * k_pad * 2);
  w.SB = (uint16_t*)(b + off);
  off += align256((size_t)nS * M * k_pad * 2);
  w.eA = (int32_t*)(b + off);
  off += align256((size_t)nS * N * 4);
  w.eB = (int32_t*)(b + off);
  off += align256((size_t)nS * M * 4);
  w.BT = (double*)(b + off);
  off += align256((size_t)bt_elems * 8);
  w.products = (float*)(b + off);
  off += align256((size_t)n_prod * N * M * 4);
  w.state = state_bytes ? (double*)(b + off) : nullptr;
  w.state_bytes = state_bytes;
  off += align256(state_bytes);
  w.gate = (int32_t*)(b + off);
  off += 256;
  w.bytes = off;
  return w;
}

// Scoped workspace: the caller's buffer, or one from the stream-ordered pool.
struct ScopedWs {
  void* ptr = nullptr;
  bool owned = false;
  cudaStream_t s = nullptr;
  int acquire(void* given, size_t given_bytes, size_t need, cudaStream_t stream) {
    s = stream;
    if (given) {
      if (given_bytes < need)
        return set_error(OZK_ERR_WORKSPACE, "workspace %zu bytes < %zu needed", given_bytes, need);
      if ((uintptr_t)given & 255) return set_error(OZK_ERR_ARG, "workspace not 256-byte aligned");
      ptr = given;
      return OZK_OK;
    }
    cudaError_t e = cudaMallocAsync(&ptr, need, stream);
    if (e != cudaSuccess) return set_cuda_error("cudaMallocAsync(workspace)", e);
    owned = true;
    return OZK_OK;
  }
  ~ScopedWs() {
    if (owned && ptr) cudaFreeAsync(ptr, s);
  }
};

static size_t cur_state_bytes() {
  int dev = 0;
  cudaGetDevice(&dev);
  return gemm_state_bytes(dev);
}

// Workspace actually usable: the full size when given (or pool-allocated),
// else the minimum without the GEMM state scratch.
static int pick_workspace(void* given, size_t given_bytes, size_t full, size_t minimum,
                          bool& with_state) {
  with_state = true;
  if (!given) return OZK_OK;
  if (given_bytes >= full) return OZK_OK;
  with_state = false;
  if (given_bytes >= minimum) return OZK_OK;
  return set_error(OZK_ERR_WORKSPACE, "workspace %zu bytes < %zu needed", given_bytes, minimum);
}

size_t matmul_min_workspace_bytes(int64_t N, int64_t K, int64_t M, int n_hi, int n_lo) {
  return layout(nullptr, N, K, M, n_hi + n_lo, 0, M * K).bytes;
}

// int8 slices for fixed-point sums where eligible (OZK_S8=0 in the
// environment turns them off, for comparisons).
bool s8_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("OZK_S8");
    v = (e && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

// C = A B with fixed-point sums.  Where the int8 GEMM applies, the slices are
// extracted as int8 codes and multiplied with kind::i8 MMAs; the BF16
// extraction and GEMM are enqueued behind them gated on w.gate, so they run
// (and overwrite the result) only if some slice had no exact int8 code.  The
// stream never waits on the host for that decision.
// C = alpha (A B) + beta Cin for at most 16 columns of B, with int8 codes and
// the skinny all-pairs GEMM (each A slice read once), and the gated BF16
// recomputation behind it.  Returns 1 when the request does not qualify.
static int skinny_fixed(const double* A, int64_t lda, const double* B, int64_t ldb, double alpha,
                        double beta, const double* Cin, int64_t ldcin, double* C, int64_t ldc,
                        int64_t N, int64_t K, int64_t M, int rho, int n_hi, int n_lo,
                        const uint8_t* pa, const uint8_t* pb, int np, const Workspace& w,
                        int32_t* status_dev, cudaStream_t s) {
  const int nS = n_hi + n_lo;
  const int64_t k_pad = round_up(K, OZK_KB);
  const int64_t k8 = round_up(K, kS8KB);
  if (!skinny_s8_eligible(N, M, k8, nS, np, rho)) return 1;
  int rc;
  cudaError_t e = cudaMemsetAsync(w.gate, 0, sizeof(int32_t), s);
  if (e != cudaSuccess) return set_cuda_error("cudaMemsetAsync(gate)", e);
  if ((rc = launch_extract_rows_s8(A, lda, N, K, rho, n_hi, n_lo, (int8_t*)w.SA, k8, w.eA,
                                   status_dev, w.gate, s)))
    return rc;
  if ((rc = launch_extract_cols_s8(B, ldb, K, M, rho, n_hi, n_lo, (int8_t*)w.SB, k8, w.eB,
                                   status_dev, w.gate, w.BT, s)))
    return rc;
  if ((rc = launch_skinny_s8((const int8_t*)w.SA, w.eA, (const int8_t*)w.SB, w.eB, nS, N, M, k8,
                             pa, pb, np, alpha, beta, Cin, ldcin, C, ldc, rho, status_dev, w.gate,
                             0, w.state, w.state_bytes, s)))
    return rc;
  if ((rc = launch_extract_rows_gated(A, lda, N, K, rho, n_hi, n_lo, w.SA, k_pad, w.eA, status_dev,
                                      w.gate, s)))
    return rc;
  if ((rc = launch_extract_rows_gated(w.BT, K, M, K, rho, n_hi, n_lo, w.SB, k_pad, w.eB,
                                      status_dev, w.gate, s)))
    return rc;
  return launch_slice_gemm_ex(w.SA, w.eA, nS, w.SB, w.eB, nS, N, M, k_pad, pa, pb, np,
                              OZK_ACC_FIXED, 0, alpha, beta, Cin, ldcin, C, ldc, nullptr, w.state,
                              w.state_bytes, rho, status_dev, false, w.gate, 1, s);
}

static int matmul_fixed(const double* A, int64_t lda, const double* B, int64_t ldb, double* C,
                        int64_t ldc, int64_t N, int64_t K, int64_t M, int rho, int n_hi, int n_lo,
                        const uint8_t* pa, const uint8_t* pb, int np, const Workspace& w,
                        int32_t* status_dev, cudaStream_t s) {
  const int nS = n_hi + n_lo;
  const int64_t k_pad = round_up(K, OZK_KB);
  const int64_t k8 = round_up(K, kS8KB);
  int rc;
  if (s8_enabled() && M <= 16) {
    rc = skinny_fixed(A, lda, B, ldb, 1.0, 0.0, nullptr, 0, C, ldc, N, K, M, rho, n_hi, n_lo, pa,
                      pb, np, w, status_dev, s);
    if (rc != 1) return rc;
  }
  if (!s8_enabled() || !slice_gemm_s8_eligible(N, M, k8, OZK_ACC_FIXED, rho, w.state_bytes)) {
    if ((rc = launch_extract_rows(A, lda, N, K, rho, n_hi, n_lo, w.SA, k_pad, w.eA, status_dev, s)))
      return rc;
    if ((rc = launch_extract_cols(B, ldb, K, M, rho, n_hi, n_lo, w.SB, k_pad, w.eB, status_dev,
                                  w.BT, s)))
      return rc;
    return launch_slice_gemm(w.SA, w.eA, nS, w.SB, w.eB, nS, N, M, k_pad, pa, pb, np,
                             OZK_ACC_FIXED, 0, 1.0, 0.0, nullptr, 0, C, ldc, nullptr, w.state,
                             w.state_bytes, rho, status_dev, s);
  }
  cudaError_t e = cudaMemsetAsync(w.gate, 0, sizeof(int32_t), s);
  if (e != cudaSuccess) return set_cuda_error("cudaMemsetAsync(gate)", e);
  if ((rc = launch_extract_rows_s8(A, lda, N, K, rho, n_hi, n_lo, (int8_t*)w.SA, k8, w.eA,
                                   status_dev, w.gate, s)))
    return rc;
  if ((rc = launch_extract_cols_s8(B, ldb, K, M, rho, n_hi, n_lo, (int8_t*)w.SB, k8, w.eB,
                                   status_dev, w.gate, w.BT, s)))
    return rc;
  if ((rc = launch_slice_gemm_ex(w.SA, w.eA, nS, w.SB, w.eB, nS, N, M, k8, pa, pb, np,
                                 OZK_ACC_FIXED, 0, 1.0, 0.0, nullptr, 0, C, ldc, nullptr, w.state,
                                 w.state_bytes, rho, status_dev, true, w.gate, 0, s)))
    return rc;
  // BF16 recomputation (B from its transposed copy), only if the gate is set.
  if ((rc = launch_extract_rows_gated(A, lda, N, K, rho, n_hi, n_lo, w.SA, k_pad, w.eA, status_dev,
                                      w.gate, s)))
    return rc;
  if ((rc = launch_extract_rows_gated(w.BT, K, M, K, rho, n_hi, n_lo, w.SB, k_pad, w.eB,
                                      status_dev, w.gate, s)))
    return rc;
  return launch_slice_gemm_ex(w.SA, w.eA, nS, w.SB, w.eB, nS, N, M, k_pad, pa, pb, np,
                              OZK_ACC_FIXED, 0, 1.0, 0.0, nullptr, 0, C, ldc, nullptr, w.state,
                              w.state_bytes, rho, status_dev, false, w.gate, 1, s);
}

}  // namespace ozk

using namespace ozk;

extern "C" {

int ozk_compute_rho_f32(int64_t K) { return rho_f32(K); }
int ozk_compute_rho_f64(int64_t K) { return rho_f64(K); }

int ozk_pair_schedule(int n_hi, int n_lo, uint8_t* pair_a, uint8_t* pair_b, int cap) {
  if (!pair_a || !pair_b) return set_error(OZK_ERR_ARG, "NULL pair arrays");
  return ondevice_pairs(n_hi, n_lo, pair_a, pair_b, cap);
}

int ozk_pair_schedule_snake(int n_hi, int n_lo, uint8_t* pair_a, uint8_t* pair_b, int cap) {
  if (!pair_a || !pair_b) return set_error(OZK_ERR_ARG, "NULL pair arrays");
  return snake_pairs(n_hi, n_lo, pair_a, pair_b, cap);
}

int ozk_triangular_schedule(int n_slices, uint8_t* pair_a, uint8_t* pair_b, int cap) {
  if (!pair_a || !pair_b || n_slices < 1 || n_slices > OZK_MAX_SLICES)
    return set_error(OZK_ERR_ARG, "n_slices out of range");
  int k = 0;
  for (int i = 0; i < n_slices; ++i)
    for (int j = 0; j < n_slices; ++j)
      if (i + j <= n_slices - 1) {
        if (k >= cap) return set_error(OZK_ERR_ARG, "pair capacity too small");
        pair_a[k] = (uint8_t)i;
        pair_b[k++] = (uint8_t)j;
      }
  return k;
}

static int check_extract_args(const void* X, int64_t ldx, int64_t lines, int64_t K, int64_t ld_min,
                              int n_hi, int n_lo, const void* slices, int64_t k_pad,
                              const void* exps) {
  if (!X || !slices || !exps) return set_error(OZK_ERR_ARG, "NULL pointer");
  if (lines < 0 || K < 1) return set_error(OZK_ERR_ARG, "bad shape");
  if (ldx < ld_min) return set_error(OZK_ERR_ARG, "leading dimension too small");
  if (n_hi < 1 || n_hi > OZK_MAX_SIDE || n_lo < 0 || n_lo > OZK_MAX_SIDE)
    return set_error(OZK_ERR_ARG, "slice counts out of range");
  if (k_pad < K || k_pad % OZK_KB) return set_error(OZK_ERR_ARG, "k_pad must be >= K and a multiple of 64");
  if (((uintptr_t)slices & 3) != 0) return set_error(OZK_ERR_ARG, "slices not 4-byte aligned");
  return OZK_OK;
}

int ozk_extract_rows_f64(const double* X, int64_t ldx, int64_t rows, int64_t K, int rho, int n_hi,
                         int n_lo, uint16_t* slices, int64_t k_pad, int32_t* exps,
                         int32_t* status_dev, void* stream) {
  int rc = check_extract_args(X, ldx, rows, K, K, n_hi, n_lo, slices, k_pad, exps);
  if (rc) return rc;
  if (rho < 0) rho = rho_f32(K);
  return launch_extract_rows(X, ldx, rows, K, rho, n_hi, n_lo, slices, k_pad, exps, status_dev,
                             (cudaStream_t)stream);
}

int ozk_extract_cols_f64(const double* X, int64_t ldx, int64_t K, int64_t cols, int rho, int n_hi,
                         int n_lo, uint16_t* slices, int64_t k_pad, int32_t* exps, double* scratch,
                         size_t scratch_bytes, int32_t* status_dev, void* stream) {
  int rc = check_extract_args(X, ldx, cols, K, cols, n_hi, n_lo, slices, k_pad, exps);
  if (rc) return rc;
  if (rho < 0) rho = rho_f32(K);
  const size_t need = (size_t)cols * K * 8;
  if (scratch && scratch_bytes < need)
    return set_error(OZK_ERR_WORKSPACE, "scratch %zu bytes < %zu needed", scratch_bytes, need);
  // The transposed fast path needs a cols x K FP64 scratch (caller's or pool).
  ScopedWs ws;
  if (!scratch && k_pad <= 65536 && cols > 0 &&
      ws.acquire(nullptr, 0, need, (cudaStream_t)stream) == OZK_OK)
    scratch = (double*)ws.ptr;
  return launch_extract_cols(X, ldx, K, cols, rho, n_hi, n_lo, slices, k_pad, exps, status_dev,
                             scratch, (cudaStream_t)stream);
}

int ozk_extract_rows_host_f64(const double* X, int64_t ldx, int64_t rows, int64_t K, int rho,
                              int n_slices, uint16_t* slices, int64_t k_pad, int32_t* exps,
                              int32_t* status_dev, void* stream) {
  if (n_slices < 1 || n_slices > OZK_MAX_SLICES)
    return set_error(OZK_ERR_ARG, "n_slices must be in [1,%d]", OZK_MAX_SLICES);
  int rc = check_extract_args(X, ldx, rows, K, K, 1, 0, slices, k_pad, exps);
  if (rc) return rc;
  if (rho < 0) rho = rho_f64(K);
  return launch_extract_rows64(X, ldx, rows, K, rho, n_slices, slices, k_pad, exps, status_dev,
                               (cudaStream_t)stream);
}

int ozk_extract_cols_host_f64(const double* X, int64_t ldx, int64_t K, int64_t cols, int rho,
                              int n_slices, uint16_t* slices, int64_t k_pad, int32_t* exps,
                              int32_t* status_dev, void* stream) {
  if (n_slices < 1 || n_slices > OZK_MAX_SLICES)
    return set_error(OZK_ERR_ARG, "n_slices must be in [1,%d]", OZK_MAX_SLICES);
  int rc = check_extract_args(X, ldx, cols, K, cols, 1, 0, slices, k_pad, exps);
  if (rc) return rc;
  if (rho < 0) rho = rho_f64(K);
  return launch_extract_cols64(X, ldx, K, cols, rho, n_slices, slices, k_pad, exps, status_dev,
                               (cudaStream_t)stream);
}

int ozk_slice_gemm(const uint16_t* SA, const int32_t* eA, int nA, const uint16_t* SB,
                   const int32_t* eB, int nB, int64_t N, int64_t M, int64_t k_pad,
                   const uint8_t* pair_a, const uint8_t* pair_b, int n_pairs, int mode,
                   int symmetric, double alpha, double beta, const double* Cin, int64_t ldcin,
                   double* C, int64_t ldc, float* products, void* workspace, size_t ws_bytes,
                   int rho, int32_t* status_dev, void* stream) {
  if (!SA || !SB || !eA || !eB || !pair_a || !pair_b) return set_error(OZK_ERR_ARG, "NULL pointer");
  if (N < 0 || M < 0) return set_error(OZK_ERR_ARG, "bad shape");
  if (mode != OZK_ACC_PRODUCTS && ldc < M) return set_error(OZK_ERR_ARG, "ldc < M");
  if (beta != 0.0 && ldcin < M) return set_error(OZK_ERR_ARG, "ldcin < M");
  if (alpha != 1.0 && alpha != -1.0) return set_error(OZK_ERR_ARG, "alpha must be +1 or -1");
  if (workspace && ((uintptr_t)workspace & 255))
    return set_error(OZK_ERR_ARG, "workspace not 256-byte aligned");
  return launch_slice_gemm(SA, eA, nA, SB, eB, nB, N, M, k_pad, pair_a, pair_b, n_pairs, mode,
                           symmetric, alpha, beta, Cin, ldcin, C, ldc, products, (double*)workspace,
                           workspace ? ws_bytes : 0, rho, status_dev, (cudaStream_t)stream);
}

size_t ozk_slice_gemm_workspace_bytes(void) { return cur_state_bytes(); }

static int check_s8_extract(int rho, int64_t k_pad, const int32_t* fail_dev) {
  if (!fail_dev) return set_error(OZK_ERR_ARG, "fail_dev is NULL");
  if (rho < kS8MinRho)
    return set_error(OZK_ERR_UNSUPPORTED, "int8 slice codes need rho >= %d (got %d)", kS8MinRho, rho);
  if (k_pad % kS8KB || k_pad > 65536)
    return set_error(OZK_ERR_ARG, "k_pad must be a multiple of %d, at most 65536", kS8KB);
  return OZK_OK;
}

int ozk_extract_rows_s8_f64(const double* X, int64_t ldx, int64_t rows, int64_t K, int rho,
                            int n_hi, int n_lo, int8_t* slices, int64_t k_pad, int32_t* exps,
                            int32_t* fail_dev, int32_t* status_dev, void* stream) {
  int rc = check_extract_args(X, ldx, rows, K, K, n_hi, n_lo, slices, k_pad, exps);
  if (rc) return rc;
  if (rho < 0) rho = rho_f32(K);
  if ((rc = check_s8_extract(rho, k_pad, fail_dev))) return rc;
  return launch_extract_rows_s8(X, ldx, rows, K, rho, n_hi, n_lo, slices, k_pad, exps, status_dev,
                                fail_dev, (cudaStream_t)stream);
}

int ozk_extract_cols_s8_f64(const double* X, int64_t ldx, int64_t K, int64_t cols, int rho,
                            int n_hi, int n_lo, int8_t* slices, int64_t k_pad, int32_t* exps,
                            double* scratch, size_t scratch_bytes, int32_t* fail_dev,
                            int32_t* status_dev, void* stream) {
  int rc = check_extract_args(X, ldx, cols, K, cols, n_hi, n_lo, slices, k_pad, exps);
  if (rc) return rc;
  if (rho < 0) rho = rho_f32(K);
  if ((rc = check_s8_extract(rho, k_pad, fail_dev))) return rc;
  const size_t need = (size_t)cols * K * 8;
  if (scratch && scratch_bytes < need)
    return set_error(OZK_ERR_WORKSPACE, "scratch %zu bytes < %zu needed", scratch_bytes, need);
  ScopedWs ws;
  if (!scratch && cols > 0) {
    if ((rc = ws.acquire(nullptr, 0, need, (cudaStream_t)stream))) return rc;
    scratch = (double*)ws.ptr;
  }
  return launch_extract_cols_s8(X, ldx, K, cols, rho, n_hi, n_lo, slices, k_pad, exps, status_dev,
                                fail_dev, scratch, (cudaStream_t)stream);
}

int ozk_slice_gemm_s8(const int8_t* SA, const int32_t* eA, int nA, const int8_t* SB,
                      const int32_t* eB, int nB, int64_t N, int64_t M, int64_t k_pad,
                      const uint8_t* pair_a, const uint8_t* pair_b, int n_pairs, int symmetric,
                      double alpha, double beta, const double* Cin, int64_t ldcin, double* C,
                      int64_t ldc, void* workspace, size_t ws_bytes, int rho,
                      const int32_t* skip_if_dev, int32_t* status_dev, void* stream) {
  if (!SA || !SB || !eA || !eB || !pair_a || !pair_b || !C)
    return set_error(OZK_ERR_ARG, "NULL pointer");
  if (N < 0 || M < 0) return set_error(OZK_ERR_ARG, "bad shape");
  if (ldc < M) return set_error(OZK_ERR_ARG, "ldc < M");
  if (beta != 0.0 && (!Cin || ldcin < M)) return set_error(OZK_ERR_ARG, "bad Cin");
  if (alpha != 1.0 && alpha != -1.0) return set_error(OZK_ERR_ARG, "alpha must be +1 or -1");
  if (!workspace || ((uintptr_t)workspace & 255))
    return set_error(OZK_ERR_ARG, "the int8 GEMM needs a 256-byte aligned workspace");
  if (ws_bytes < cur_state_bytes())
    return set_error(OZK_ERR_WORKSPACE, "workspace %zu bytes < %zu needed", ws_bytes,
                     cur_state_bytes());
  return launch_slice_gemm_ex(SA, eA, nA, SB, eB, nB, N, M, k_pad, pair_a, pair_b, n_pairs,
                              OZK_ACC_FIXED, symmetric, alpha, beta, Cin, ldcin, C, ldc, nullptr,
                              (double*)workspace, ws_bytes, rho, status_dev, true, skip_if_dev, 0,
                              (cudaStream_t)stream);
}

int ozk_accumulate_2sum(const float* products, const int32_t* eA, const int32_t* eB, int64_t N,
                        int64_t M, int n_hi, int n_lo, float* C_hi, float* C_lo, double* C,
                        int64_t ldc, void* stream) {
  if (!products || !eA || !eB) return set_error(OZK_ERR_ARG, "NULL pointer");
  if (N < 0 || M < 0 || n_hi < 1 || n_lo < 0) return set_error(OZK_ERR_ARG, "bad arguments");
  if (C && ldc < M) return set_error(OZK_ERR_ARG, "ldc < M");
  return launch_accumulate_2sum(products, eA, eB, N, M, n_hi, n_lo, C_hi, C_lo, C, ldc,
                                (cudaStream_t)stream);
}

int ozk_accumulate_2sum_scaled(const float* products, const float* col_scales,
                               const float* row_scales, const int32_t* group_sizes, int n_groups,
                               const int32_t* block_ends, int n_blocks, int64_t N, int64_t M,
                               float* C_hi, float* C_lo, void* stream) {
  if (!products || !col_scales || !row_scales || !group_sizes || !block_ends)
    return set_error(OZK_ERR_ARG, "NULL pointer");
  if (N < 0 || M < 0) return set_error(OZK_ERR_ARG, "bad shape");
  return launch_accumulate_2sum_scaled(products, col_scales, row_scales, group_sizes, n_groups,
                                       block_ends, n_blocks, N, M, C_hi, C_lo,
                                       (cudaStream_t)stream);
}

size_t ozk_matmul_workspace_bytes(int64_t N, int64_t K, int64_t M, int n_hi, int n_lo) {
  return layout(nullptr, N, K, M, n_hi + n_lo, 0, M * K, cur_state_bytes()).bytes;
}

static size_t matmul_ws_bytes_mode(int64_t N, int64_t K, int64_t M, int n_hi, int n_lo, int mode,
                                   bool with_state) {
  int n_prod = mode == OZK_ACC_PRODUCTS ? n_hi * n_hi + 2 * n_hi * n_lo : 0;
  return layout(nullptr, N, K, M, n_hi + n_lo, n_prod, M * K, with_state ? cur_state_bytes() : 0)
      .bytes;
}

int ozk_matmul_f64(const double* A, int64_t lda, const double* B, int64_t ldb, double* C,
                   int64_t ldc, int64_t N, int64_t K, int64_t M, int rho, int n_hi, int n_lo,
                   int acc_mode, void* workspace, size_t ws_bytes, int32_t* status_dev,
                   void* stream) {
  if (!A || !B || !C) return set_error(OZK_ERR_ARG, "NULL pointer");
  if (N < 0 || M < 0 || K < 1) return set_error(OZK_ERR_ARG, "bad shape (K must be >= 1)");
  if (lda < K || ldb < M || ldc < M) return set_error(OZK_ERR_ARG, "leading dimension too small");
  if (acc_mode != OZK_ACC_F64 && acc_mode != OZK_ACC_PRODUCTS && acc_mode != OZK_ACC_FIXED)
    return set_error(OZK_ERR_ARG, "bad acc_mode");
  uint8_t pa[OZK_MAX_PAIRS], pb[OZK_MAX_PAIRS];
  int np = acc_mode == OZK_ACC_FIXED ? snake_pairs(n_hi, n_lo, pa, pb, OZK_MAX_PAIRS)
                                     : ondevice_pairs(n_hi, n_lo, pa, pb, OZK_MAX_PAIRS);
  if (np < 0) return np;
  if (rho < 0) rho = rho_f32(K);
  int rc = check_bound(K, 24 - rho);
  if (rc) return rc;
  if (N == 0 || M == 0) return OZK_OK;
  cudaStream_t s = (cudaStream_t)stream;
  const int nS = n_hi + n_lo;
  const int64_t k_pad = round_up(K, OZK_KB);
  const bool prod = acc_mode == OZK_ACC_PRODUCTS;
  bool with_state;
  if ((rc = pick_workspace(workspace, ws_bytes,
                           matmul_ws_bytes_mode(N, K, M, n_hi, n_lo, acc_mode, !prod),
                           matmul_ws_bytes_mode(N, K, M, n_hi, n_lo, acc_mode, false), with_state)))
    return rc;
  with_state = with_state && !prod;
  size_t need = matmul_ws_bytes_mode(N, K, M, n_hi, n_lo, acc_mode, with_state);
  ScopedWs ws;
  if ((rc = ws.acquire(workspace, workspace ? ws_bytes : need, need, s))) return rc;
  Workspace w = layout(ws.ptr, N, K, M, nS, prod ? np : 0, M * K,
                       with_state ? cur_state_bytes() : 0);
  if (acc_mode == OZK_ACC_FIXED)
    return matmul_fixed(A, lda, B, ldb, C, ldc, N, K, M, rho, n_hi, n_lo, pa, pb, np, w, status_dev,
                        s);
  if ((rc = launch_extract_rows(A, lda, N, K, rho, n_hi, n_lo, w.SA, k_pad, w.eA, status_dev, s)))
    return rc;
  if ((rc = launch_extract_cols(B, ldb, K, M, rho, n_hi, n_lo, w.SB, k_pad, w.eB, status_dev, w.BT,
                                s)))
    return rc;
  if (!prod)
    return launch_slice_gemm(w.SA, w.eA, nS, w.SB, w.eB, nS, N, M, k_pad, pa, pb, np, acc_mode, 0,
                             1.0, 0.0, nullptr, 0, C, ldc, nullptr, w.state, w.state_bytes, rho,
                             status_dev, s);
  if ((rc = launch_slice_gemm(w.SA, w.eA, nS, w.SB, w.eB, nS, N, M, k_pad, pa, pb, np,
                              OZK_ACC_PRODUCTS, 0, 1.0, 0.0, nullptr, 0, nullptr, 0, w.products,
                              nullptr, 0, rho, status_dev, s)))
    return rc;
  return launch_accumulate_2sum(w.products, w.eA, w.eB, N, M, n_hi, n_lo, nullptr, nullptr, C, ldc,
                                s);
}

size_t ozk_matmul_host_workspace_bytes(int64_t N, int64_t K, int64_t M, int n_slices) {
  return layout(nullptr, N, K, M, n_slices, 0, 0, cur_state_bytes()).bytes;
}

int ozk_matmul_host_f64(const double* A, int64_t lda, const double* B, int64_t ldb, double* C,
                        int64_t ldc, int64_t N, int64_t K, int64_t M, int rho, int n_slices,
                        void* workspace, size_t ws_bytes, int32_t* status_dev, void* stream) {
  if (!A || !B || !C) return set_error(OZK_ERR_ARG, "NULL pointer");
  if (N < 0 || M < 0 || K < 1) return set_error(OZK_ERR_ARG, "bad shape (K must be >= 1)");
  if (lda < K || ldb < M || ldc < M) return set_error(OZK_ERR_ARG, "leading dimension too small");
  if (n_slices < 1 || n_slices > OZK_MAX_SLICES)
    return set_error(OZK_ERR_ARG, "n_slices must be in [1,%d]", OZK_MAX_SLICES);
  uint8_t pa[OZK_MAX_PAIRS], pb[OZK_MAX_PAIRS];
  int np = ozk_triangular_schedule(n_slices, pa, pb, OZK_MAX_PAIRS);
  if (np < 0) return np;
  if (rho < 0) rho = rho_f64(K);
  int rc = check_bound(K, 53 - rho);
  if (rc) return rc;
  if (n_slices * (53 - rho) < 53)
    return set_error(OZK_ERR_UNSAFE, "insufficient slice budget: n_slices*bits_per_slice=%d < 53",
                     n_slices * (53 - rho));
  if (N == 0 || M == 0) return OZK_OK;
  cudaStream_t s = (cudaStream_t)stream;
  const int64_t k_pad = round_up(K, OZK_KB);
  bool with_state;
  if ((rc = pick_workspace(workspace, ws_bytes, ozk_matmul_host_workspace_bytes(N, K, M, n_slices),
                           layout(nullptr, N, K, M, n_slices, 0, 0).bytes, with_state)))
    return rc;
  const size_t sb = with_state ? cur_state_bytes() : 0;
  const size_t need = layout(nullptr, N, K, M, n_slices, 0, 0, sb).bytes;
  ScopedWs ws;
  if ((rc = ws.acquire(workspace, workspace ? ws_bytes : need, need, s))) return rc;
  Workspace w = layout(ws.ptr, N, K, M, n_slices, 0, 0, sb);
  if ((rc = launch_extract_rows64(A, lda, N, K, rho, n_slices, w.SA, k_pad, w.eA, status_dev, s)))
    return rc;
  if ((rc = launch_extract_cols64(B, ldb, K, M, rho, n_slices, w.SB, k_pad, w.eB, status_dev, s)))
    return rc;
  return launch_slice_gemm(w.SA, w.eA, n_slices, w.SB, w.eB, n_slices, N, M, k_pad, pa, pb, np,
                           OZK_ACC_F64, 0, 1.0, 0.0, nullptr, 0, C, ldc, nullptr, w.state,
                           w.state_bytes, rho, status_dev, s);
}

// gram: the column extraction of A (N x K) gives, per column of A, slices over
// the N rows -- both the row extraction of A^T and the column extraction of
// A in the reference (gram.py:22-35), which coincide.
size_t ozk_gram_workspace_bytes(int64_t N, int64_t K, int n_hi, int n_lo) {
  return layout(nullptr, K, N, 0, n_hi + n_lo, 0, K * N, cur_state_bytes()).bytes;
}

int ozk_gram_f64(const double* A, int64_t lda, double* G, int64_t ldg, int64_t N, int64_t K,
                 int rho, int n_hi, int n_lo, void* workspace, size_t ws_bytes,
                 int32_t* status_dev, void* stream) {
  if (!A || !G) return set_error(OZK_ERR_ARG, "NULL pointer");
  if (N < 1 || K < 0) return set_error(OZK_ERR_ARG, "bad shape (N must be >= 1)");
  if (lda < K || ldg < K) return set_error(OZK_ERR_ARG, "leading dimension too small");
  uint8_t pa[OZK_MAX_PAIRS], pb[OZK_MAX_PAIRS];
  int np = snake_pairs(n_hi, n_lo, pa, pb, OZK_MAX_PAIRS);
  if (np < 0) return np;
  if (rho < 0) rho = rho_f32(N);
  int rc = check_bound(N, 24 - rho);
  if (rc) return rc;
  if (K == 0) return OZK_OK;
  cudaStream_t s = (cudaStream_t)stream;
  const int nS = n_hi + n_lo;
  const int64_t k_pad = round_up(N, OZK_KB);
  bool with_state;
  if ((rc = pick_workspace(workspace, ws_bytes, ozk_gram_workspace_bytes(N, K, n_hi, n_lo),
                           layout(nullptr, K, N, 0, nS, 0, K * N).bytes, with_state)))
    return rc;
  const size_t sb = with_state ? cur_state_bytes() : 0;
  const size_t need = layout(nullptr, K, N, 0, nS, 0, K * N, sb).bytes;
  ScopedWs ws;
  if ((rc = ws.acquire(workspace, workspace ? ws_bytes : need, need, s))) return rc;
  Workspace w = layout(ws.ptr, K, N, 0, nS, 0, K * N, sb);
  const int64_t k8 = round_up(N, kS8KB);
  if (s8_enabled() && slice_gemm_s8_eligible(K, K, k8, OZK_ACC_FIXED, rho, w.state_bytes)) {
    // int8 pass, then the gated BF16 recomputation from the transposed copy
    cudaError_t e = cudaMemsetAsync(w.gate, 0, sizeof(int32_t), s);
    if (e != cudaSuccess) return set_cuda_error("cudaMemsetAsync(gate)", e);
    if ((rc = launch_extract_cols_s8(A, lda, N, K, rho, n_hi, n_lo, (int8_t*)w.SA, k8, w.eA,
                                     status_dev, w.gate, w.BT, s)))
      return rc;
    if ((rc = launch_slice_gemm_ex(w.SA, w.eA, nS, w.SA, w.eA, nS, K, K, k8, pa, pb, np,
                                   OZK_ACC_FIXED, 1, 1.0, 0.0, nullptr, 0, G, ldg, nullptr, w.state,
                                   w.state_bytes, rho, status_dev, true, w.gate, 0, s)))
      return rc;
    if ((rc = launch_extract_rows_gated(w.BT, N, K, N, rho, n_hi, n_lo, w.SA, k_pad, w.eA,
                                        status_dev, w.gate, s)))
      return rc;
    return launch_slice_gemm_ex(w.SA, w.eA, nS, w.SA, w.eA, nS, K, K, k_pad, pa, pb, np,
                                OZK_ACC_FIXED, 1, 1.0, 0.0, nullptr, 0, G, ldg, nullptr, w.state,
                                w.state_bytes, rho, status_dev, false, w.gate, 1, s);
  }
  if ((rc = launch_extract_cols(A, lda, N, K, rho, n_hi, n_lo, w.SA, k_pad, w.eA, status_dev, w.BT,
                                s)))
    return rc;
  return launch_slice_gemm(w.SA, w.eA, nS, w.SA, w.eA, nS, K, K, k_pad, pa, pb, np, OZK_ACC_FIXED,
                           1, 1.0, 0.0, nullptr, 0, G, ldg, nullptr, w.state, w.state_bytes, rho,
                           status_dev, s);
}

size_t ozk_residual_workspace_bytes(int64_t N, int64_t K, int64_t M, int n_hi, int n_lo) {
  return layout(nullptr, N, K, M, n_hi + n_lo, 0, M * K, cur_state_bytes()).bytes;
}

int ozk_residual_f64(const double* A, int64_t lda, const double* X, int64_t ldx, const double* Bv,
                     int64_t ldb, double* R, int64_t ldr, int64_t N, int64_t K, int64_t M, int rho,
                     int n_hi, int n_lo, void* workspace, size_t ws_bytes, int32_t* status_dev,
                     void* stream) {
  if (!A || !X || !Bv || !R) return set_error(OZK_ERR_ARG, "NULL pointer");
  if (N < 0 || M < 0 || K < 1) return set_error(OZK_ERR_ARG, "bad shape (K must be >= 1)");
  if (lda < K || ldx < M || ldb < M || ldr < M)
    return set_error(OZK_ERR_ARG, "leading dimension too small");
  uint8_t pa[OZK_MAX_PAIRS], pb[OZK_MAX_PAIRS];
  int np = snake_pairs(n_hi, n_lo, pa, pb, OZK_MAX_PAIRS);
  if (np < 0) return np;
  if (rho < 0) rho = rho_f32(K);
  int rc = check_bound(K, 24 - rho);
  if (rc) return rc;
  if (N == 0 || M == 0) return OZK_OK;
  cudaStream_t s = (cudaStream_t)stream;
  const int nS = n_hi + n_lo;
  const int64_t k_pad = round_up(K, OZK_KB);
  bool with_state;
  if ((rc = pick_workspace(workspace, ws_bytes, ozk_residual_workspace_bytes(N, K, M, n_hi, n_lo),
                           layout(nullptr, N, K, M, nS, 0, M * K).bytes, with_state)))
    return rc;
  const size_t sb = with_state ? cur_state_bytes() : 0;
  const size_t need = layout(nullptr, N, K, M, nS, 0, M * K, sb).bytes;
  ScopedWs ws;
  if ((rc = ws.acquire(workspace, workspace ? ws_bytes : need, need, s))) return rc;
  Workspace w = layout(ws.ptr, N, K, M, nS, 0, M * K, sb);
  if (s8_enabled() && M <= 16) {
    rc = skinny_fixed(A, lda, X, ldx, -1.0, 1.0, Bv, ldb, R, ldr, N, K, M, rho, n_hi, n_lo, pa, pb,
                      np, w, status_dev, s);
    if (rc != 1) return rc;
  }
  if ((rc = launch_extract_rows(A, lda, N, K, rho, n_hi, n_lo, w.SA, k_pad, w.eA, status_dev, s)))
    return rc;
  if ((rc = launch_extract_cols(X, ldx, K, M, rho, n_hi, n_lo, w.SB, k_pad, w.eB, status_dev, w.BT,
                                s)))
    return rc;
  return launch_slice_gemm(w.SA, w.eA, nS, w.SB, w.eB, nS, N, M, k_pad, pa, pb, np, OZK_ACC_FIXED,
                           0, -1.0, 1.0, Bv, ldb, R, ldr, nullptr, w.state, w.state_bytes, rho,
                           status_dev, s);
}

int ozk_check_status(const int32_t* status_dev, void* stream) {
  if (!status_dev) return OZK_OK;
  int32_t v = 0;
  cudaError_t e = cudaMemcpyAsync(&v, status_dev, sizeof(v), cudaMemcpyDeviceToHost,
                                  (cudaStream_t)stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize((cudaStream_t)stream);
  if (e != cudaSuccess) return set_cuda_error("reading status", e);
  if (v & OZK_FLAG_TIMEOUT) return set_error(OZK_ERR_TIMEOUT, "a device wait exceeded its budget");
  if (v & (OZK_FLAG_NONFINITE | OZK_FLAG_RANGE))
    return set_error(OZK_ERR_NONFINITE, "inputs contain NaN or Inf or exceed the FP32 range");
  return OZK_OK;
}

const char* ozk_strerror(int status) {
  switch (status) {
    case OZK_OK: return "ok";
    case OZK_ERR_ARG: return "invalid argument";
    case OZK_ERR_UNSAFE: return "input violates the Ozaki exactness preflight";
    case OZK_ERR_NONFINITE: return "input contains NaN/Inf or exceeds the FP32 range";
    case OZK_ERR_CUDA: return "CUDA error";
    case OZK_ERR_NCCL: return "NCCL error";
    case OZK_ERR_TIMEOUT: return "device wait timed out";
    case OZK_ERR_WORKSPACE: return "workspace too small";
    case OZK_ERR_UNSUPPORTED: return "unsupported request";
    default: return "unknown status";
  }
}

int ozk_last_error_detail(char* buf, size_t len) {
  if (!buf || !len) return OZK_ERR_ARG;
  snprintf(buf, len, "%s", t_detail);
  return OZK_OK;
}

int ozk_set_l2_persisting(size_t bytes, size_t* previous) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_cuda_error("cudaGetDevice", e);
  size_t prev = 0;
  if ((e = cudaDeviceGetLimit(&prev, cudaLimitPersistingL2CacheSize)) != cudaSuccess)
    return set_cuda_error("cudaDeviceGetLimit(persisting L2)", e);
  int mx = 0;
  if ((e = cudaDeviceGetAttribute(&mx, cudaDevAttrMaxPersistingL2CacheSize, dev)) != cudaSuccess)
    return set_cuda_error("cudaDeviceGetAttribute(max persisting L2)", e);
  if (previous) *previous = prev;
  if (bytes == (size_t)-1) return OZK_OK;  // query only
  if (bytes > (size_t)mx) bytes = (size_t)mx;
  if ((e = cudaDeviceSetLimit(cudaLimitPersistingL2CacheSize, bytes)) != cudaSuccess)
    return set_cuda_error("cudaDeviceSetLimit(persisting L2)", e);
  return OZK_OK;
}

const char* ozk_version(void) { return "ozaki-b200 0.1.0 (sm_100a)"; }

}  // extern "C"
