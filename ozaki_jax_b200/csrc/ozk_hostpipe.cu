// ozk_matmul_f64_hostbuf: the on-device pipeline driven from host arrays, with
// the PCIe copies overlapped with the compute.
//
// The reference's ozaki_jax.matmul on NumPy inputs (ozaki_jax/matmul.py:781-821)
// moves A and B to the device, runs the jitted pipeline (:641-686) and brings C
// back, one stage after the other.  Here the three stages overlap:
//
//   copy stream H2D :  B  | A[0] | A[1] | ...
//   caller's stream :        extract(B) | extract(A[0]) GEMM[0] | extract(A[1]) GEMM[1] | ...
//   copy stream D2H :                                           | C[0] ...          | C[1]
//
// A and C move in row blocks.  Row extraction is row-local and each block's
// GEMM produces exactly the rows of C the full product would (same slices, same
// exponents, same per-element sums), so the result does not depend on the
// blocking.  Events order the three streams; nothing here synchronises the
// host until the last copy has been issued.  The copies use unified
// addressing, so any of A, B and C may also be device memory (a B already
// gathered on this GPU is copied on the device, not over PCIe).
//
// Ordinary pageable host arrays (what a NumPy caller passes) are moved through
// the library's page-locked staging ring with host memcpy threads
// (ozk_staging.cu): the H2D side stages B, then each block of A, enqueueing
// each block's compute as soon as its rows are on their way; a pageable C is
// copied out by a helper thread block by block as each block's GEMM finishes,
// while the calling thread is still staging later blocks of A.
#include <cuda_runtime.h>
#include <stdint.h>

#include <condition_variable>
#include <mutex>
#include <thread>
#include <vector>

#include "ozaki_b200.h"
#include "ozk_internal.h"

namespace {

using namespace ozk;

struct CopyStreams {
  cudaStream_t h2d = nullptr;
  cudaStream_t d2h = nullptr;
};

CopyStreams g_copy_streams[64];
std::mutex g_copy_mu;

// The two copy streams of the current device, created on first use and kept
// for the life of the process (non-blocking: they never wait on stream 0).
int copy_streams(CopyStreams* out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_cuda_error("cudaGetDevice", e);
  if (dev < 0 || dev >= 64) return set_error(OZK_ERR_ARG, "device index %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_copy_mu);
  CopyStreams& cs = g_copy_streams[dev];
  if (!cs.h2d) {
    cudaStream_t a = nullptr, b = nullptr;
    if ((e = cudaStreamCreateWithFlags(&a, cudaStreamNonBlocking)) != cudaSuccess)
      return set_cuda_error("cudaStreamCreate(h2d)", e);
    if ((e = cudaStreamCreateWithFlags(&b, cudaStreamNonBlocking)) != cudaSuccess) {
      cudaStreamDestroy(a);
      return set_cuda_error("cudaStreamCreate(d2h)", e);
    }
    cs.h2d = a;
    cs.d2h = b;
  }
  *out = cs;
  return OZK_OK;
}

size_t a256(size_t x) { return (x + 255) & ~(size_t)255; }

struct HostbufLayout {
  double* A;       // [N][K]
  double* B;       // [K][M]
  double* BT;      // [M][K] transposed B for the column extraction
  double* C;       // [N][M]
  uint16_t* SA;    // per row block b (rows r0..r1): [nS][r1-r0][k_pad] at nS*r0*k_pad
  uint16_t* SB;    // [nS][M][k_pad]
  int32_t* eA;     // per row block: [nS][r1-r0] at nS*r0
  int32_t* eB;     // [nS][M]
  float* products; // [n_pairs][block_rows][M] (OZK_ACC_PRODUCTS only)
  double* state;   // GEMM state scratch (other modes)
  size_t state_bytes;
  int32_t* status;
  int32_t* gate;   // set when an int8 slice code failed (BF16 recomputation runs)
  size_t bytes;
};

HostbufLayout hostbuf_layout(void* base, int64_t N, int64_t K, int64_t M, int nS, int n_prod,
                             int64_t block_rows, size_t state_bytes) {
  const int64_t k_pad = round_up(K, OZK_KB);
  HostbufLayout w;
  char* b = (char*)base;
  size_t off = 0;
  auto take = [&](size_t n) {
    char* p = b + off;
    off += a256(n);
    return p;
  };
  w.A = (double*)take((size_t)N * K * 8);
  w.B = (double*)take((size_t)K * M * 8);
  w.BT = (double*)take((size_t)M * K * 8);
  w.C = (double*)take((size_t)N * M * 8);
  w.SA = (uint16_t*)take((size_t)nS * N * k_pad * 2);
  w.SB = (uint16_t*)take((size_t)nS * M * k_pad * 2);
  w.eA = (int32_t*)take((size_t)nS * N * 4);
  w.eB = (int32_t*)take((size_t)nS * M * 4);
  w.products = (float*)take((size_t)n_prod * block_rows * M * 4);
  w.state = state_bytes ? (double*)take(state_bytes) : nullptr;
  w.state_bytes = state_bytes;
  w.status = (int32_t*)take(4);
  w.gate = (int32_t*)take(4);
  w.bytes = off;
  return w;
}

// Rows per block: about N/8 rounded to 256 rows, at least 512.  Smaller
// blocks start the first GEMM sooner (it waits for B and one block of A) and
// leave less copy-out after the last one, at the price of a less full last
// wave per GEMM; measured on B200 at 8192^3 over PCIe Gen5, 512-1024-row
// blocks gave the shortest end-to-end time.  A last block under 256 rows is
// merged into the one before.
int64_t pick_block_rows(int64_t N, int64_t block_rows) {
  int64_t br = block_rows;
  if (br <= 0) {
    br = round_up((N + 7) / 8, 256);
    if (br < 512) br = 512;
  }
  if (br >= N) return N;
  const int64_t tail = N % br;
  if (tail > 0 && tail < 256 && N / br >= 1 && block_rows <= 0) {
    // spread the short tail over the blocks
    const int64_t nblk = N / br;
    br = round_up((N + nblk - 1) / nblk, 256);
  }
  return br < N ? br : N;
}

int n_pairs_of(int n_hi, int n_lo) { return n_hi * n_hi + 2 * n_hi * n_lo; }

// The helper thread that copies C's blocks out to pageable memory: block b is
// taken once the calling thread has enqueued its compute (enqueued(b + 1)).
// finish(abort) waits for the thread; with abort set it stops before the
// blocks not yet enqueued.  Returns the thread's first error.
class BlockCopyOut {
 public:
  template <class F>
  void start(int dev, int nblk, F copy_block) {
    th_ = std::thread([this, dev, nblk, copy_block] {
      cudaSetDevice(dev);
      for (int b = 0; b < nblk; ++b) {
        {
          std::unique_lock<std::mutex> lk(mu_);
          cv_.wait(lk, [&] { return abort_ || enqueued_ > b; });
          if (enqueued_ <= b) return;  // aborted before this block was enqueued
        }
        const int rc = copy_block(b);
        if (rc) {
          std::lock_guard<std::mutex> lk(mu_);
          if (!rc_) rc_ = rc;
          return;
        }
      }
    });
  }
  void enqueued(int n) {
    if (!th_.joinable()) return;
    {
      std::lock_guard<std::mutex> lk(mu_);
      enqueued_ = n;
    }
    cv_.notify_all();
  }
  int finish(bool abort) {
    if (!th_.joinable()) return OZK_OK;
    {
      std::lock_guard<std::mutex> lk(mu_);
      if (abort) abort_ = true;
    }
    cv_.notify_all();
    th_.join();
    return rc_;
  }
  ~BlockCopyOut() { finish(true); }

 private:
  std::thread th_;
  std::mutex mu_;
  std::condition_variable cv_;
  int enqueued_ = 0;
  bool abort_ = false;
  int rc_ = OZK_OK;
};

}  // namespace

extern "C" size_t ozk_matmul_hostbuf_workspace_bytes(int64_t N, int64_t K, int64_t M, int n_hi,
                                                     int n_lo, int acc_mode, int64_t block_rows) {
  if (N < 0 || K < 1 || M < 0 || n_hi < 1 || n_lo < 0) return 0;
  const bool prod = acc_mode == OZK_ACC_PRODUCTS;
  const int64_t br = pick_block_rows(N, block_rows);
  return hostbuf_layout(nullptr, N, K, M, n_hi + n_lo, prod ? n_pairs_of(n_hi, n_lo) : 0, br,
                        prod ? 0 : ozk_slice_gemm_workspace_bytes())
      .bytes;
}

extern "C" int ozk_matmul_f64_hostbuf(const double* A, int64_t lda, const double* B, int64_t ldb,
                                      double* C, int64_t ldc, int64_t N, int64_t K, int64_t M,
                                      int rho, int n_hi, int n_lo, int acc_mode,
                                      int64_t block_rows, void* workspace, size_t ws_bytes,
                                      int32_t* status_host, void* stream) {
  if (!A || !B || !C || !status_host) return set_error(OZK_ERR_ARG, "NULL pointer");
  if (N < 0 || M < 0 || K < 1) return set_error(OZK_ERR_ARG, "bad shape (K must be >= 1)");
  if (lda < K || ldb < M || ldc < M) return set_error(OZK_ERR_ARG, "leading dimension too small");
  if (acc_mode != OZK_ACC_F64 && acc_mode != OZK_ACC_PRODUCTS && acc_mode != OZK_ACC_FIXED)
    return set_error(OZK_ERR_ARG, "bad acc_mode");
  uint8_t pa[OZK_MAX_PAIRS], pb[OZK_MAX_PAIRS];
  const int np = acc_mode == OZK_ACC_FIXED
                     ? ozk_pair_schedule_snake(n_hi, n_lo, pa, pb, OZK_MAX_PAIRS)
                     : ozk_pair_schedule(n_hi, n_lo, pa, pb, OZK_MAX_PAIRS);
  if (np < 0) return np;
  if (rho < 0) rho = ozk_compute_rho_f32(K);
  int rc = check_bound(K, 24 - rho);
  if (rc) return rc;
  *status_host = 0;
  if (N == 0 || M == 0) return OZK_OK;

  const int nS = n_hi + n_lo;
  const int64_t k_pad = round_up(K, OZK_KB);
  const bool prod = acc_mode == OZK_ACC_PRODUCTS;
  const int64_t br = pick_block_rows(N, block_rows);
  const int nblk = (int)((N + br - 1) / br);
  const size_t need = ozk_matmul_hostbuf_workspace_bytes(N, K, M, n_hi, n_lo, acc_mode, br);
  if (workspace && ws_bytes < need)
    return set_error(OZK_ERR_WORKSPACE, "workspace %zu bytes < %zu needed", ws_bytes, need);
  if (workspace && ((uintptr_t)workspace & 255))
    return set_error(OZK_ERR_ARG, "workspace not 256-byte aligned");

  cudaStream_t s = (cudaStream_t)stream;
  CopyStreams cs;
  if ((rc = copy_streams(&cs))) return rc;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return set_error(OZK_ERR_CUDA, "cudaGetDevice failed");
  const bool a_pageable = is_pageable(A), b_pageable = is_pageable(B);
  const bool c_pageable = is_pageable(C);
  BlockCopyOut d2h;

  // Events: entry, B ready, A block ready x nblk, C block ready x nblk, copies done x 2.
  std::vector<cudaEvent_t> ev(4 + 2 * (size_t)nblk, nullptr);
  for (auto& e : ev) {
    cudaError_t ce = cudaEventCreateWithFlags(&e, cudaEventDisableTiming);
    if (ce != cudaSuccess) {
      for (auto& x : ev)
        if (x) cudaEventDestroy(x);
      return set_cuda_error("cudaEventCreate", ce);
    }
  }
  cudaEvent_t ev_entry = ev[0], ev_b = ev[1], ev_h2d_done = ev[2], ev_d2h_done = ev[3];
  cudaEvent_t* ev_a = ev.data() + 4;
  cudaEvent_t* ev_c = ev.data() + 4 + nblk;

  void* base = workspace;
  bool owned = false;
  cudaError_t ce = cudaSuccess;
  if (!base) {
    if ((ce = cudaMallocAsync(&base, need, s)) != cudaSuccess) {
      for (auto& x : ev) cudaEventDestroy(x);
      return set_cuda_error("cudaMallocAsync(workspace)", ce);
    }
    owned = true;
  }
  HostbufLayout w = hostbuf_layout(base, N, K, M, nS, prod ? np : 0, br,
                                   prod ? 0 : ozk_slice_gemm_workspace_bytes());
  // int8 slices when every block's GEMM can take them
  const int64_t k8 = round_up(K, kS8KB);
  const int64_t last_rows = N - (int64_t)(nblk - 1) * br;
  const bool s8 = acc_mode == OZK_ACC_FIXED && s8_enabled() &&
                  slice_gemm_s8_eligible(br < last_rows ? br : last_rows, M, k8, OZK_ACC_FIXED,
                                         rho, w.state_bytes);

#define OZK_TRY_CUDA(call, what)                 \
  do {                                           \
    ce = (call);                                 \
    if (ce != cudaSuccess) {                     \
      rc = set_cuda_error(what, ce);             \
      goto done;                                 \
    }                                            \
  } while (0)
#define OZK_TRY(call)     \
  do {                    \
    rc = (call);          \
    if (rc) goto done;    \
  } while (0)

  OZK_TRY_CUDA(cudaMemsetAsync(w.status, 0, 4, s), "cudaMemsetAsync(status)");
  OZK_TRY_CUDA(cudaMemsetAsync(w.gate, 0, 4, s), "cudaMemsetAsync(gate)");
  OZK_TRY_CUDA(cudaEventRecord(ev_entry, s), "cudaEventRecord");
  OZK_TRY_CUDA(cudaStreamWaitEvent(cs.h2d, ev_entry, 0), "cudaStreamWaitEvent");
  OZK_TRY_CUDA(cudaStreamWaitEvent(cs.d2h, ev_entry, 0), "cudaStreamWaitEvent");

  // A pageable C is copied out by a helper thread, block by block, as each
  // block's compute is enqueued and then finished.
  if (c_pageable) {
    d2h.start(dev, nblk, [&, C](int b) -> int {
      const int64_t r0 = b * br, nb = (r0 + br <= N ? br : N - r0);
      cudaError_t e = cudaStreamWaitEvent(cs.d2h, ev_c[b], 0);
      if (e != cudaSuccess) return set_cuda_error("cudaStreamWaitEvent", e);
      return staged_d2h_2d(C + r0 * ldc, (size_t)ldc * 8, w.C + r0 * M, (size_t)M * 8,
                           (size_t)M * 8, (size_t)nb, cs.d2h);
    });
  }

  // Host -> device: B first, then its column extraction.
  if (b_pageable)
    OZK_TRY(staged_h2d_2d(w.B, (size_t)M * 8, B, (size_t)ldb * 8, (size_t)M * 8, (size_t)K,
                          cs.h2d));
  else
    OZK_TRY_CUDA(cudaMemcpy2DAsync(w.B, (size_t)M * 8, B, (size_t)ldb * 8, (size_t)M * 8,
                                   (size_t)K, cudaMemcpyDefault, cs.h2d),
                 "cudaMemcpy2DAsync(B)");
  OZK_TRY_CUDA(cudaEventRecord(ev_b, cs.h2d), "cudaEventRecord");
  OZK_TRY_CUDA(cudaStreamWaitEvent(s, ev_b, 0), "cudaStreamWaitEvent");
  if (s8)
    OZK_TRY(launch_extract_cols_s8(w.B, M, K, M, rho, n_hi, n_lo, (int8_t*)w.SB, k8, w.eB, w.status,
                                   w.gate, w.BT, s));
  else
    OZK_TRY(launch_extract_cols(w.B, M, K, M, rho, n_hi, n_lo, w.SB, k_pad, w.eB, w.status, w.BT,
                                s));
  // Then block by block: the rows of A, and the block's compute behind them.
  for (int b = 0; b < nblk; ++b) {
    const int64_t r0 = b * br, nb = (r0 + br <= N ? br : N - r0);
    if (a_pageable)
      OZK_TRY(staged_h2d_2d(w.A + r0 * K, (size_t)K * 8, A + r0 * lda, (size_t)lda * 8,
                            (size_t)K * 8, (size_t)nb, cs.h2d));
    else
      OZK_TRY_CUDA(cudaMemcpy2DAsync(w.A + r0 * K, (size_t)K * 8, A + r0 * lda, (size_t)lda * 8,
                                     (size_t)K * 8, (size_t)nb, cudaMemcpyDefault, cs.h2d),
                   "cudaMemcpy2DAsync(A)");
    OZK_TRY_CUDA(cudaEventRecord(ev_a[b], cs.h2d), "cudaEventRecord");
    uint16_t* SA = w.SA + (size_t)nS * r0 * k_pad;
    int32_t* eA = w.eA + (size_t)nS * r0;
    double* Cb = w.C + r0 * M;
    OZK_TRY_CUDA(cudaStreamWaitEvent(s, ev_a[b], 0), "cudaStreamWaitEvent");
    if (s8) {
      // int8 pass; then the BF16 recomputation of B's and this block's slices
      // and of the block's GEMM, which run only if some int8 code failed (the
      // gate stays set for the rest of the call).
      OZK_TRY(launch_extract_rows_s8(w.A + r0 * K, K, nb, K, rho, n_hi, n_lo, (int8_t*)SA, k8, eA,
                                     w.status, w.gate, s));
      OZK_TRY(launch_slice_gemm_ex(SA, eA, nS, w.SB, w.eB, nS, nb, M, k8, pa, pb, np,
                                   OZK_ACC_FIXED, 0, 1.0, 0.0, nullptr, 0, Cb, M, nullptr, w.state,
                                   w.state_bytes, rho, w.status, true, w.gate, 0, s));
      OZK_TRY(launch_extract_rows_gated(w.BT, K, M, K, rho, n_hi, n_lo, w.SB, k_pad, w.eB,
                                        w.status, w.gate, s));
      OZK_TRY(launch_extract_rows_gated(w.A + r0 * K, K, nb, K, rho, n_hi, n_lo, SA, k_pad, eA,
                                        w.status, w.gate, s));
      OZK_TRY(launch_slice_gemm_ex(SA, eA, nS, w.SB, w.eB, nS, nb, M, k_pad, pa, pb, np,
                                   OZK_ACC_FIXED, 0, 1.0, 0.0, nullptr, 0, Cb, M, nullptr, w.state,
                                   w.state_bytes, rho, w.status, false, w.gate, 1, s));
    } else {
      OZK_TRY(launch_extract_rows(w.A + r0 * K, K, nb, K, rho, n_hi, n_lo, SA, k_pad, eA,
                                  w.status, s));
      if (!prod) {
        OZK_TRY(launch_slice_gemm(SA, eA, nS, w.SB, w.eB, nS, nb, M, k_pad, pa, pb, np, acc_mode,
                                  0, 1.0, 0.0, nullptr, 0, Cb, M, nullptr, w.state, w.state_bytes,
                                  rho, w.status, s));
      } else {
        OZK_TRY(launch_slice_gemm(SA, eA, nS, w.SB, w.eB, nS, nb, M, k_pad, pa, pb, np,
                                  OZK_ACC_PRODUCTS, 0, 1.0, 0.0, nullptr, 0, nullptr, 0,
                                  w.products, nullptr, 0, rho, w.status, s));
        OZK_TRY(launch_accumulate_2sum(w.products, eA, w.eB, nb, M, n_hi, n_lo, nullptr, nullptr,
                                       Cb, M, s));
      }
    }
    OZK_TRY_CUDA(cudaEventRecord(ev_c[b], s), "cudaEventRecord");
    d2h.enqueued(b + 1);
  }

  // Device -> host into page-locked or device memory: block by block as each
  // GEMM finishes, issued after all compute.
  if (!c_pageable) {
    for (int b = 0; b < nblk; ++b) {
      const int64_t r0 = b * br, nb = (r0 + br <= N ? br : N - r0);
      OZK_TRY_CUDA(cudaStreamWaitEvent(cs.d2h, ev_c[b], 0), "cudaStreamWaitEvent");
      OZK_TRY_CUDA(cudaMemcpy2DAsync(C + r0 * ldc, (size_t)ldc * 8, w.C + r0 * M, (size_t)M * 8,
                                     (size_t)M * 8, (size_t)nb, cudaMemcpyDefault, cs.d2h),
                   "cudaMemcpy2DAsync(C)");
    }
  }

done:
#undef OZK_TRY
#undef OZK_TRY_CUDA
  {
    // the copy-out thread finishes (or gives up after an error) before the
    // workspace and the events go
    const int rc_d2h = d2h.finish(rc != OZK_OK);
    if (!rc) rc = rc_d2h;
    // Whatever happened, the copy streams must be finished with the workspace
    // (and with the caller's host buffers) before it is released and before we
    // return.
    cudaEventRecord(ev_h2d_done, cs.h2d);
    cudaEventRecord(ev_d2h_done, cs.d2h);
    cudaStreamWaitEvent(s, ev_h2d_done, 0);
    cudaStreamWaitEvent(s, ev_d2h_done, 0);
    int32_t flags = 0;
    cudaError_t e2 = cudaMemcpyAsync(&flags, w.status, 4, cudaMemcpyDeviceToHost, s);
    if (owned) cudaFreeAsync(base, s);
    cudaError_t e3 = cudaStreamSynchronize(s);
    cudaStreamSynchronize(cs.d2h);
    cudaStreamSynchronize(cs.h2d);
    for (auto& x : ev) cudaEventDestroy(x);
    if (!rc && e2 != cudaSuccess) rc = set_cuda_error("cudaMemcpyAsync(status)", e2);
    if (!rc && e3 != cudaSuccess) rc = set_cuda_error("cudaStreamSynchronize", e3);
    if (!rc) *status_host = flags;
  }
  return rc;
}
