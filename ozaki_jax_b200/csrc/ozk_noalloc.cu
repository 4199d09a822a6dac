// ozk_matmul_f64_noalloc: the on-device Ozaki matmul without any device
// allocation, for callers that cannot call cudaMalloc.
//
// Who needs it: code running inside a host framework that owns the GPU's
// memory -- e.g. a JAX/XLA process, which by default reserves most of the
// device for its own allocator, or a plugin's enqueue/execute callback that
// its host forbids from allocating -- cannot count on a cudaMalloc (or a
// stream-ordered pool allocation) succeeding mid-call.  ozk_matmul_f64 needs
// a workspace for the BF16 slices and exponents; this variant takes it from a
// fixed device array compiled into the library instead.
//
// What runs: the same extraction kernels as ozk_matmul_f64 and, because the
// array holds no GEMM state scratch, the slice GEMM's 128-wide BF16 tiles
// that keep their running sums in TMEM (products with at most 16 columns use
// the int8 skinny kernel).  Sums are exact fixed-point integers either way,
// so C is bit-identical to ozk_matmul_f64 with OZK_ACC_FIXED.
//
// The scratch is a file-scope __device__ array of OZK_NOALLOC_SCRATCH_BYTES
// (32 MiB).  Every GPU that loads the library holds it until the process
// exits.  That bounds the problem size: the slices-only workspace of an
// N x K by K x M product with (n_hi, n_lo) slices must fit, i.e.
//   align256(2 nS N k_pad) + align256(2 nS M k_pad) + align256(4 nS N)
//   + align256(4 nS M) + align256(8 K M) + 256 <= 32 MiB,
// nS = n_hi + n_lo, k_pad = K rounded up to 64 (1024 x 1024 x 1024 at
// precision 'high' fits); larger requests are refused with OZK_ERR_WORKSPACE.
// Host code never hands the array's name to a kernel (on the host it is only
// a stand-in for the symbol); its device address is looked up with
// cudaGetSymbolAddress in the current context on every call (a cheap lookup),
// so nothing goes stale when a caller switches or recreates contexts.  The
// first call in a context also loads the library's module there, so it
// should come before any stream capture.  All calls on a device share
// the one array and it keeps the last call's contents: nothing in it needs to
// start at zero (the extraction kernels write every slice element, padding
// included, and every exponent before the GEMM reads them), but calls whose
// executions overlap on the GPU -- concurrent streams, or other host threads
// using the same device -- race on it and must be serialised by the caller.
#include <cuda_runtime.h>
#include <stdint.h>

#include "ozaki_b200.h"
#include "ozk_internal.h"

namespace {

__device__ __align__(256) unsigned char g_noalloc_scratch[OZK_NOALLOC_SCRATCH_BYTES];

// The array's address in the current context.  A __device__ symbol's address
// belongs to a context, not to a device index, so it is not cached.
int scratch_for_current_context(void** out) {
  void* p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess || !p) return ozk::set_cuda_error("cudaGetSymbolAddress(scratch)", e);
  *out = p;
  return OZK_OK;
}

}  // namespace

extern "C" int ozk_matmul_f64_noalloc(const double* A, int64_t lda, const double* B, int64_t ldb,
                                      double* C, int64_t ldc, int64_t N, int64_t K, int64_t M,
                                      int n_hi, int n_lo, int32_t* status_dev, void* stream) {
  if (N < 0 || K < 0 || M < 0) return ozk::set_error(OZK_ERR_ARG, "bad shape");
  if (n_hi < 1 || n_lo < 0 || n_hi > OZK_MAX_SIDE || n_lo > OZK_MAX_SIDE)
    return ozk::set_error(OZK_ERR_ARG, "n_hi must be in [1,%d] and n_lo in [0,%d]", OZK_MAX_SIDE,
                          OZK_MAX_SIDE);
  const size_t need = ozk::matmul_min_workspace_bytes(N, K, M, n_hi, n_lo);
  if (need > (size_t)OZK_NOALLOC_SCRATCH_BYTES)
    return ozk::set_error(OZK_ERR_WORKSPACE,
                          "ozk_matmul_f64_noalloc: %lld x %lld x %lld with %d+%d slices needs %zu "
                          "bytes of scratch, more than its fixed %d-byte device array; use "
                          "ozk_matmul_f64 with a workspace",
                          (long long)N, (long long)K, (long long)M, n_hi, n_lo, need,
                          (int)OZK_NOALLOC_SCRATCH_BYTES);
  void* scratch = nullptr;
  int rc = scratch_for_current_context(&scratch);
  if (rc) return rc;
  return ozk_matmul_f64(A, lda, B, ldb, C, ldc, N, K, M, -1, n_hi, n_lo, OZK_ACC_FIXED, scratch,
                        (size_t)OZK_NOALLOC_SCRATCH_BYTES, status_dev, stream);
}
