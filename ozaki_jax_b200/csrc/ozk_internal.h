// Host-side internals shared by the library's translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "ozaki_b200.h"

#define OZK_MAX_SIDE 8      // slices per hi/lo side (per operand side for host pipeline: 16)
#define OZK_MAX_SLICES 16   // slices per operand
#define OZK_MAX_PAIRS 256   // pairs per GEMM launch
#define OZK_KB 64           // K elements per pipeline stage (128 bytes of BF16)

namespace ozk {

// Error reporting: records a per-thread detail string and returns the code.
int set_error(int code, const char* fmt, ...);
int set_cuda_error(const char* what, cudaError_t e);

int device_sm_count(int dev);
uint64_t wait_budget_ns();

inline int64_t round_up(int64_t x, int64_t m) { return (x + m - 1) / m * m; }

int launch_extract_rows(const double* X, int64_t ldx, int64_t rows, int64_t K, int rho, int n_hi,
                        int n_lo, uint16_t* slices, int64_t k_pad, int32_t* exps, int32_t* status,
                        cudaStream_t stream);
// scratch: cols x K FP64 buffer for the transposed fast path (NULL selects the
// multi-pass column kernel).
int launch_extract_cols(const double* X, int64_t ldx, int64_t K, int64_t cols, int rho, int n_hi,
                        int n_lo, uint16_t* slices, int64_t k_pad, int32_t* exps, int32_t* status,
                        double* scratch, cudaStream_t stream);
int launch_transpose_f64(const double* X, int64_t ldx, int64_t rows, int64_t cols, double* XT,
                         cudaStream_t stream);
int launch_extract_rows64(const double* X, int64_t ldx, int64_t rows, int64_t K, int rho, int ns,
                          uint16_t* slices, int64_t k_pad, int32_t* exps, int32_t* status,
                          cudaStream_t stream);
int launch_extract_cols64(const double* X, int64_t ldx, int64_t K, int64_t cols, int rho, int ns,
                          uint16_t* slices, int64_t k_pad, int32_t* exps, int32_t* status,
                          cudaStream_t stream);
int launch_slice_gemm(const uint16_t* SA, const int32_t* eA, int nA, const uint16_t* SB,
                      const int32_t* eB, int nB, int64_t N, int64_t M, int64_t k_pad,
                      const uint8_t* pair_a, const uint8_t* pair_b, int n_pairs, int mode,
                      int symmetric, double alpha, double beta, const double* Cin, int64_t ldcin,
                      double* C, int64_t ldc, float* products, double* state, size_t state_bytes,
                      int rho, int32_t* status, cudaStream_t stream);
// Bytes of the per-CTA FP64 state scratch the 256-wide GEMM tiles need.
size_t gemm_state_bytes(int dev);
// Smallest workspace ozk_matmul_f64 (OZK_ACC_F64) accepts: without the state
// scratch it runs 128-wide tiles.
size_t matmul_min_workspace_bytes(int64_t N, int64_t K, int64_t M, int n_hi, int n_lo);
int launch_accumulate_2sum(const float* products, const int32_t* eA, const int32_t* eB, int64_t N,
                           int64_t M, int n_hi, int n_lo, float* C_hi, float* C_lo, double* C,
                           int64_t ldc, cudaStream_t stream);

}  // namespace ozk
