// Host-side internals shared by the library's translation units.
#pragma once

#include <cuda.h>
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
// BF16 -> FP32 exact inner-product bound K * (2^bits - 1)^2 < 2^24; returns
// OZK_ERR_UNSAFE (with the detail text) when violated.
int check_bound(int64_t K, int bits);
uint64_t wait_budget_ns();

inline int64_t round_up(int64_t x, int64_t m) { return (x + m - 1) / m * m; }

// int8 slices: exact for rho >= 19 (|code| <= 64); a pipeline stage holds 128
// int8 K-elements (the same 128 bytes per row as 64 BF16 elements).
constexpr int kS8MinRho = 19;
constexpr int kS8KB = 128;

int launch_extract_rows(const double* X, int64_t ldx, int64_t rows, int64_t K, int rho, int n_hi,
                        int n_lo, uint16_t* slices, int64_t k_pad, int32_t* exps, int32_t* status,
                        cudaStream_t stream);
// With gate non-NULL the kernels do nothing unless *gate != 0 (device-side
// recomputation after a failed int8 extraction); needs k_pad <= 65536.
int launch_extract_rows_gated(const double* X, int64_t ldx, int64_t rows, int64_t K, int rho,
                              int n_hi, int n_lo, uint16_t* slices, int64_t k_pad, int32_t* exps,
                              int32_t* status, const int32_t* gate, cudaStream_t stream);
// int8 slice codes (slice * 2^(24 - rho)), [n_hi+n_lo][rows][k_pad] int8; needs
// rho >= kS8MinRho and k_pad a multiple of kS8KB, <= 65536.  Sets *s8_fail = 1
// when a slice value has no exact code (the caller then recomputes in BF16).
int launch_extract_rows_s8(const double* X, int64_t ldx, int64_t rows, int64_t K, int rho,
                           int n_hi, int n_lo, int8_t* slices, int64_t k_pad, int32_t* exps,
                           int32_t* status, int32_t* s8_fail, cudaStream_t stream);
int launch_extract_cols_s8(const double* X, int64_t ldx, int64_t K, int64_t cols, int rho,
                           int n_hi, int n_lo, int8_t* slices, int64_t k_pad, int32_t* exps,
                           int32_t* status, int32_t* s8_fail, double* scratch,
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
// The same with the slice type and a device-side gate: s8 selects int8 slice
// codes (layout [n][rows][k_pad] int8, k_pad a multiple of kS8KB) and the
// kind::i8 kernel; with gate non-NULL the kernel does nothing unless
// (*gate != 0) == gate_want.
int launch_slice_gemm_ex(const void* SA, const int32_t* eA, int nA, const void* SB,
                         const int32_t* eB, int nB, int64_t N, int64_t M, int64_t k_pad,
                         const uint8_t* pair_a, const uint8_t* pair_b, int n_pairs, int mode,
                         int symmetric, double alpha, double beta, const double* Cin,
                         int64_t ldcin, double* C, int64_t ldc, float* products, double* state,
                         size_t state_bytes, int rho, int32_t* status, bool s8,
                         const int32_t* gate, int gate_want, cudaStream_t stream,
                         long long* C64 = nullptr);
// Whether the int8 GEMM serves this request (fixed-point sums, rho >= 19,
// 256-wide tiles with the state scratch, k_pad within the extraction limits).
bool slice_gemm_s8_eligible(int64_t N, int64_t M, int64_t k_pad, int mode, int rho,
                            size_t state_bytes);
// Skinny int8 slice GEMM (M <= 16 right-hand sides, fixed-point sums): every
// pair product of a 128-row tile accumulates at once, so each A slice is read
// once.  SX [nS][M][k8] int8 codes of X's columns, eX [nS][M].
bool skinny_s8_eligible(int64_t N, int64_t M, int64_t k8, int nS, int n_pairs, int rho);
int launch_skinny_s8(const int8_t* SA, const int32_t* eA, const int8_t* SX, const int32_t* eX,
                     int nS, int64_t N, int64_t M, int64_t k8, const uint8_t* pair_a,
                     const uint8_t* pair_b, int n_pairs, double alpha, double beta,
                     const double* Cin, int64_t ldcin, double* C, int64_t ldc, int rho,
                     int32_t* status, const int32_t* gate, int gate_want, void* scratch,
                     size_t scratch_bytes, cudaStream_t stream);
// int8 slices enabled (OZK_S8=0 in the environment turns them off).
bool s8_enabled();
// Tensor map over a [depth][rows][k_pad] slice stack (BF16, or int8 codes
// with s8), box of 128 bytes x box_rows, 128-byte swizzle.
int make_slice_map(CUtensorMap* map, const void* base, int64_t k_pad, int64_t rows, int depth,
                   int box_rows, bool s8);
// One slice pass of the int8 line extraction over this GPU's part of each
// line (X: lines x n, ldx): t = -1 writes the part's maxima of the split
// values to pmax [2][lines]; t >= 0 takes pass t's line maxima from gmax,
// writes exps and the codes of slice t (and n_hi + t), and, while t + 1 <
// npass, the part's maxima after the pass to pmax.  See k_line_pass_s8.
int launch_line_pass_s8(const double* X, int64_t ldx, int64_t lines, int64_t n, int t, int npass,
                        int rho, int n_hi, int n_lo, const float* gmax, float* pmax,
                        int8_t* slices, int64_t k_pad, int32_t* exps, int32_t* status,
                        int32_t* s8_fail, cudaStream_t stream);
// Bytes of the per-CTA FP64 state scratch the 256-wide GEMM tiles need.
size_t gemm_state_bytes(int dev);
// Smallest workspace ozk_matmul_f64 (OZK_ACC_F64) accepts: without the state
// scratch it runs 128-wide tiles.
size_t matmul_min_workspace_bytes(int64_t N, int64_t K, int64_t M, int n_hi, int n_lo);
int launch_accumulate_2sum_scaled(const float* products, const float* col_scales,
                                  const float* row_scales, const int32_t* group_sizes,
                                  int n_groups, const int32_t* block_ends, int n_blocks, int64_t N,
                                  int64_t M, float* C_hi, float* C_lo, cudaStream_t stream);
// Pageable host memory (neither page-locked, registered, managed nor device).
bool is_pageable(const void* p);
// Copies between pageable host memory and the device through the library's
// page-locked staging ring with host memcpy threads (ozk_staging.cu), rows of
// `width` bytes with the given pitches, ordered on `s`.  staged_h2d_2d returns
// once the source has been read (DMAs may still run on s); staged_d2h_2d
// returns when the destination holds the data.
int staged_h2d_2d(void* dst, size_t dpitch, const void* src, size_t spitch, size_t width,
                  size_t rows, cudaStream_t s);
int staged_d2h_2d(void* dst, size_t dpitch, const void* src, size_t spitch, size_t width,
                  size_t rows, cudaStream_t s);
int launch_accumulate_2sum(const float* products, const int32_t* eA, const int32_t* eB, int64_t N,
                           int64_t M, int n_hi, int n_lo, float* C_hi, float* C_lo, double* C,
                           int64_t ldc, cudaStream_t stream);

}  // namespace ozk
