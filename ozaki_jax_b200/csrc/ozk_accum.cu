// Reference-order FP32 2Sum accumulation over materialised slice products
// (ozaki_jax/pallas_ops.py:178-239 with the scales of :107-175), one thread
// per output element.  Used by accumulation='ondevice' and by parity tests
// that need the reference's (C_hi, C_lo) words bit for bit.
#include <cuda_runtime.h>
#include <stdint.h>

#include "ozk_device.cuh"
#include "ozk_internal.h"

namespace ozk {

struct TwoSum {
  float hi, lo;
  __device__ __forceinline__ void add(float x) {  // pallas_ops.py:195-199
    float t = __fadd_rn(hi, x);
    float e = __fadd_rn(__fsub_rn(hi, t), x);
    lo = __fadd_rn(lo, e);
    hi = t;
  }
};

// One block of groups: groups g in [0, n_groups), group g uses left slice
// a0 + g and right slices b0 .. b0 + n_per - 1; products are consumed in order.
__device__ __forceinline__ TwoSum block_2sum(const float* __restrict__ P, int64_t& p,
                                             int64_t plane, int n_groups, int a0, int n_per,
                                             int b0, const int32_t* __restrict__ eA,
                                             const int32_t* __restrict__ eB, int64_t N, int64_t M,
                                             int64_t r, int64_t c) {
  TwoSum blk{0.0f, 0.0f};
  for (int g = 0; g < n_groups; ++g) {
    TwoSum in{0.0f, 0.0f};
    for (int j = 0; j < n_per; ++j) {
      float cs = pow2f(eB[(int64_t)(b0 + j) * M + c]);
      in.add(__fmul_rn(P[p * plane], cs));
      ++p;
    }
    float rs = pow2f(eA[(int64_t)(a0 + g) * N + r]);
    blk.add(__fmul_rn(in.hi, rs));
    blk.add(__fmul_rn(in.lo, rs));
  }
  return blk;
}

__global__ void k_accumulate_2sum(const float* __restrict__ products, const int32_t* __restrict__ eA,
                                  const int32_t* __restrict__ eB, int64_t N, int64_t M, int n_hi,
                                  int n_lo, float* C_hi, float* C_lo, double* C, int64_t ldc) {
  const int64_t plane = N * M;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < plane;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = idx / M, c = idx % M;
    const float* P = products + idx;
    int64_t p = 0;
    // hi x hi, hi x lo, lo x hi (pallas_gemm_accum.py:26-87 order)
    TwoSum hh = block_2sum(P, p, plane, n_hi, 0, n_hi, 0, eA, eB, N, M, r, c);
    TwoSum hl = block_2sum(P, p, plane, n_lo > 0 ? n_hi : 0, 0, n_lo, n_hi, eA, eB, N, M, r, c);
    TwoSum lh = block_2sum(P, p, plane, n_lo, n_hi, n_hi, 0, eA, eB, N, M, r, c);
    TwoSum out{0.0f, 0.0f};
    out.add(hh.hi);
    out.add(hl.hi);
    out.add(lh.hi);
    out.add(hh.lo);
    out.add(hl.lo);
    out.add(lh.lo);
    if (C_hi) C_hi[idx] = out.hi;
    if (C_lo) C_lo[idx] = out.lo;
    if (C) C[r * ldc + c] = __dadd_rn((double)out.hi, (double)out.lo);
  }
}

// The general form of the reference's accumulate_2sum (pallas_ops.py:178-239,
// :372-396): caller-given FP32 scales and block/group structure.  Block b
// holds groups [block_end[b-1], block_end[b]); group g consumes group_size[g]
// products in order, each times its column scale, then both words times the
// group's row scale.
struct GroupSpec {
  int16_t size[OZK_MAX_PAIRS];
  int16_t block_end[8];
  int n_groups;
  int n_blocks;
};

__global__ void k_accumulate_2sum_scaled(const float* __restrict__ products,
                                         const float* __restrict__ col_scales,
                                         const float* __restrict__ row_scales,
                                         const __grid_constant__ GroupSpec spec, int64_t N,
                                         int64_t M, float* C_hi, float* C_lo) {
  const int64_t plane = N * M;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < plane;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = idx / M, c = idx % M;
    int64_t p = 0;
    int g = 0;
    float blo[8];
    TwoSum out{0.0f, 0.0f};
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      blo[b] = 0.0f;
      if (b >= spec.n_blocks) continue;
      TwoSum blk{0.0f, 0.0f};
      for (; g < spec.block_end[b]; ++g) {
        TwoSum in{0.0f, 0.0f};
        for (int j = 0; j < spec.size[g]; ++j, ++p)
          in.add(__fmul_rn(products[p * plane + idx], col_scales[p * M + c]));
        const float rs = row_scales[(int64_t)g * N + r];
        blk.add(__fmul_rn(in.hi, rs));
        blk.add(__fmul_rn(in.lo, rs));
      }
      out.add(blk.hi);  // block hi words in block order ...
      blo[b] = blk.lo;
    }
#pragma unroll
    for (int b = 0; b < 8; ++b)  // ... then the lo words
      if (b < spec.n_blocks) out.add(blo[b]);
    if (C_hi) C_hi[idx] = out.hi;
    if (C_lo) C_lo[idx] = out.lo;
  }
}

int launch_accumulate_2sum_scaled(const float* products, const float* col_scales,
                                  const float* row_scales, const int32_t* group_sizes,
                                  int n_groups, const int32_t* block_ends, int n_blocks, int64_t N,
                                  int64_t M, float* C_hi, float* C_lo, cudaStream_t stream) {
  if (n_groups < 1 || n_groups > OZK_MAX_PAIRS || n_blocks < 1 || n_blocks > 8)
    return set_error(OZK_ERR_ARG, "accumulate_2sum: 1..%d groups in 1..8 blocks", OZK_MAX_PAIRS);
  GroupSpec spec;
  int prev = 0;
  for (int b = 0; b < n_blocks; ++b) {
    if (block_ends[b] < prev || block_ends[b] > n_groups)
      return set_error(OZK_ERR_ARG, "accumulate_2sum: bad block boundaries");
    spec.block_end[b] = (int16_t)(prev = block_ends[b]);
  }
  if (prev != n_groups) return set_error(OZK_ERR_ARG, "accumulate_2sum: blocks do not cover the groups");
  for (int g = 0; g < n_groups; ++g) {
    if (group_sizes[g] < 0 || group_sizes[g] > OZK_MAX_PAIRS)
      return set_error(OZK_ERR_ARG, "accumulate_2sum: bad group size");
    spec.size[g] = (int16_t)group_sizes[g];
  }
  spec.n_groups = n_groups;
  spec.n_blocks = n_blocks;
  const int64_t plane = N * M;
  if (plane == 0) return OZK_OK;
  int dev;
  cudaGetDevice(&dev);
  int64_t blocks = (plane + 255) / 256;
  int64_t cap = (int64_t)device_sm_count(dev) * 8;
  k_accumulate_2sum_scaled<<<(unsigned)(blocks < cap ? blocks : cap), 256, 0, stream>>>(
      products, col_scales, row_scales, spec, N, M, C_hi, C_lo);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? OZK_OK : set_cuda_error("k_accumulate_2sum_scaled launch", e);
}

int launch_accumulate_2sum(const float* products, const int32_t* eA, const int32_t* eB, int64_t N,
                           int64_t M, int n_hi, int n_lo, float* C_hi, float* C_lo, double* C,
                           int64_t ldc, cudaStream_t stream) {
  const int64_t plane = N * M;
  if (plane == 0) return OZK_OK;
  int dev;
  cudaGetDevice(&dev);
  int64_t blocks = (plane + 255) / 256;
  int64_t cap = (int64_t)device_sm_count(dev) * 8;
  k_accumulate_2sum<<<(unsigned)(blocks < cap ? blocks : cap), 256, 0, stream>>>(
      products, eA, eB, N, M, n_hi, n_lo, C_hi, C_lo, C, ldc);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? OZK_OK : set_cuda_error("k_accumulate_2sum launch", e);
}

}  // namespace ozk
