// K1: FP64 -> double-FP32 split -> sigma-trick BF16 slices, per row (left
// operand) or per column (right operand, written transposed so both GEMM
// operands are K-major).  Bit-identical to the reference's
// f32_extract_split_rows / _cols applied to _double_f32_split
// (ozaki_jax/extract.py:116-191, ozaki_jax/matmul.py:197-213).
//
// Per slice t of a line (row or column) the recurrence is
//   m = max |r|;  c = floor(RN32 log2 m) (0 if m == 0);
//   sigma = RN32(0.75 * 2^(rho + c));  v = RN32(RN32(r + sigma) - sigma) (0 if m == 0);
//   r = RN32(r - v);  slice = RN32(v * 2^-c)  (exactly a BF16 value).
// Every FP32 step uses an explicit _rn intrinsic, so nothing is contracted.
//
// The maximum of slice t depends on slice t-1 over the whole line, so a line
// is swept max(n_hi, n_lo) + 1 times: pass t recomputes the residual from the
// FP64 input (an L2 hit after the first, DRAM-bound pass) and reduces its
// maximum; the last pass emits every slice.  The FP64 input is read from DRAM
// once when a block's lines stay resident in L2, which the launch shapes
// below are sized for.
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdlib.h>

#include "ozk_device.cuh"
#include "ozk_internal.h"
#include "ozk_log2_table.h"

namespace ozk {

__constant__ uint32_t c_log2_thr[OZK_LOG2_TABLE_LEN];
__constant__ unsigned long long c_log2_thr64[OZK_LOG2_TABLE64_LEN];

// floor(RN64(log2 m)) for finite m > 0 (ozaki_jax/extract.py:37, :82); an
// infinite or NaN m (a flagged line) gives 1024, and m = 0 (a zero line,
// which callers handle before asking) -1075, without reading outside the table.
__device__ __forceinline__ int floor_log2_rn64(double m) {
  unsigned long long b = (unsigned long long)__double_as_longlong(m);
  int ex = (int)(b >> 52);
  int e = ex > 0 ? ex - 1023 : -1074 + (63 - __clzll((long long)b));
  if (e > 1023) return 1024;
  if (e < -1074) return -1075;
  return e + (b >= c_log2_thr64[e + 1074] ? 1 : 0);
}

struct SliceState {
  float sig[OZK_MAX_SIDE];
  float inv[OZK_MAX_SIDE];
  int zero[OZK_MAX_SIDE];
};

// Residual of the hi (or lo) part after the first `t` slices.
__device__ __forceinline__ float residual_after(float r, int t, const SliceState& s) {
  for (int i = 0; i < t; ++i) {
    float v = s.zero[i] ? 0.0f : __fsub_rn(__fadd_rn(r, s.sig[i]), s.sig[i]);
    r = __fsub_rn(r, v);
  }
  return r;
}

__device__ __forceinline__ void split_f64(double x, float& hi, float& lo) {
  hi = __double2float_rn(x);
  lo = __double2float_rn(__dsub_rn(x, (double)hi));
}

__device__ __forceinline__ int32_t check_value(double x, float hi) {
  int32_t f = 0;
  if (!isfinite(x)) f |= OZK_FLAG_NONFINITE;
  else if (!isfinite(hi)) f |= OZK_FLAG_RANGE;
  return f;
}

// Slice parameters from a line maximum (extract.py:125-137).
__device__ __forceinline__ void slice_params(float m, int rho, float& sig, float& inv, int& zero,
                                             int& c) {
  zero = (m == 0.0f);
  c = zero ? 0 : floor_log2_rn32(m, c_log2_thr);
  sig = __fmul_rn(0.75f, pow2f(rho + c));
  inv = pow2f(-c);
}

// ---------------------------------------------------------------- rows

template <int NT>
__global__ void __launch_bounds__(NT) k_extract_rows(const double* __restrict__ X, int64_t ldx,
                                                     int64_t rows, int64_t K, int rho, int n_hi,
                                                     int n_lo, uint16_t* __restrict__ slices,
                                                     int64_t k_pad, int32_t* __restrict__ exps,
                                                     int32_t* status) {
  __shared__ SliceState s_hi, s_lo;
  __shared__ float s_red[2][NT / 32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int npass = n_hi > n_lo ? n_hi : n_lo;
  const int64_t slice_stride = rows * k_pad;

  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const double* x = X + row * ldx;
    int32_t flags = 0;
    for (int t = 0; t < npass; ++t) {
      float mh = 0.0f, ml = 0.0f;
      for (int64_t k = tid; k < K; k += NT) {
        double xv = __ldg(x + k);
        float hi, lo;
        split_f64(xv, hi, lo);
        if (t == 0) flags |= check_value(xv, hi);
        if (t < n_hi) mh = fmaxf(mh, fabsf(residual_after(hi, t, s_hi)));
        if (t < n_lo) ml = fmaxf(ml, fabsf(residual_after(lo, t, s_lo)));
      }
      for (int o = 16; o; o >>= 1) {
        mh = fmaxf(mh, __shfl_xor_sync(0xffffffffu, mh, o));
        ml = fmaxf(ml, __shfl_xor_sync(0xffffffffu, ml, o));
      }
      if (lane == 0) {
        s_red[0][warp] = mh;
        s_red[1][warp] = ml;
      }
      __syncthreads();
      if (tid == 0) {
        for (int w = 1; w < NT / 32; ++w) {
          mh = fmaxf(mh, s_red[0][w]);
          ml = fmaxf(ml, s_red[1][w]);
        }
        int c;
        if (t < n_hi) {
          slice_params(mh, rho, s_hi.sig[t], s_hi.inv[t], s_hi.zero[t], c);
          exps[(int64_t)t * rows + row] = c;
        }
        if (t < n_lo) {
          slice_params(ml, rho, s_lo.sig[t], s_lo.inv[t], s_lo.zero[t], c);
          exps[(int64_t)(n_hi + t) * rows + row] = c;
        }
      }
      __syncthreads();
    }
    if (flags) raise_flag(status, flags);
    // Emit pass: two columns per thread per step, written as one 32-bit word.
    uint16_t* out = slices + row * k_pad;
    for (int64_t k = 2 * tid; k < k_pad; k += 2 * NT) {
      uint32_t wh[OZK_MAX_SIDE], wl[OZK_MAX_SIDE];
#pragma unroll
      for (int i = 0; i < OZK_MAX_SIDE; ++i) wh[i] = wl[i] = 0;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        if (k + h < K) {
          float rh, rl;
          split_f64(__ldg(x + k + h), rh, rl);
#pragma unroll
          for (int i = 0; i < OZK_MAX_SIDE; ++i) {
            if (i < n_hi) {
              float v = s_hi.zero[i] ? 0.0f : __fsub_rn(__fadd_rn(rh, s_hi.sig[i]), s_hi.sig[i]);
              rh = __fsub_rn(rh, v);
              wh[i] |= (uint32_t)bf16_bits_exact(__fmul_rn(v, s_hi.inv[i])) << (16 * h);
            }
          }
#pragma unroll
          for (int i = 0; i < OZK_MAX_SIDE; ++i) {
            if (i < n_lo) {
              float v = s_lo.zero[i] ? 0.0f : __fsub_rn(__fadd_rn(rl, s_lo.sig[i]), s_lo.sig[i]);
              rl = __fsub_rn(rl, v);
              wl[i] |= (uint32_t)bf16_bits_exact(__fmul_rn(v, s_lo.inv[i])) << (16 * h);
            }
          }
        }
      }
#pragma unroll
      for (int i = 0; i < OZK_MAX_SIDE; ++i)
        if (i < n_hi) *reinterpret_cast<uint32_t*>(out + i * slice_stride + k) = wh[i];
#pragma unroll
      for (int i = 0; i < OZK_MAX_SIDE; ++i)
        if (i < n_lo) *reinterpret_cast<uint32_t*>(out + (n_hi + i) * slice_stride + k) = wl[i];
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------- rows, register resident

// One line per CTA (or per cluster of CL CTAs that split K), the split FP32
// residuals held in registers: the line is read from DRAM once and every
// slice costs one block (and cluster) max-reduction followed by an in-register
// update that emits the slice (columns K..k_pad-1 are written as zeros).
// Thread `tid` owns the column pairs
// kbase + 2*(p*256 + tid) + {0,1}, p < EPT/2, so the loads are 16-byte vectors
// and the slice stores 4-byte words, both coalesced.  Line maxima are shared
// across the cluster through distributed shared memory.
//
// S8 = true writes each slice as int8 codes q = slice * 2^(24 - rho) instead
// of BF16 bits: every slice is an integer multiple of 2^(rho - 24) of
// magnitude <= 2^(25 - rho), so for rho >= 19 the code is exact and |q| <= 64.
// A value that is not (non-finite slices of out-of-range lines) sets
// *s8_fail; the caller then recomputes with BF16 slices.  With `gate`
// non-NULL the kernel runs only when *gate != 0 (the BF16 recomputation).
constexpr int kRegNT = 256;

__device__ __forceinline__ uint32_t s8_code(float v, float inv, float scale, bool& bad) {
  const float q = __fmul_rn(__fmul_rn(v, inv), scale);
  const int iq = __float2int_rn(q);
  if (!(fabsf(q) <= 127.0f) || (float)iq != q) bad = true;
  return (uint32_t)(uint8_t)(int8_t)iq;
}

template <int EPT, int CL, bool S8>
__global__ void __launch_bounds__(kRegNT, 2) k_extract_rows_reg(
    const double* __restrict__ X, int64_t ldx, int64_t rows, int64_t K, int rho, int n_hi,
    int n_lo, void* __restrict__ slices_v, int64_t k_pad, int32_t* __restrict__ exps,
    int32_t* status, int vec, int32_t* s8_fail, const int32_t* gate) {
  static_assert(EPT % 2 == 0, "EPT must be even");
  if (gate && *(volatile const int32_t*)gate == 0) return;  // uniform over the grid
  const float s8_scale = pow2f(24 - rho);
  bool s8_bad = false;
  __shared__ float s_part[2][2][kRegNT / 32];  // [parity][hi, lo][warp]
  __shared__ float s_cta[2][2];                // [parity][hi, lo] CTA maxima for the cluster
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t crank = CL > 1 ? cluster_ctarank() : 0;
  const int64_t kbase = (int64_t)crank * kRegNT * EPT;
  const int npass = n_hi > n_lo ? n_hi : n_lo;
  const int64_t slice_stride = rows * k_pad;
  uint32_t g = 0;  // running slice counter: parity of the reduction buffers

  for (int64_t row = blockIdx.x / CL; row < rows; row += gridDim.x / CL) {
    const double* x = X + row * ldx;
    float rh[EPT], rl[EPT];
    int32_t flags = 0;
#pragma unroll
    for (int p = 0; p < EPT / 2; ++p) {
      const int64_t k = kbase + 2 * ((int64_t)p * kRegNT + tid);
      double x0 = 0.0, x1 = 0.0;
      if (vec && k + 1 < K) {
        double2 v2 = __ldg(reinterpret_cast<const double2*>(x + k));
        x0 = v2.x;
        x1 = v2.y;
      } else {
        if (k < K) x0 = __ldg(x + k);
        if (k + 1 < K) x1 = __ldg(x + k + 1);
      }
      split_f64(x0, rh[2 * p], rl[2 * p]);
      split_f64(x1, rh[2 * p + 1], rl[2 * p + 1]);
      flags |= check_value(x0, rh[2 * p]) | check_value(x1, rh[2 * p + 1]);
    }
    if (flags) raise_flag(status, flags);

    for (int t = 0; t < npass; ++t, ++g) {
      const int par = g & 1;
      const bool do_hi = t < n_hi, do_lo = t < n_lo;
      float mh = 0.0f, ml = 0.0f;
#pragma unroll
      for (int e = 0; e < EPT; ++e) {
        mh = fmaxf(mh, fabsf(rh[e]));
        ml = fmaxf(ml, fabsf(rl[e]));
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) {
        mh = fmaxf(mh, __shfl_xor_sync(0xffffffffu, mh, o));
        ml = fmaxf(ml, __shfl_xor_sync(0xffffffffu, ml, o));
      }
      if (lane == 0) {
        s_part[par][0][warp] = mh;
        s_part[par][1][warp] = ml;
      }
      __syncthreads();
#pragma unroll
      for (int w = 0; w < kRegNT / 32; ++w) {
        mh = fmaxf(mh, s_part[par][0][w]);
        ml = fmaxf(ml, s_part[par][1][w]);
      }
      if constexpr (CL > 1) {
        if (tid == 0) {
          s_cta[par][0] = mh;
          s_cta[par][1] = ml;
        }
        cluster_sync();
        for (uint32_t r = 0; r < (uint32_t)CL; ++r) {
          mh = fmaxf(mh, ld_dsmem_f32(&s_cta[par][0], r));
          ml = fmaxf(ml, ld_dsmem_f32(&s_cta[par][1], r));
        }
      }
      float sh = 0.f, ih = 0.f, sl = 0.f, il = 0.f;
      int zh = 1, zl = 1, ch = 0, cl = 0;
      if (do_hi) slice_params(mh, rho, sh, ih, zh, ch);
      if (do_lo) slice_params(ml, rho, sl, il, zl, cl);
      if (crank == 0 && tid == 0) {
        if (do_hi) exps[(int64_t)t * rows + row] = ch;
        if (do_lo) exps[(int64_t)(n_hi + t) * rows + row] = cl;
      }
      // Element offsets of this row in the hi and lo slices (BF16: 2 bytes,
      // S8: 1 byte per element).
      const int64_t off_h = (int64_t)t * slice_stride + row * k_pad;
      const int64_t off_l = (int64_t)(n_hi + t) * slice_stride + row * k_pad;
#pragma unroll
      for (int p = 0; p < EPT / 2; ++p) {
        const int64_t k = kbase + 2 * ((int64_t)p * kRegNT + tid);
#pragma unroll
        for (int side = 0; side < 2; ++side) {
          if (side == 0 ? !do_hi : !do_lo) continue;
          const float sg = side == 0 ? sh : sl, iv = side == 0 ? ih : il;
          const int zz = side == 0 ? zh : zl;
          uint32_t w = 0;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            float& r = side == 0 ? rh[2 * p + h] : rl[2 * p + h];
            float v = zz ? 0.0f : __fsub_rn(__fadd_rn(r, sg), sg);
            r = __fsub_rn(r, v);
            if (k + h < K) {
              if constexpr (S8) w |= s8_code(v, iv, s8_scale, s8_bad) << (8 * h);
              else w |= (uint32_t)bf16_bits_exact(__fmul_rn(v, iv)) << (16 * h);
            }
          }
          const int64_t off = (side == 0 ? off_h : off_l) + k;
          if (k < k_pad) {
            if constexpr (S8) reinterpret_cast<uint16_t*>(static_cast<int8_t*>(slices_v) + off)[0] = (uint16_t)w;
            else *reinterpret_cast<uint32_t*>(static_cast<uint16_t*>(slices_v) + off) = w;
          }
        }
      }
    }
  }
  if constexpr (S8) {
    if (s8_bad) *s8_fail = 1;
  }
  if constexpr (CL > 1) cluster_sync();  // peers may still read this CTA's s_cta
}

// ---------------------------------------------------------------- rows, staged by bulk copies

// Rows of 1024 < K <= 65536 FP64 values (even K, 16-byte aligned rows): a
// persistent CTA of NT threads (or a cluster of CL CTAs, each owning NT*EPT
// columns) walks rows blockIdx.x / CL, += gridDim.x / CL.  A row arrives in
// shared memory through bulk copies, is moved into registers (EPT columns per
// thread, in groups of four adjacent columns) and split, and the buffer is
// refilled with the CTA's next row at once, so its DRAM transfer overlaps the
// slice passes of this one; several CTAs per SM keep several rows in flight.
//
// A slice pass is one CTA barrier: each warp posts its partial line maxima,
// and after the barrier every warp reduces all partials of the line and
// derives the slice parameters itself, then sweeps its registers, taking the
// next pass's maxima on the way.  In a cluster each partial is one 64-bit word
// (pass << 32) | FP32 bits, which the warp stores into the inbox of every CTA
// of the cluster (remote stores, not waited for); a reader polls its own CTA's
// inbox until the tag matches (a bounded spin), so the CTAs need no cluster
// barrier per pass and no poll crosses the cluster.  Two parity slots
// suffice: a warp posts its pass-g+1 partial only after reading every pass-g
// partial, so no CTA can reach pass g+2, and rewrite a slot, before every warp
// of every CTA has read that slot's pass-g value.  Slices are
// written as 8-byte (BF16) or 4-byte (int8) words, all columns up to k_pad
// included; int8 codes are staged in shared memory (two buffers per side), and
// one thread bulk-stores a pass's codes after the next barrier, which takes
// the address arithmetic and most store instructions off the sweeps.
//
// int8 codes: with the slice exponent c of a line in [-127, 127 - rho] (and
// the line finite), t = RN32(r + sigma) lies in [2^(rho+c-1), 2^(rho+c)), a
// binade whose spacing 2^(rho+c-24) is the grid of v = t - sigma, with
// |v| <= 2^(c+1).  So the code q = v * 2^(24-rho-c), an integer with
// |q| <= 2^(25-rho) <= 64, is the difference of the bit patterns of t and
// sigma.  Lines outside that range (or holding NaN/Inf or values beyond the
// FP32 range) set *s8_fail instead, once per line.
constexpr uint32_t kBulkChunk = 16384;  // bytes per bulk copy instruction

template <bool S8, int CL>
constexpr bool kStageCodes = S8;

// Dynamic shared memory of k_extract_rows_bulk: the row buffer, then (staged
// codes) 2 buffers x 2 sides of NT*EPT int8 codes.
template <int NT, int EPT, bool S8, int CL>
inline size_t bulk_smem_bytes(int64_t K) {
  return kStageCodes<S8, CL>
             ? (size_t)NT * EPT * 8 + 4 * (size_t)NT * EPT
             : (size_t)round_up((K < (int64_t)NT * EPT ? K : (int64_t)NT * EPT) * 8, 128);
}

// max(m, |a|, |b|) as one three-input maximum; like fmaxf, a NaN operand is
// ignored in favour of the others.
__device__ __forceinline__ float max3_abs(float m, float a, float b) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(m), "f"(fabsf(a)), "f"(fabsf(b)));
  return d;
}

// max(m, |a|, |b|), NaN if any operand is NaN.
__device__ __forceinline__ float max3_abs_nan(float m, float a, float b) {
  float d;
  asm("max.NaN.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(m), "f"(fabsf(a)), "f"(fabsf(b)));
  return d;
}


// PRESET = 16 n_hi + n_lo fixes the slice counts at compile time (the pass
// loop unrolls, the lo residuals die after their last pass); 0 takes them
// from the arguments.
template <int NT, int EPT, int MINB, bool S8, int CL, int PRESET>
__global__ void __launch_bounds__(NT, MINB) k_extract_rows_bulk(
    const double* __restrict__ X, int64_t ldx, int64_t rows, int64_t K, int rho, int n_hi_arg,
    int n_lo_arg, void* __restrict__ slices_v, int64_t k_pad, int32_t* __restrict__ exps,
    int32_t* status, int32_t* s8_fail, const int32_t* gate, uint64_t budget_ns) {
  const int n_hi = PRESET ? PRESET / 16 : n_hi_arg;
  const int n_lo = PRESET ? PRESET % 16 : n_lo_arg;
  static_assert(EPT % 4 == 0, "EPT must be a multiple of 4");
  constexpr int NG = EPT / 4;
  constexpr int NW = NT / 32;
  constexpr int NP = NW * CL;  // partial maxima of a line: one per warp of the cluster
  static_assert(NP <= 64, "at most two partials per lane");
  constexpr int ESZ = S8 ? 1 : 2;  // bytes per slice element
  constexpr bool STAGE = kStageCodes<S8, CL>;
  constexpr uint32_t kCodeBytes = (uint32_t)NT * EPT;  // int8 codes of one slice of a CTA's columns
  if (gate && *(volatile const int32_t*)gate == 0) return;  // uniform over the grid
  extern __shared__ __align__(128) uint8_t smem_raw[];
  __shared__ uint64_t s_bar;
  __shared__ float s_part[2][2][NW];  // CL == 1: [parity][hi max, lo max][warp]
  // CL > 1: the inbox of every warp's partials in the cluster, [parity][hi, lo]
  // [CTA rank * NW + warp], (pass << 32) | FP32 bits (lo: bit 31 = line flags)
  __shared__ uint64_t s_tag[2][2][CL > 1 ? NP : 1];
  __shared__ int s_abort;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t crank = CL > 1 ? cluster_ctarank() : 0;
  // This CTA's columns of every row: [kbase, kbase + NT*EPT) of [0, K).
  const int64_t kbase = (int64_t)crank * NT * EPT;
  const int64_t kown = K - kbase < (int64_t)NT * EPT ? (K - kbase > 0 ? K - kbase : 0)
                                                      : (int64_t)NT * EPT;
  const uint32_t own_bytes = (uint32_t)(kown * 8);
  const int npass = n_hi > n_lo ? n_hi : n_lo;
  const int64_t slice_stride = rows * k_pad;
  const double* xb = reinterpret_cast<const double*>(smem_raw);
  uint8_t* const s_code = smem_raw + (size_t)NT * EPT * 8;  // STAGE: [buffer][side][kCodeBytes]
  // STAGE: code bytes of a slice this CTA writes, columns [kbase, min(k_pad, kbase + NT*EPT))
  const uint32_t code_bytes =
      (uint32_t)(k_pad - kbase <= 0 ? 0 : (k_pad - kbase < (int64_t)kCodeBytes ? k_pad - kbase : kCodeBytes));
  // groups of this thread that lie inside [0, k_pad): q < nq
  int nq = 0;
  {
    const int64_t left = k_pad - kbase - 4 * (int64_t)tid;
    if (left > 0) nq = (int)((left + 4 * NT - 1) / (4 * NT));
    if (nq > NG) nq = NG;
  }

  if (tid == 0) {
    mbar_init(&s_bar, 1);
    s_abort = 0;
    fence_mbar_init();
  }
  if constexpr (CL > 1)
    for (int i = tid; i < 4 * NP; i += NT) (&s_tag[0][0][0])[i] = ~0ull;  // no pass has tag ~0
  // the tagged slots are initialised before any peer reads them
  if constexpr (CL > 1) cluster_sync();
  else __syncthreads();
  auto issue = [&](int64_t row) {
    const uint8_t* src = reinterpret_cast<const uint8_t*>(X + row * ldx + kbase);
    mbar_arrive_expect_tx(&s_bar, own_bytes);
    for (uint32_t off = 0; off < own_bytes; off += kBulkChunk)
      bulk_load_g2s(smem_raw + off, src + off, min(kBulkChunk, own_bytes - off), &s_bar);
  };
  // STAGE: the codes of the last pass wait in s_code[pend_buf] for thread 0
  // to store them after the next barrier.
  bool pend = false;
  int64_t pend_row = 0;
  int pend_hi = -1, pend_lo = -1;
  uint32_t pend_buf = 0;
  auto flush = [&]() {
    if (code_bytes) {
      uint8_t* dst = static_cast<uint8_t*>(slices_v) + pend_row * k_pad + kbase;
      if (pend_hi >= 0)
        bulk_store_s2g(dst + pend_hi * slice_stride, s_code + (2 * pend_buf) * kCodeBytes, code_bytes);
      if (pend_lo >= 0)
        bulk_store_s2g(dst + pend_lo * slice_stride, s_code + (2 * pend_buf + 1) * kCodeBytes,
                       code_bytes);
    }
    bulk_commit();
  };
  // A cluster's CTAs go through every row together.  If a wait runs out of
  // time the CTA keeps stepping with its peers (so no cluster barrier is left
  // waiting) but issues no more copies; the timeout flag reports the failure.
  const int64_t row0 = blockIdx.x / CL, rstride = gridDim.x / CL;
  uint32_t issued = 0;  // rows whose copy was issued (thread 0's count)
  uint32_t landed = 0;  // rows whose copy was waited for
  bool live = true;     // no wait has run out of time (uniform over the CTA)
  if (tid == 0 && row0 < rows && own_bytes) {
    issue(row0);
    ++issued;
  }
  uint32_t it = 0, par = 0;
  uint32_t gpass = 0;  // passes so far over all rows: the mailbox tag
  for (int64_t row = row0; row < rows; row += rstride, ++it) {
    bool got = true;
    if (live && own_bytes)
      got = mbar_wait(&s_bar, it & 1, (volatile int*)&s_abort, status, budget_ns);
    if (__syncthreads_or(!got)) live = false;
    else if (live && own_bytes) ++landed;
    // residuals in pairs of adjacent columns, for the packed FP32 arithmetic
    float2 rh[EPT / 2], rl[EPT / 2];
    float mh = 0.0f, ml = 0.0f;
#pragma unroll
    for (int q = 0; q < NG; ++q) {
      const int64_t k = 4 * ((int64_t)q * NT + tid);  // within this CTA's columns
      double x[4] = {0.0, 0.0, 0.0, 0.0};
      if (k + 3 < kown) {
        const double2 a2 = *reinterpret_cast<const double2*>(xb + k);
        const double2 b2 = *reinterpret_cast<const double2*>(xb + k + 2);
        x[0] = a2.x, x[1] = a2.y, x[2] = b2.x, x[3] = b2.y;
      } else {
#pragma unroll
        for (int h = 0; h < 4; ++h)
          if (k + h < kown) x[h] = xb[k + h];
      }
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        float2& hi = rh[2 * q + j];
        float2& lo = rl[2 * q + j];
        split_f64(x[2 * j], hi.x, lo.x);
        split_f64(x[2 * j + 1], hi.y, lo.y);
        mh = max3_abs_nan(mh, hi.x, hi.y);  // keeps a NaN, so the check below sees it
        ml = max3_abs(ml, lo.x, lo.y);
      }
    }
    // a non-finite split value: the input is non-finite or beyond FP32.  Such a
    // line is flagged below; its maxima (NaN or inf) give it garbage slices,
    // which the flag keeps from being used.
    const bool odd = !(mh <= 3.402823466e38f);
    int32_t flags = 0;
    if (odd) {  // rare: tell non-finite input from FP32 overflow
#pragma unroll
      for (int q = 0; q < NG; ++q)
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          const int64_t k = 4 * ((int64_t)q * NT + tid) + h;
          const float2 hp = rh[2 * q + (h >> 1)];
          if (k < kown) flags |= check_value(xb[k], (h & 1) ? hp.y : hp.x);
        }
      raise_flag(status, flags);
    }
    // The buffer is free: fetch this CTA's share of its next row while slicing
    // this one.
    const int line_bad = __syncthreads_or(flags);
    if (tid == 0 && live && own_bytes) {
      const int64_t nx = row + rstride;
      if (nx < rows) {
        fence_proxy_async_smem();
        issue(nx);
        ++issued;
      }
    }
#pragma unroll
    for (int t = 0; t < (PRESET ? (PRESET / 16 > PRESET % 16 ? PRESET / 16 : PRESET % 16) : npass);
         ++t, par ^= 1, ++gpass) {
      const bool do_hi = t < n_hi, do_lo = t < n_lo;
      // Partial line maxima of each warp (and, in the first pass, the line's
      // input flags), one barrier, then the line maxima in every warp.  The
      // maxima are >= 0, so their bit patterns order as unsigned integers (a
      // NaN, only in a line already flagged, is the positive canonical NaN):
      // one redux per reduction.
      mh = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(mh)));
      ml = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(ml)));
      bool bad = t == 0 && line_bad;
      float gh = 0.0f, gl = 0.0f;
      if constexpr (CL == 1) {
        if (lane == 0) {
          s_part[par][0][warp] = mh;
          s_part[par][1][warp] = ml;
        }
      } else if (lane < CL) {
        // lane r sends the warp's partials to CTA r's inbox
        const uint64_t tag = (uint64_t)gpass << 32;
        const int slot = (int)crank * NW + warp;
        st_dsmem_relaxed_u64(&s_tag[par][0][slot], lane, tag | __float_as_uint(mh));
        st_dsmem_relaxed_u64(&s_tag[par][1][slot], lane,
                             tag | __float_as_uint(ml) | (bad ? 0x80000000u : 0u));
      }
      if constexpr (STAGE) {
        fence_proxy_async_smem();            // this thread's staged codes, for the bulk store
        if (tid == 0) bulk_wait_read_all();  // the buffer this pass writes is no longer read
      }
      // A CTA barrier, not a cluster one: the tags carry the exchange between
      // CTAs.  A warp posts its pass-g+1 partial only after it has read every
      // pass-g partial, so when any CTA posts pass g+2 into a parity slot, all
      // warps of all peers have read that slot's pass-g value.
      __syncthreads();
      if constexpr (STAGE) {
        if (tid == 0 && pend) flush();
        pend = false;
      }
      if constexpr (CL == 1) {
        if (lane < NW) {
          gh = s_part[par][0][lane];
          gl = s_part[par][1][lane];
        }
      } else {
#pragma unroll
        for (int e0 = 0; e0 < NP; e0 += 32) {
          const int e = e0 + lane;
          if (e < NP) {
            uint32_t vh, vl;
            tag_wait_local(&s_tag[par][0][e], gpass, vh, (volatile int*)&s_abort, status,
                           budget_ns);
            tag_wait_local(&s_tag[par][1][e], gpass, vl, (volatile int*)&s_abort, status,
                           budget_ns);
            gh = fmaxf(gh, __uint_as_float(vh));
            gl = fmaxf(gl, __uint_as_float(vl & 0x7fffffffu));
            bad = bad || (vl >> 31);
          }
        }
        bad = __any_sync(0xffffffffu, bad);
      }
      gh = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(gh)));
      gl = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(gl)));
      float sh = 0.f, ih = 0.f, sl = 0.f, il = 0.f;
      int zh = 1, zl = 1, ch = 0, cl = 0;
      if (do_hi) slice_params(gh, rho, sh, ih, zh, ch);
      if (do_lo) slice_params(gl, rho, sl, il, zl, cl);
      if (tid == 0 && crank == 0) {
        if (S8) {
          if (do_hi && !zh && (ch < -127 || rho + ch > 127)) bad = true;
          if (do_lo && !zl && (cl < -127 || rho + cl > 127)) bad = true;
          if (bad) *s8_fail = 1;
        }
        if (do_hi) exps[(int64_t)t * rows + row] = ch;
        if (do_lo) exps[(int64_t)(n_hi + t) * rows + row] = cl;
      }
      mh = 0.0f;
      ml = 0.0f;
      // A zero line has all residuals 0, so RN(r + sigma) - sigma is 0 there and
      // the zero-line rule needs no select.
#pragma unroll
      for (int side = 0; side < 2; ++side) {
        if (side == 0 ? !do_hi : !do_lo) continue;
        const float sg = side == 0 ? sh : sl, iv = side == 0 ? ih : il;
        const float2 sg2 = make_float2(sg, sg), nsg2 = make_float2(-sg, -sg);
        const float2 iv2 = make_float2(iv, iv), neg1 = make_float2(-1.0f, -1.0f);
        uint8_t* out;
        if constexpr (STAGE)
          out = s_code + (2 * par + side) * kCodeBytes + 4 * tid;
        else
          out = static_cast<uint8_t*>(slices_v) +
                ((int64_t)(side == 0 ? t : n_hi + t) * slice_stride + row * k_pad + kbase +
                 4 * (int64_t)tid) * ESZ;
        float mnext = 0.0f;
#pragma unroll
        for (int q = 0; q < NG; ++q) {
          uint32_t u[4];
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            float2& r = side == 0 ? rh[2 * q + j] : rl[2 * q + j];
            const float2 tt = __fadd2_rn(r, sg2);   // RN(r + sigma)
            const float2 v = __fadd2_rn(tt, nsg2);  // the slice value, exact
            r = __ffma2_rn(v, neg1, r);             // r - v, exact
            mnext = max3_abs(mnext, r.x, r.y);
            if constexpr (S8) {
              // the int8 code bits(t) - bits(sigma) fits in a byte, and sigma =
              // 0.75 * 2^(rho+c) has the mantissa 0x400000, whose low byte is
              // 0: so the code is the low byte of bits(t) itself
              u[2 * j] = __float_as_uint(tt.x);
              u[2 * j + 1] = __float_as_uint(tt.y);
            } else {  // BF16 in the top halves
              const float2 b = __fmul2_rn(v, iv2);
              u[2 * j] = __float_as_uint(b.x);
              u[2 * j + 1] = __float_as_uint(b.y);
            }
          }
          if constexpr (!S8) {
            // columns K..k_pad-1 are zeros even where 2^-c is not finite
            const int64_t k = kbase + 4 * ((int64_t)q * NT + tid);
            if (k + 3 >= K) {
#pragma unroll
              for (int h = 0; h < 4; ++h)
                if (k + h >= K) u[h] = 0;
            }
          }
          if constexpr (S8) {
            const uint32_t w = __byte_perm(__byte_perm(u[0], u[1], 0x0040),
                                           __byte_perm(u[2], u[3], 0x0040), 0x5410);
            // staged: every group (the bulk store takes the first code_bytes)
            if (STAGE || q < nq) *reinterpret_cast<uint32_t*>(out + (int64_t)q * 4 * NT) = w;
          } else if (q < nq) {
            *reinterpret_cast<uint2*>(out + (int64_t)q * 8 * NT) =
                make_uint2(__byte_perm(u[0], u[1], 0x7632), __byte_perm(u[2], u[3], 0x7632));
          }
        }
        if (side == 0) mh = mnext;
        else ml = mnext;
      }
      if constexpr (STAGE) {
        pend = true;
        pend_row = row;
        pend_hi = do_hi ? t : -1;
        pend_lo = do_lo ? n_hi + t : -1;
        pend_buf = par;
      }
    }
  }
  if constexpr (STAGE) {
    // the last pass's codes
    fence_proxy_async_smem();
    __syncthreads();
    if (tid == 0) {
      if (pend) flush();
      bulk_wait_all();
    }
  }
  // Every issued copy lands before the CTA's shared memory is released.
  if (tid == 0) {
    for (uint32_t j = landed; j < issued; ++j)
      mbar_wait(&s_bar, j & 1, nullptr, status, budget_ns);
  }
  __syncthreads();
  if constexpr (CL > 1) cluster_sync();  // no peer reads this CTA's tagged slots any more
}

int upload_log2_table(int dev);  // below: the exponent rule's threshold table

// ---------------------------------------------------------------- lines, one pass per launch

// Line extraction split into one launch per slice pass, for lines whose
// elements live on several GPUs (the multi-GPU gram: a column of A split by
// rows over the ranks).  Launch t (-1 <= t < npass) re-derives every element's
// residual from its FP64 value and the exponents of slices 0..t-1 (exps), then:
//   t >= 0: takes the slice parameters of pass t from the line maxima gmax
//           (the maxima over all ranks' parts of the line, [2][lines]: hi
//           side then lo side), writes exps[t] (and exps[n_hi + t]) and the
//           int8 codes of slice t of this rank's part (hi: slice t if t < n_hi,
//           lo: slice n_hi + t if t < n_lo), columns n..k_pad-1 as zeros;
//   t + 1 < npass: writes the maxima of the residual after pass t over this
//           rank's part, pmax [2][lines], for the next launch (t = -1: of the
//           split values themselves);
//   t == -1: raises OZK_FLAG_NONFINITE / _RANGE for bad values (and *s8_fail).
// The arithmetic is the row kernels' (the same split, sigma, RN sums and
// codes), so the codes of every part are those the whole line would get from
// one GPU once gmax is the whole line's maximum.  One CTA of kLpNT threads per
// line (grid-stride), element e of the part at e = tid, tid + kLpNT, ...
constexpr int kLpNT = 256;

__global__ void __launch_bounds__(kLpNT) k_line_pass_s8(
    const double* __restrict__ X, int64_t ldx, int64_t lines, int64_t n, int t, int npass,
    int rho, int n_hi, int n_lo, const float* __restrict__ gmax, float* __restrict__ pmax,
    int8_t* __restrict__ slices, int64_t k_pad, int32_t* __restrict__ exps, int32_t* status,
    int32_t* s8_fail) {
  __shared__ float s_red[2][kLpNT / 32];
  __shared__ float s_sig[2][8];  // sigma of slices 0..t per side
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t slice_stride = lines * k_pad;
  for (int64_t line = blockIdx.x; line < lines; line += gridDim.x) {
    // sigma of the slices before t from their exponents, of slice t from gmax
    if (tid < 2 * 8) {
      const int side = tid >> 3, s = tid & 7;
      const int ns = side == 0 ? n_hi : n_lo;
      float sg = 0.0f;
      if (s < t && s < ns) {
        const int c = exps[(int64_t)(side == 0 ? s : n_hi + s) * lines + line];
        sg = __fmul_rn(0.75f, pow2f(rho + c));
      } else if (s == t && s < ns) {
        float sig, inv;
        int zero, c;
        slice_params(gmax[side * lines + line], rho, sig, inv, zero, c);
        sg = sig;
        exps[(int64_t)(side == 0 ? s : n_hi + s) * lines + line] = c;
        if (!zero && (c < -127 || rho + c > 127)) *(volatile int32_t*)s8_fail = 1;
      }
      s_sig[side][s] = sg;
    }
    __syncthreads();
    float mh = 0.0f, ml = 0.0f;
    int32_t flags = 0;
    for (int64_t e = tid; e < k_pad; e += kLpNT) {
      if (e >= n) {  // padding columns: code 0
        if (t >= 0) {
          if (t < n_hi) slices[(int64_t)t * slice_stride + line * k_pad + e] = 0;
          if (t < n_lo) slices[(int64_t)(n_hi + t) * slice_stride + line * k_pad + e] = 0;
        }
        continue;
      }
      const double x = X[line * ldx + e];
      float r[2];
      split_f64(x, r[0], r[1]);
      if (t < 0) {
        if (!(fabsf(r[0]) <= 3.402823466e38f)) flags |= check_value(x, r[0]);
      }
#pragma unroll
      for (int side = 0; side < 2; ++side) {
        const int ns = side == 0 ? n_hi : n_lo;
        for (int s = 0; s <= t && s < ns; ++s) {
          const float sg = s_sig[side][s];
          const float tt = __fadd_rn(r[side], sg);  // RN(r + sigma)
          const float v = __fadd_rn(tt, -sg);       // the slice value, exact
          r[side] = __fadd_rn(r[side], -v);         // exact
          if (s == t)
            slices[(int64_t)(side == 0 ? t : n_hi + t) * slice_stride + line * k_pad + e] =
                (int8_t)(__float_as_uint(tt) - __float_as_uint(sg));
        }
      }
      mh = fmaxf(mh, fabsf(r[0]));
      ml = fmaxf(ml, fabsf(r[1]));
    }
    if (t < 0 && flags) {
      raise_flag(status, flags);
      *(volatile int32_t*)s8_fail = 1;
    }
    if (t + 1 < npass) {
      // the line's maxima are >= 0 and never NaN here (fmaxf skips NaN), so
      // their bit patterns order as unsigned integers
      mh = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(mh)));
      ml = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(ml)));
      if (lane == 0) {
        s_red[0][warp] = mh;
        s_red[1][warp] = ml;
      }
      __syncthreads();
      if (tid < 2) {
        float m = 0.0f;
#pragma unroll
        for (int w = 0; w < kLpNT / 32; ++w) m = fmaxf(m, s_red[tid][w]);
        pmax[tid * lines + line] = m;
      }
    }
    __syncthreads();  // s_sig and s_red are rewritten for the next line
  }
}

int launch_line_pass_s8(const double* X, int64_t ldx, int64_t lines, int64_t n, int t, int npass,
                        int rho, int n_hi, int n_lo, const float* gmax, float* pmax,
                        int8_t* slices, int64_t k_pad, int32_t* exps, int32_t* status,
                        int32_t* s8_fail, cudaStream_t stream) {
  if (lines == 0) return OZK_OK;
  if (n_hi > 8 || n_lo > 8) return set_error(OZK_ERR_ARG, "at most 8 slices per side");
  int dev;
  cudaGetDevice(&dev);
  int rc = upload_log2_table(dev);
  if (rc) return rc;
  int64_t grid = lines < 65535 ? lines : 65535;
  k_line_pass_s8<<<(unsigned)grid, kLpNT, 0, stream>>>(X, ldx, lines, n, t, npass, rho, n_hi,
                                                      n_lo, gmax, pmax, slices, k_pad, exps,
                                                      status, s8_fail);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? OZK_OK : set_cuda_error("k_line_pass_s8 launch", e);
}

// ---------------------------------------------------------------- transpose

// XT (cols x rows, leading dimension rows) = X^T for X (rows x cols, ldx):
// 32 x 32 tiles through shared memory, both sides coalesced.
__global__ void __launch_bounds__(256) k_transpose_f64(const double* __restrict__ X, int64_t ldx,
                                                       int64_t rows, int64_t cols,
                                                       double* __restrict__ XT) {
  __shared__ double tile[32][33];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  for (int64_t tr = blockIdx.y; tr * 32 < rows; tr += gridDim.y) {
    for (int64_t tc = blockIdx.x; tc * 32 < cols; tc += gridDim.x) {
      const int64_t r0 = tr * 32, c0 = tc * 32;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        int64_t r = r0 + ty + 8 * i, c = c0 + tx;
        if (r < rows && c < cols) tile[ty + 8 * i][tx] = __ldg(X + r * ldx + c);
      }
      __syncthreads();
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        int64_t c = c0 + ty + 8 * i, r = r0 + tx;
        if (r < rows && c < cols) XT[c * rows + r] = tile[tx][ty + 8 * i];
      }
      __syncthreads();
    }
  }
}

// ---------------------------------------------------------------- columns

// A block owns 32 adjacent columns (lane = column) and all K rows; its 8
// warps split the rows.  The emit pass stages 64 rows x 32 columns per slice
// in shared memory and writes them transposed, 128 bytes per column.
constexpr int kColW = 32;
constexpr int kColNT = 256;
constexpr int kColChunk = 64;

__global__ void __launch_bounds__(kColNT) k_extract_cols(const double* __restrict__ X, int64_t ldx,
                                                         int64_t K, int64_t cols, int rho,
                                                         int n_hi, int n_lo,
                                                         uint16_t* __restrict__ slices,
                                                         int64_t k_pad, int32_t* __restrict__ exps,
                                                         int32_t* status) {
  __shared__ float s_sig[2][OZK_MAX_SIDE][kColW];
  __shared__ float s_inv[2][OZK_MAX_SIDE][kColW];
  __shared__ int s_zero[2][OZK_MAX_SIDE][kColW];
  __shared__ float s_red[2][kColNT / 32][kColW];
  // [slice][column][k] staging for the transposed write (+2 to spread banks).
  extern __shared__ uint16_t s_tile[];
  constexpr int kRowPitch = kColChunk + 2;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int npass = n_hi > n_lo ? n_hi : n_lo;
  const int ns = n_hi + n_lo;
  const int64_t slice_stride = cols * k_pad;

  for (int64_t c0 = (int64_t)blockIdx.x * kColW; c0 < cols; c0 += (int64_t)gridDim.x * kColW) {
    const int64_t col = c0 + lane;
    const bool valid = col < cols;
    int32_t flags = 0;
    for (int t = 0; t < npass; ++t) {
      float mh = 0.0f, ml = 0.0f;
      if (valid) {
        for (int64_t k = warp; k < K; k += kColNT / 32) {
          double xv = __ldg(X + k * ldx + col);
          float hi, lo;
          split_f64(xv, hi, lo);
          if (t == 0) flags |= check_value(xv, hi);
          float rh = hi, rl = lo;
          for (int i = 0; i < t; ++i) {
            if (i < n_hi) {
              float sg = s_sig[0][i][lane];
              float v = s_zero[0][i][lane] ? 0.0f : __fsub_rn(__fadd_rn(rh, sg), sg);
              rh = __fsub_rn(rh, v);
            }
            if (i < n_lo) {
              float sg = s_sig[1][i][lane];
              float v = s_zero[1][i][lane] ? 0.0f : __fsub_rn(__fadd_rn(rl, sg), sg);
              rl = __fsub_rn(rl, v);
            }
          }
          if (t < n_hi) mh = fmaxf(mh, fabsf(rh));
          if (t < n_lo) ml = fmaxf(ml, fabsf(rl));
        }
      }
      s_red[0][warp][lane] = mh;
      s_red[1][warp][lane] = ml;
      __syncthreads();
      if (warp == 0) {
        for (int w = 1; w < kColNT / 32; ++w) {
          mh = fmaxf(mh, s_red[0][w][lane]);
          ml = fmaxf(ml, s_red[1][w][lane]);
        }
        int c;
        if (t < n_hi) {
          slice_params(mh, rho, s_sig[0][t][lane], s_inv[0][t][lane], s_zero[0][t][lane], c);
          if (valid) exps[(int64_t)t * cols + col] = c;
        }
        if (t < n_lo) {
          slice_params(ml, rho, s_sig[1][t][lane], s_inv[1][t][lane], s_zero[1][t][lane], c);
          if (valid) exps[(int64_t)(n_hi + t) * cols + col] = c;
        }
      }
      __syncthreads();
    }
    if (flags) raise_flag(status, flags);

    for (int64_t k0 = 0; k0 < k_pad; k0 += kColChunk) {
      // compute: each thread handles rows k0 + warp + 8*j of its column
      for (int j = 0; j < kColChunk / (kColNT / 32); ++j) {
        int kk = warp + j * (kColNT / 32);
        int64_t k = k0 + kk;
        float rh = 0.0f, rl = 0.0f;
        bool live = valid && k < K;
        if (live) split_f64(__ldg(X + k * ldx + col), rh, rl);
        for (int i = 0; i < n_hi; ++i) {
          float v = 0.0f;
          if (live) {
            float sg = s_sig[0][i][lane];
            v = s_zero[0][i][lane] ? 0.0f : __fsub_rn(__fadd_rn(rh, sg), sg);
            rh = __fsub_rn(rh, v);
            v = __fmul_rn(v, s_inv[0][i][lane]);
          }
          s_tile[(i * kColW + lane) * kRowPitch + kk] = bf16_bits_exact(v);
        }
        for (int i = 0; i < n_lo; ++i) {
          float v = 0.0f;
          if (live) {
            float sg = s_sig[1][i][lane];
            v = s_zero[1][i][lane] ? 0.0f : __fsub_rn(__fadd_rn(rl, sg), sg);
            rl = __fsub_rn(rl, v);
            v = __fmul_rn(v, s_inv[1][i][lane]);
          }
          s_tile[((n_hi + i) * kColW + lane) * kRowPitch + kk] = bf16_bits_exact(v);
        }
      }
      __syncthreads();
      // write: per slice, 32 columns x 64 k; a thread writes 4 consecutive k.
      for (int e = tid; e < ns * kColW * (kColChunk / 4); e += kColNT) {
        int q = e % (kColChunk / 4);
        int cl = (e / (kColChunk / 4)) % kColW;
        int s = e / ((kColChunk / 4) * kColW);
        int64_t cc = c0 + cl;
        if (cc < cols) {
          const uint16_t* src = &s_tile[(s * kColW + cl) * kRowPitch + 4 * q];
          uint2 w;
          w.x = (uint32_t)src[0] | ((uint32_t)src[1] << 16);
          w.y = (uint32_t)src[2] | ((uint32_t)src[3] << 16);
          *reinterpret_cast<uint2*>(slices + s * slice_stride + cc * k_pad + k0 + 4 * q) = w;
        }
      }
      __syncthreads();
    }
  }
}

// ---------------------------------------------------------------- FP64 (host pipeline)

// The host pipeline's extraction (extract_split_rows / _cols,
// ozaki_jax/extract.py:21-103): the same recurrence on the FP64 input itself,
// in FP64, n_slices slices; each normalised slice is rounded to FP32 storage
// by the reference and is exactly a BF16 value (at most 54 - rho <= 8 bits).
struct SliceState64 {
  double sig[OZK_MAX_SLICES];
  double inv[OZK_MAX_SLICES];
  int zero[OZK_MAX_SLICES];
};

__device__ __forceinline__ void slice_params64(double m, int rho, double& sig, double& inv,
                                               int& zero, int& c) {
  zero = (m == 0.0);
  c = zero ? 0 : floor_log2_rn64(m);
  sig = __dmul_rn(0.75, pow2d(rho + c));
  inv = pow2d(-c);
}

__device__ __forceinline__ uint16_t slice_bits64(double v, double inv) {
  return bf16_bits_exact(__double2float_rn(__dmul_rn(v, inv)));
}

template <int NT>
__global__ void __launch_bounds__(NT) k_extract_rows64(const double* __restrict__ X, int64_t ldx,
                                                       int64_t rows, int64_t K, int rho, int ns,
                                                       uint16_t* __restrict__ slices,
                                                       int64_t k_pad, int32_t* __restrict__ exps,
                                                       int32_t* status) {
  __shared__ SliceState64 st;
  __shared__ double s_red[NT / 32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t slice_stride = rows * k_pad;
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const double* x = X + row * ldx;
    int32_t flags = 0;
    for (int t = 0; t < ns; ++t) {
      double m = 0.0;
      for (int64_t k = tid; k < K; k += NT) {
        double r = __ldg(x + k);
        if (t == 0 && !isfinite(r)) flags |= OZK_FLAG_NONFINITE;
        for (int i = 0; i < t; ++i) {
          double v = st.zero[i] ? 0.0 : __dsub_rn(__dadd_rn(r, st.sig[i]), st.sig[i]);
          r = __dsub_rn(r, v);
        }
        m = fmax(m, fabs(r));
      }
      for (int o = 16; o; o >>= 1) m = fmax(m, __shfl_xor_sync(0xffffffffu, m, o));
      if (lane == 0) s_red[warp] = m;
      __syncthreads();
      if (tid == 0) {
        for (int w = 1; w < NT / 32; ++w) m = fmax(m, s_red[w]);
        int c;
        slice_params64(m, rho, st.sig[t], st.inv[t], st.zero[t], c);
        exps[(int64_t)t * rows + row] = c;
      }
      __syncthreads();
    }
    if (flags) raise_flag(status, flags);
    uint16_t* out = slices + row * k_pad;
    for (int64_t k = 2 * tid; k < k_pad; k += 2 * NT) {
      uint32_t w[OZK_MAX_SLICES];
#pragma unroll
      for (int i = 0; i < OZK_MAX_SLICES; ++i) w[i] = 0;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        if (k + h < K) {
          double r = __ldg(x + k + h);
#pragma unroll
          for (int i = 0; i < OZK_MAX_SLICES; ++i) {
            if (i < ns) {
              double v = st.zero[i] ? 0.0 : __dsub_rn(__dadd_rn(r, st.sig[i]), st.sig[i]);
              r = __dsub_rn(r, v);
              w[i] |= (uint32_t)slice_bits64(v, st.inv[i]) << (16 * h);
            }
          }
        }
      }
#pragma unroll
      for (int i = 0; i < OZK_MAX_SLICES; ++i)
        if (i < ns) *reinterpret_cast<uint32_t*>(out + i * slice_stride + k) = w[i];
    }
    __syncthreads();
  }
}

__global__ void __launch_bounds__(kColNT) k_extract_cols64(const double* __restrict__ X,
                                                           int64_t ldx, int64_t K, int64_t cols,
                                                           int rho, int ns,
                                                           uint16_t* __restrict__ slices,
                                                           int64_t k_pad,
                                                           int32_t* __restrict__ exps,
                                                           int32_t* status) {
  __shared__ double s_sig[OZK_MAX_SLICES][kColW];
  __shared__ double s_inv[OZK_MAX_SLICES][kColW];
  __shared__ int s_zero[OZK_MAX_SLICES][kColW];
  __shared__ double s_red[kColNT / 32][kColW];
  extern __shared__ uint16_t s_tile[];
  constexpr int kRowPitch = kColChunk + 2;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t slice_stride = cols * k_pad;

  for (int64_t c0 = (int64_t)blockIdx.x * kColW; c0 < cols; c0 += (int64_t)gridDim.x * kColW) {
    const int64_t col = c0 + lane;
    const bool valid = col < cols;
    int32_t flags = 0;
    for (int t = 0; t < ns; ++t) {
      double m = 0.0;
      if (valid) {
        for (int64_t k = warp; k < K; k += kColNT / 32) {
          double r = __ldg(X + k * ldx + col);
          if (t == 0 && !isfinite(r)) flags |= OZK_FLAG_NONFINITE;
          for (int i = 0; i < t; ++i) {
            double sg = s_sig[i][lane];
            double v = s_zero[i][lane] ? 0.0 : __dsub_rn(__dadd_rn(r, sg), sg);
            r = __dsub_rn(r, v);
          }
          m = fmax(m, fabs(r));
        }
      }
      s_red[warp][lane] = m;
      __syncthreads();
      if (warp == 0) {
        for (int w = 1; w < kColNT / 32; ++w) m = fmax(m, s_red[w][lane]);
        int c;
        slice_params64(m, rho, s_sig[t][lane], s_inv[t][lane], s_zero[t][lane], c);
        if (valid) exps[(int64_t)t * cols + col] = c;
      }
      __syncthreads();
    }
    if (flags) raise_flag(status, flags);
    for (int64_t k0 = 0; k0 < k_pad; k0 += kColChunk) {
      for (int j = 0; j < kColChunk / (kColNT / 32); ++j) {
        int kk = warp + j * (kColNT / 32);
        int64_t k = k0 + kk;
        bool live = valid && k < K;
        double r = live ? __ldg(X + k * ldx + col) : 0.0;
        for (int i = 0; i < ns; ++i) {
          uint16_t bits = 0;
          if (live) {
            double sg = s_sig[i][lane];
            double v = s_zero[i][lane] ? 0.0 : __dsub_rn(__dadd_rn(r, sg), sg);
            r = __dsub_rn(r, v);
            bits = slice_bits64(v, s_inv[i][lane]);
          }
          s_tile[(i * kColW + lane) * kRowPitch + kk] = bits;
        }
      }
      __syncthreads();
      for (int e = tid; e < ns * kColW * (kColChunk / 4); e += kColNT) {
        int q = e % (kColChunk / 4);
        int cl = (e / (kColChunk / 4)) % kColW;
        int s = e / ((kColChunk / 4) * kColW);
        int64_t cc = c0 + cl;
        if (cc < cols) {
          const uint16_t* src = &s_tile[(s * kColW + cl) * kRowPitch + 4 * q];
          uint2 w;
          w.x = (uint32_t)src[0] | ((uint32_t)src[1] << 16);
          w.y = (uint32_t)src[2] | ((uint32_t)src[3] << 16);
          *reinterpret_cast<uint2*>(slices + s * slice_stride + cc * k_pad + k0 + 4 * q) = w;
        }
      }
      __syncthreads();
    }
  }
}

// ---------------------------------------------------------------- host side

static int g_table_uploaded[64] = {0};

int upload_log2_table(int dev) {
  if (dev < 0 || dev >= 64) return OZK_ERR_ARG;
  if (g_table_uploaded[dev]) return OZK_OK;
  cudaError_t e = cudaMemcpyToSymbol(c_log2_thr, kOzkLog2ThreshHost, sizeof(kOzkLog2ThreshHost));
  if (e == cudaSuccess)
    e = cudaMemcpyToSymbol(c_log2_thr64, kOzkLog2Thresh64Host, sizeof(kOzkLog2Thresh64Host));
  if (e != cudaSuccess) return set_cuda_error("cudaMemcpyToSymbol(log2 table)", e);
  g_table_uploaded[dev] = 1;
  return OZK_OK;
}

template <int EPT, int CL, bool S8 = false>
static int launch_rows_reg(const double* X, int64_t ldx, int64_t rows, int64_t K, int rho, int n_hi,
                           int n_lo, void* slices, int64_t k_pad, int32_t* exps,
                           int32_t* status, int dev, cudaStream_t stream,
                           int32_t* s8_fail = nullptr, const int32_t* gate = nullptr) {
  const int vec = (((uintptr_t)X & 15) == 0) && (ldx % 2 == 0);
  // Enough lines in flight per SM to cover the reduction latencies.
  int64_t per_sm = EPT <= 8 ? 8 : (EPT <= 16 ? 6 : 3);
  int64_t clusters = (int64_t)device_sm_count(dev) * per_sm / CL;
  if (clusters > rows) clusters = rows;
  if (clusters < 1) clusters = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(clusters * CL));
  cfg.blockDim = dim3(kRegNT);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = CL;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, k_extract_rows_reg<EPT, CL, S8>, X, ldx, rows, K, rho,
                                     n_hi, n_lo, slices, k_pad, exps, status, vec, s8_fail, gate);
  return e == cudaSuccess ? OZK_OK : set_cuda_error("k_extract_rows_reg launch", e);
}

template <int NT, int EPT, int MINB, bool S8, int CL = 1, int PRESET = 0>
static int launch_rows_bulk_p(const double* X, int64_t ldx, int64_t rows, int64_t K, int rho,
                              int n_hi, int n_lo, void* slices, int64_t k_pad, int32_t* exps,
                              int32_t* status, int32_t* s8_fail, const int32_t* gate, int dev,
                              cudaStream_t stream) {
  const size_t kMaxSmem = bulk_smem_bytes<NT, EPT, S8, CL>((int64_t)NT * EPT);
  auto kern = k_extract_rows_bulk<NT, EPT, MINB, S8, CL, PRESET>;
  static int configured[64] = {0};
  if (!configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)kMaxSmem);
    if (e != cudaSuccess) return set_cuda_error("cudaFuncSetAttribute(k_extract_rows_bulk)", e);
    if (CL > 1) cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    configured[dev] = 1;
  }
  // CTA r of a cluster stages columns [r*NT*EPT, (r+1)*NT*EPT) of a row
  const size_t smem = bulk_smem_bytes<NT, EPT, S8, CL>(K);
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, NT, smem) != cudaSuccess ||
      per_sm < 1)
    per_sm = 1;
  int64_t clusters = (int64_t)device_sm_count(dev) * per_sm / CL;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(clusters * CL));
  cfg.blockDim = dim3(NT);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = CL;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (CL > 1) {
    // Only as many clusters as are resident at once: a GPC need not hold a
    // whole number of them, and a second wave of clusters would double the
    // time of the persistent row loop.
    static int fit[64] = {0};
    if (!fit[dev]) {
      int n = 0;
      fit[dev] = (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) == cudaSuccess && n > 0) ? n : -1;
      cudaGetLastError();
    }
    if (fit[dev] > 0 && fit[dev] < clusters) clusters = fit[dev];
  }
  if (clusters > rows) clusters = rows;
  if (clusters < 1) clusters = 1;
  cfg.gridDim = dim3((unsigned)(clusters * CL));
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, X, ldx, rows, K, rho, n_hi, n_lo, slices, k_pad,
                                     exps, status, s8_fail, gate, wait_budget_ns());
  return e == cudaSuccess ? OZK_OK : set_cuda_error("k_extract_rows_bulk launch", e);
}

// The presets 'high' (4, 1) and 'medium' (3, 1) get kernels with the slice
// counts fixed at compile time; other counts take them at run time.
template <int NT, int EPT, int MINB, bool S8, int CL = 1>
static int launch_rows_bulk(const double* X, int64_t ldx, int64_t rows, int64_t K, int rho,
                            int n_hi, int n_lo, void* slices, int64_t k_pad, int32_t* exps,
                            int32_t* status, int32_t* s8_fail, const int32_t* gate, int dev,
                            cudaStream_t stream) {
  // (not for clustered BF16 lines, the gated recomputation: there the
  // unrolled passes would spill)
  if constexpr (S8 || CL == 1) {
    if (n_hi == 4 && n_lo == 1)
      return launch_rows_bulk_p<NT, EPT, MINB, S8, CL, 0x41>(X, ldx, rows, K, rho, n_hi, n_lo,
                                                             slices, k_pad, exps, status, s8_fail,
                                                             gate, dev, stream);
    if (n_hi == 3 && n_lo == 1)
      return launch_rows_bulk_p<NT, EPT, MINB, S8, CL, 0x31>(X, ldx, rows, K, rho, n_hi, n_lo,
                                                             slices, k_pad, exps, status, s8_fail,
                                                             gate, dev, stream);
  }
  return launch_rows_bulk_p<NT, EPT, MINB, S8, CL, 0>(X, ldx, rows, K, rho, n_hi, n_lo, slices,
                                                      k_pad, exps, status, s8_fail, gate, dev,
                                                      stream);
}

// The bulk-staged kernel serves rows of 1024 < K, k_pad <= 65536 with even K
// and ldx and a 16-byte aligned base (OZK_EXTRACT_BULK=0 turns it off).
static bool bulk_rows_ok(const double* X, int64_t ldx, int64_t K, int64_t k_pad) {
  static int on = -1;
  if (on < 0) {
    const char* e = getenv("OZK_EXTRACT_BULK");
    on = (e && e[0] == '0') ? 0 : 1;
  }
  return on && K > 1024 && k_pad <= 65536 && K % 2 == 0 && ldx % 2 == 0 &&
         ((uintptr_t)X & 15) == 0;
}

template <bool S8>
static int launch_rows_bulk_any(const double* X, int64_t ldx, int64_t rows, int64_t K, int rho,
                                int n_hi, int n_lo, void* slices, int64_t k_pad, int32_t* exps,
                                int32_t* status, int32_t* s8_fail, const int32_t* gate, int dev,
                                cudaStream_t stream) {
  // 256-thread CTAs, several per SM (each with one row in flight), up to
  // 8192 columns; 512 threads (one CTA per SM) beyond.
  if (k_pad <= 2048)
    return launch_rows_bulk<256, 8, 4, S8>(X, ldx, rows, K, rho, n_hi, n_lo, slices, k_pad, exps,
                                           status, s8_fail, gate, dev, stream);
  if (k_pad <= 4096)
    return launch_rows_bulk<256, 16, 3, S8>(X, ldx, rows, K, rho, n_hi, n_lo, slices, k_pad, exps,
                                            status, s8_fail, gate, dev, stream);
  if (k_pad <= 8192)
    return launch_rows_bulk<256, 32, 2, S8>(X, ldx, rows, K, rho, n_hi, n_lo, slices, k_pad, exps,
                                            status, s8_fail, gate, dev, stream);
  if (k_pad <= 12288)
    return launch_rows_bulk<512, 24, 1, S8>(X, ldx, rows, K, rho, n_hi, n_lo, slices, k_pad, exps,
                                            status, s8_fail, gate, dev, stream);
  // Longer rows: a cluster of CTAs per row, line maxima exchanged through
  // distributed shared memory.  Up to 32768 columns, CTAs of 128 threads
  // holding 4096 columns each (four CTAs of different rows per SM); longer,
  // 256 threads and 8192 columns (two per SM), so the cluster stays at 8.
  if (k_pad <= 16384)
    return launch_rows_bulk<128, 32, 4, S8, 4>(X, ldx, rows, K, rho, n_hi, n_lo, slices, k_pad,
                                               exps, status, s8_fail, gate, dev, stream);
  if (k_pad <= 32768)
    return launch_rows_bulk<128, 32, 4, S8, 8>(X, ldx, rows, K, rho, n_hi, n_lo, slices, k_pad,
                                               exps, status, s8_fail, gate, dev, stream);
  return launch_rows_bulk<256, 32, 2, S8, 8>(X, ldx, rows, K, rho, n_hi, n_lo, slices, k_pad,
                                             exps, status, s8_fail, gate, dev, stream);
}

int launch_extract_rows_s8(const double* X, int64_t ldx, int64_t rows, int64_t K, int rho,
                           int n_hi, int n_lo, int8_t* slices, int64_t k_pad, int32_t* exps,
                           int32_t* status, int32_t* s8_fail, cudaStream_t stream) {
  if (rows == 0) return OZK_OK;
  if (rho < kS8MinRho || k_pad % kS8KB || k_pad > 65536)
    return set_error(OZK_ERR_UNSUPPORTED, "int8 slices need rho >= %d and k_pad <= 65536, a multiple of %d",
                     kS8MinRho, kS8KB);
  if (!s8_fail) return set_error(OZK_ERR_ARG, "s8_fail is NULL");
  int dev;
  cudaGetDevice(&dev);
  int rc = upload_log2_table(dev);
  if (rc) return rc;
  // (bulk stores of the codes: 16-byte aligned rows)
  if (bulk_rows_ok(X, ldx, K, k_pad) && ((uintptr_t)slices & 15) == 0)
    return launch_rows_bulk_any<true>(X, ldx, rows, K, rho, n_hi, n_lo, slices, k_pad, exps,
                                      status, s8_fail, nullptr, dev, stream);
  // rho >= 19 means K > 4096, so 8192-column CTAs (and clusters for longer lines)
  if (k_pad <= 8192)
    return launch_rows_reg<32, 1, true>(X, ldx, rows, K, rho, n_hi, n_lo, slices, k_pad, exps, status, dev, stream, s8_fail);
  if (k_pad <= 16384)
    return launch_rows_reg<32, 2, true>(X, ldx, rows, K, rho, n_hi, n_lo, slices, k_pad, exps, status, dev, stream, s8_fail);
  if (k_pad <= 32768)
    return launch_rows_reg<32, 4, true>(X, ldx, rows, K, rho, n_hi, n_lo, slices, k_pad, exps, status, dev, stream, s8_fail);
  return launch_rows_reg<32, 8, true>(X, ldx, rows, K, rho, n_hi, n_lo, slices, k_pad, exps, status, dev, stream, s8_fail);
}

int launch_extract_rows(const double* X, int64_t ldx, int64_t rows, int64_t K, int rho, int n_hi,
                        int n_lo, uint16_t* slices, int64_t k_pad, int32_t* exps, int32_t* status,
                        cudaStream_t stream) {
  return launch_extract_rows_gated(X, ldx, rows, K, rho, n_hi, n_lo, slices, k_pad, exps, status,
                                   nullptr, stream);
}

int launch_extract_rows_gated(const double* X, int64_t ldx, int64_t rows, int64_t K, int rho,
                              int n_hi, int n_lo, uint16_t* slices, int64_t k_pad, int32_t* exps,
                              int32_t* status, const int32_t* gate, cudaStream_t stream) {
  if (rows == 0) return OZK_OK;
  if (gate && k_pad > 65536) return set_error(OZK_ERR_UNSUPPORTED, "gated extraction needs k_pad <= 65536");
  int dev;
  cudaGetDevice(&dev);
  int rc = upload_log2_table(dev);
  if (rc) return rc;
  if (bulk_rows_ok(X, ldx, K, k_pad))
    return launch_rows_bulk_any<false>(X, ldx, rows, K, rho, n_hi, n_lo, slices, k_pad, exps,
                                       status, nullptr, gate, dev, stream);
  // Register-resident path: one CTA covers 256*EPT columns, a cluster of up to
  // 8 CTAs covers k_pad <= 65536.
  if (k_pad <= 512)
    return launch_rows_reg<2, 1>(X, ldx, rows, K, rho, n_hi, n_lo, slices, k_pad, exps, status, dev, stream, nullptr, gate);
  if (k_pad <= 1024)
    return launch_rows_reg<4, 1>(X, ldx, rows, K, rho, n_hi, n_lo, slices, k_pad, exps, status, dev, stream, nullptr, gate);
  if (k_pad <= 2048)
    return launch_rows_reg<8, 1>(X, ldx, rows, K, rho, n_hi, n_lo, slices, k_pad, exps, status, dev, stream, nullptr, gate);
  if (k_pad <= 4096)
    return launch_rows_reg<16, 1>(X, ldx, rows, K, rho, n_hi, n_lo, slices, k_pad, exps, status, dev, stream, nullptr, gate);
  if (k_pad <= 8192)
    return launch_rows_reg<32, 1>(X, ldx, rows, K, rho, n_hi, n_lo, slices, k_pad, exps, status, dev, stream, nullptr, gate);
  if (k_pad <= 16384)
    return launch_rows_reg<32, 2>(X, ldx, rows, K, rho, n_hi, n_lo, slices, k_pad, exps, status, dev, stream, nullptr, gate);
  if (k_pad <= 32768)
    return launch_rows_reg<32, 4>(X, ldx, rows, K, rho, n_hi, n_lo, slices, k_pad, exps, status, dev, stream, nullptr, gate);
  if (k_pad <= 65536)
    return launch_rows_reg<32, 8>(X, ldx, rows, K, rho, n_hi, n_lo, slices, k_pad, exps, status, dev, stream, nullptr, gate);
  // Longer lines: multi-pass kernel (passes 2.. re-read the line from L2).
  int sms = device_sm_count(dev);
  int64_t grid = rows < sms * 2 ? rows : sms * 2;
  k_extract_rows<512><<<(unsigned)grid, 512, 0, stream>>>(X, ldx, rows, K, rho, n_hi, n_lo, slices,
                                                           k_pad, exps, status);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? OZK_OK : set_cuda_error("k_extract_rows launch", e);
}

int launch_transpose_f64(const double* X, int64_t ldx, int64_t rows, int64_t cols, double* XT,
                         cudaStream_t stream) {
  if (rows == 0 || cols == 0) return OZK_OK;
  int64_t gx = (cols + 31) / 32, gy = (rows + 31) / 32;
  if (gx > 65535) gx = 65535;
  if (gy > 65535) gy = 65535;
  k_transpose_f64<<<dim3((unsigned)gx, (unsigned)gy), 256, 0, stream>>>(X, ldx, rows, cols, XT);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? OZK_OK : set_cuda_error("k_transpose_f64 launch", e);
}

int launch_extract_cols(const double* X, int64_t ldx, int64_t K, int64_t cols, int rho, int n_hi,
                        int n_lo, uint16_t* slices, int64_t k_pad, int32_t* exps, int32_t* status,
                        double* scratch, cudaStream_t stream) {
  if (cols == 0) return OZK_OK;
  // Fast path: transpose into the caller's scratch (cols x K FP64), then the
  // register-resident row kernel on the transposed lines.
  if (scratch && k_pad <= 65536) {
    int rc = launch_transpose_f64(X, ldx, K, cols, scratch, stream);
    if (rc) return rc;
    return launch_extract_rows(scratch, K, cols, K, rho, n_hi, n_lo, slices, k_pad, exps, status,
                               stream);
  }
  int dev;
  cudaGetDevice(&dev);
  int rc = upload_log2_table(dev);
  if (rc) return rc;
  size_t smem = (size_t)(n_hi + n_lo) * kColW * (kColChunk + 2) * sizeof(uint16_t);
  static int configured[64] = {0};
  if (!configured[dev]) {
    cudaFuncSetAttribute(k_extract_cols, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024);
    configured[dev] = 1;
  }
  int64_t strips = (cols + kColW - 1) / kColW;
  int sms = device_sm_count(dev);
  int64_t grid = strips < 2 * sms ? strips : 2 * sms;
  k_extract_cols<<<(unsigned)grid, kColNT, smem, stream>>>(X, ldx, K, cols, rho, n_hi, n_lo,
                                                            slices, k_pad, exps, status);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? OZK_OK : set_cuda_error("k_extract_cols launch", e);
}

int launch_extract_cols_s8(const double* X, int64_t ldx, int64_t K, int64_t cols, int rho,
                           int n_hi, int n_lo, int8_t* slices, int64_t k_pad, int32_t* exps,
                           int32_t* status, int32_t* s8_fail, double* scratch,
                           cudaStream_t stream) {
  if (cols == 0) return OZK_OK;
  if (!scratch) return set_error(OZK_ERR_ARG, "int8 column extraction needs the transpose scratch");
  int rc = launch_transpose_f64(X, ldx, K, cols, scratch, stream);
  if (rc) return rc;
  return launch_extract_rows_s8(scratch, K, cols, K, rho, n_hi, n_lo, slices, k_pad, exps, status,
                                s8_fail, stream);
}

int launch_extract_rows64(const double* X, int64_t ldx, int64_t rows, int64_t K, int rho, int ns,
                          uint16_t* slices, int64_t k_pad, int32_t* exps, int32_t* status,
                          cudaStream_t stream) {
  if (rows == 0) return OZK_OK;
  int dev;
  cudaGetDevice(&dev);
  int rc = upload_log2_table(dev);
  if (rc) return rc;
  int sms = device_sm_count(dev);
  int64_t per_sm = K <= 4096 ? 8 : (K <= 16384 ? 4 : 2);
  int64_t grid = rows < sms * per_sm ? rows : sms * per_sm;
  k_extract_rows64<256><<<(unsigned)grid, 256, 0, stream>>>(X, ldx, rows, K, rho, ns, slices,
                                                             k_pad, exps, status);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? OZK_OK : set_cuda_error("k_extract_rows64 launch", e);
}

int launch_extract_cols64(const double* X, int64_t ldx, int64_t K, int64_t cols, int rho, int ns,
                          uint16_t* slices, int64_t k_pad, int32_t* exps, int32_t* status,
                          cudaStream_t stream) {
  if (cols == 0) return OZK_OK;
  int dev;
  cudaGetDevice(&dev);
  int rc = upload_log2_table(dev);
  if (rc) return rc;
  size_t smem = (size_t)ns * kColW * (kColChunk + 2) * sizeof(uint16_t);
  static int configured[64] = {0};
  if (!configured[dev]) {
    cudaFuncSetAttribute(k_extract_cols64, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024);
    configured[dev] = 1;
  }
  int64_t strips = (cols + kColW - 1) / kColW;
  int sms = device_sm_count(dev);
  int64_t grid = strips < 2 * sms ? strips : 2 * sms;
  k_extract_cols64<<<(unsigned)grid, kColNT, smem, stream>>>(X, ldx, K, cols, rho, ns, slices,
                                                              k_pad, exps, status);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? OZK_OK : set_cuda_error("k_extract_cols64 launch", e);
}

}  // namespace ozk
