// Exact fixed-point accumulation of slice-pair products, shared by the slice
// GEMM kernels.
#pragma once

#include <stdint.h>

#include "ozk_device.cuh"

namespace ozk {

// Fixed-point accumulation.  With the top slices' exponents eA0 (row) and
// eB0 (column), every exact slice product P of a pair is an integer number
// of product-grid units g = 2^G (G = 2 (rho - 24)) with |P/g| < 2^26 (the
// preflight bound); scaled by 2^(ea + eb - eA0 - eB0) <= 1 it is summed
// exactly in an int64 whose unit is g * 2^(eA0 + eB0 - kFixFrac).  Terms are
// < 2^62 and only parts below the unit (2^-36 of the top grid) are rounded
// away, so the sum is as accurate as FP64 accumulation and independent of the
// order -- and the per-pair work uses only the integer pipes (FP64 arithmetic
// shares a pipe with the tensor cores on this part).
constexpr int kFixFrac = 36;

// A non-finite product (from non-finite slices of out-of-range inputs, where
// the reference's sums are NaN) marks the element with this value, which a
// real sum never reaches (|terms| < 2^62); it stays set and becomes NaN.
constexpr long long kFixNaN = (long long)0x8000000000000000ull;

// Term of the FP32 product bits u, t_off = (ea - eA0) + (eb - eB0) + fix_off:
// round(P * 2^(ea + eb) / unit).
__device__ __forceinline__ long long fixed_term(uint32_t u, int t_off) {
  const uint32_t ex = (u >> 23) & 0xFFu;
  if (ex == 0xFFu) return kFixNaN;
  const uint32_t m = (u & 0x7FFFFFu) | (ex ? 0x800000u : 0u);  // products are 0 or normal
  const int T = (int)ex + t_off;
  const int L = min(max(T, 0), 40);
  const int R = min(max(-T, 0), 31);
  const uint32_t mr = (m + ((1u << R) >> 1)) >> R;  // round half up
  const long long v = (long long)((unsigned long long)mr << L);
  const long long sg = (long long)((int)u >> 31);  // 0 or -1
  return (v ^ sg) - sg;
}

// The same term from an exact int32 product P of int8 slice codes (the
// product in units of the product grid): round(P * 2^T), half away from zero,
// T = (ea - eA0) + (eb - eB0) + kFixFrac.  It equals fixed_term of the FP32
// product of the corresponding BF16 slices bit for bit (the same real number,
// rounded the same way).
__device__ __forceinline__ long long fixed_term_s32(int32_t P, int T) {
  // T >= 0 (the common case): P * 2^T exactly; a two's-complement shift of P
  // gives the same 64 bits as shifting |P| and restoring the sign
  if (T >= 0) return (long long)((unsigned long long)(long long)P << min(T, 40));
  const unsigned long long a = (unsigned long long)(P < 0 ? -(long long)P : (long long)P);
  const int R = min(-T, 40);
  const unsigned long long v = (a + (1ull << (R - 1))) >> R;
  const long long sg = (long long)(P >> 31);  // 0 or -1
  return ((long long)v ^ sg) - sg;
}

// The FP64 value of a fixed-point sum: acc * 2^e, exact scaling.
__device__ __forceinline__ double fixed_value(long long acc, int e) {
  const double v = __ll2double_rn(acc);
  if (e >= -1022 && e <= 1023) return v * __longlong_as_double((long long)(e + 1023) << 52);
  return (v * pow2d(e / 2)) * pow2d(e - e / 2);
}

}  // namespace ozk
