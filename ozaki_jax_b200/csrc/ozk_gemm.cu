// K2: persistent slice-pair GEMM on the 5th-generation tensor cores.
//
// One CTA per SM walks output tiles (128 rows x BN columns); for each tile it
// walks the pair list in order and, per pair, the K dimension in 64-deep
// stages.  Warp roles:
//   warp 0      TMA producer: stages A-slice and B-slice tiles (128-byte
//               swizzle, K-major) into a STAGES-deep shared-memory ring.
//   warp 1      MMA issuer: one elected thread issues tcgen05.mma
//               (BF16 x BF16 -> FP32, M = 128, N = BN, K = 16) into one of two
//               TMEM accumulators, so pair p+1 computes while the epilogue
//               drains pair p; it also owns the TMEM allocation.
//   warps 2..5  epilogue: TMEM lane quadrant (warp % 4), one output row per
//               thread.  Per pair it reads the exact FP32 product, scales it by
//               2^(eA[a][row] + eB[b][col]) and adds it to an FP64 running sum
//               kept in TMEM (two 32-bit planes), so per-pair products never
//               touch HBM.  After the last pair the FP64 sum goes to C.
// Products are exact (every partial sum is an integer multiple of the slice
// grid below 2^24), so the tensor-core result does not depend on summation
// order; the FP64 epilogue replaces the reference's FP32 2Sum (same
// accuracy class, no FP32 overflow).
//
// TMEM columns: [0, BN) and [BN, 2BN) accumulators, [2BN, 3BN) low words and
// [3BN, 4BN) high words of the FP64 sum.
//
// Every wait is bounded (mbar_wait); on a timeout the CTA stops issuing work,
// waits for its own copies and MMAs in flight, frees TMEM and exits with
// OZK_FLAG_TIMEOUT raised.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <stdint.h>
#include <string.h>

#include "ozk_device.cuh"
#include "ozk_internal.h"

namespace ozk {

constexpr int kBM = 128;
constexpr int kThreads = 192;

struct PairList {
  uint8_t a[OZK_MAX_PAIRS];
  uint8_t b[OZK_MAX_PAIRS];
  int n;
};

struct GemmArgs {
  const int32_t* eA;
  const int32_t* eB;
  int64_t N, M;
  int num_kb;
  int nB;
  int tiles_m, tiles_n, num_tiles, group_m;
  int mode, symmetric;
  double alpha, beta;
  const double* Cin;
  int64_t ldcin;
  double* C;
  int64_t ldc;
  float* products;
  int32_t* status;
  uint64_t budget_ns;
};

template <int BN>
struct GemmCfg {
  static constexpr int STAGES = BN >= 64 ? 6 : 8;
  static constexpr int A_BYTES = kBM * OZK_KB * 2;
  static constexpr int B_BYTES = BN * OZK_KB * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TMEM_COLS = 4 * BN < 32 ? 32 : 4 * BN;
  static constexpr int CH = BN < 32 ? BN : 32;  // epilogue column chunk
  static constexpr int EB_BYTES = OZK_MAX_SLICES * BN * 4;
  static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + EB_BYTES + 256;
};

// Output tile of a linear tile index: group-of-rows raster for L2 reuse, or
// the upper triangle (tm <= tn) in column order when symmetric.
__device__ __forceinline__ void tile_coords(const GemmArgs& g, int t, int& tm, int& tn) {
  if (g.symmetric) {
    int c = (int)((sqrtf(8.0f * (float)t + 1.0f) - 1.0f) * 0.5f);
    while ((c + 1) * (c + 2) / 2 <= t) ++c;
    while (c * (c + 1) / 2 > t) --c;
    tn = c;
    tm = t - c * (c + 1) / 2;
    return;
  }
  int per_group = g.group_m * g.tiles_n;
  int grp = t / per_group;
  int first = grp * g.group_m;
  int gsz = g.tiles_m - first < g.group_m ? g.tiles_m - first : g.group_m;
  int r = t - grp * per_group;
  tm = first + r % gsz;
  tn = r / gsz;
}

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    k_slice_gemm(const __grid_constant__ CUtensorMap mapA, const __grid_constant__ CUtensorMap mapB,
                 const __grid_constant__ PairList pairs, const __grid_constant__ GemmArgs g) {
  using Cfg = GemmCfg<BN>;
  constexpr int STAGES = Cfg::STAGES;
  constexpr int CH = Cfg::CH;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * Cfg::A_BYTES;
  int32_t* s_eB = (int32_t*)(smem + STAGES * Cfg::STAGE_BYTES);
  uint64_t* bars = (uint64_t*)(smem + STAGES * Cfg::STAGE_BYTES + Cfg::EB_BYTES);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* accf = bars + 2 * STAGES;
  uint64_t* acce = accf + 2;
  uint64_t* mma_done = acce + 2;
  uint32_t* s_tmem = (uint32_t*)(mma_done + 1);
  volatile int* s_abort = (volatile int*)(s_tmem + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&accf[i], 1);
      mbar_init(&acce[i], 4);
    }
    mbar_init(mma_done, 1);
    *s_abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(s_tmem, Cfg::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;
  const int npairs = pairs.n;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&mapA);
      tma_prefetch_desc(&mapB);
      uint32_t it = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < g.num_tiles; t += gridDim.x) {
        int tm, tn;
        tile_coords(g, t, tm, tn);
        for (int p = 0; ok && p < npairs; ++p) {
          const int a = pairs.a[p], b = pairs.b[p];
          for (int kb = 0; kb < g.num_kb; ++kb) {
            const uint32_t s = it % STAGES, ph = (it / STAGES) & 1;
            if (!mbar_wait(&empty[s], ph ^ 1, s_abort, g.status, g.budget_ns)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&full[s], Cfg::STAGE_BYTES);
            tma_load_3d(sA + s * Cfg::A_BYTES, &mapA, &full[s], kb * OZK_KB, tm * kBM, a);
            tma_load_3d(sB + s * Cfg::B_BYTES, &mapB, &full[s], kb * OZK_KB, tn * BN, b);
            ++it;
          }
        }
      }
      // Drain: every issued copy must land before shared memory is released.
      uint32_t first = it > (uint32_t)STAGES ? it - STAGES : 0;
      for (uint32_t j = first; j < it; ++j)
        mbar_wait(&full[j % STAGES], (j / STAGES) & 1, nullptr, g.status, g.budget_ns);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16(kBM, BN);
      uint32_t it = 0, acc_it = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < g.num_tiles; t += gridDim.x) {
        for (int p = 0; ok && p < npairs; ++p) {
          const uint32_t buf = acc_it & 1, aph = (acc_it >> 1) & 1;
          if (!mbar_wait(&acce[buf], aph ^ 1, s_abort, g.status, g.budget_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem + buf * BN;
          for (int kb = 0; kb < g.num_kb; ++kb) {
            const uint32_t s = it % STAGES, ph = (it / STAGES) & 1;
            if (!mbar_wait(&full[s], ph, s_abort, g.status, g.budget_ns)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a0 = smem_u32(sA + s * Cfg::A_BYTES);
            const uint32_t b0 = smem_u32(sB + s * Cfg::B_BYTES);
#pragma unroll
            for (int kk = 0; kk < OZK_KB / 16; ++kk)
              umma_bf16(d, umma_desc_sw128(a0 + kk * 32), umma_desc_sw128(b0 + kk * 32), idesc,
                        (kb | kk) != 0);
            umma_commit(&empty[s]);
            ++it;
          }
          if (!ok) break;
          umma_commit(&accf[buf]);
          ++acc_it;
        }
      }
      // All MMAs issued by this thread complete before TMEM is released.
      umma_commit(mma_done);
      mbar_wait(mma_done, 0, nullptr, g.status, g.budget_ns);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;                 // TMEM lane quadrant of this warp
    const int etid = threadIdx.x - 64;      // 0..127 among epilogue threads
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    uint32_t acc_it = 0;
    bool ok = true;
    for (int t = blockIdx.x; ok && t < g.num_tiles; t += gridDim.x) {
      int tm, tn;
      tile_coords(g, t, tm, tn);
      const int64_t col0 = (int64_t)tn * BN;
      named_bar(1, 128);
      for (int e = etid; e < g.nB * BN; e += 128) {
        int64_t c = col0 + (e % BN);
        s_eB[e] = c < g.M ? g.eB[(int64_t)(e / BN) * g.M + c] : 0;
      }
      named_bar(1, 128);
      const int64_t row = (int64_t)tm * kBM + q * 32 + lane;
      const bool rvalid = row < g.N;
      for (int p = 0; p < npairs; ++p) {
        const uint32_t buf = acc_it & 1, aph = (acc_it >> 1) & 1;
        int got = 1;
        if (lane == 0) got = mbar_wait(&accf[buf], aph, s_abort, g.status, g.budget_ns);
        got = __shfl_sync(0xffffffffu, got, 0);
        if (!got) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int a = pairs.a[p], b = pairs.b[p];
        const int ea = rvalid ? g.eA[(int64_t)a * g.N + row] : 0;
        const bool first = (p == 0), last = (p == npairs - 1);
        const uint32_t t_acc = tmem + lane_base + buf * BN;
        const uint32_t t_lo = tmem + lane_base + 2 * BN;
        const uint32_t t_hi = tmem + lane_base + 3 * BN;
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += CH) {
          uint32_t P[CH], L[CH], H[CH];
          if constexpr (CH == 32) {
            tmem_ld32(t_acc + c0, P);
            if (g.mode == OZK_ACC_F64 && !first) {
              tmem_ld32(t_lo + c0, L);
              tmem_ld32(t_hi + c0, H);
            }
          } else {
            tmem_ld16(t_acc + c0, P);
            if (g.mode == OZK_ACC_F64 && !first) {
              tmem_ld16(t_lo + c0, L);
              tmem_ld16(t_hi + c0, H);
            }
          }
          tmem_wait_ld();
          if (g.mode == OZK_ACC_PRODUCTS) {
            if (rvalid) {
              float* dst = g.products + ((int64_t)p * g.N + row) * g.M + col0 + c0;
#pragma unroll
              for (int j = 0; j < CH; ++j)
                if (col0 + c0 + j < g.M) dst[j] = __uint_as_float(P[j]);
            }
            continue;
          }
#pragma unroll
          for (int j = 0; j < CH; ++j) {
            double acc;
            if (first) {
              acc = 0.0;
              if (g.beta != 0.0 && rvalid && col0 + c0 + j < g.M)
                acc = g.beta * g.Cin[row * g.ldcin + col0 + c0 + j];
            } else {
              acc = __hiloint2double((int)H[j], (int)L[j]);
            }
            const int eb = s_eB[b * BN + c0 + j];
            const double pj = (double)__uint_as_float(P[j]);
            if (ea + eb >= -1022 && ea + eb <= 1023)
              acc = fma(pj, g.alpha * __longlong_as_double((long long)(ea + eb + 1023) << 52), acc);
            else  // outside the normal range: scale in two exact steps
              acc = fma(pj * pow2d(ea), g.alpha * pow2d(eb), acc);
            if (last) {
              L[j] = (uint32_t)__double2loint(acc);
              H[j] = (uint32_t)__double2hiint(acc);
              if (rvalid && col0 + c0 + j < g.M) {
                const int64_t col = col0 + c0 + j;
                if (!g.symmetric) {
                  g.C[row * g.ldc + col] = acc;
                } else if (tm != tn || col >= row) {
                  g.C[row * g.ldc + col] = acc;
                  g.C[col * g.ldc + row] = acc;
                }
              }
            } else {
              L[j] = (uint32_t)__double2loint(acc);
              H[j] = (uint32_t)__double2hiint(acc);
            }
          }
          if (!last) {
            if constexpr (CH == 32) {
              tmem_st32(t_lo + c0, L);
              tmem_st32(t_hi + c0, H);
            } else {
              tmem_st16(t_lo + c0, L);
              tmem_st16(t_hi + c0, H);
            }
          }
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acce[buf]);
        ++acc_it;
      }
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::TMEM_COLS);
  }
}

// ---------------------------------------------------------------- host side

static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

static int get_encode_fn() {
  if (g_encode) return OZK_OK;
  cudaDriverEntryPointQueryResult q;
  void* fn = nullptr;
  cudaError_t e = cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000,
                                                   cudaEnableDefault, &q);
  if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
    return set_error(OZK_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  g_encode = (PFN_cuTensorMapEncodeTiled_v12000)fn;
  return OZK_OK;
}

// Tensor map over a [depth][rows][k_pad] BF16 slice stack, box 64 x box_rows.
static int make_slice_map(CUtensorMap* map, const uint16_t* base, int64_t k_pad, int64_t rows,
                          int depth, int box_rows) {
  if (((uintptr_t)base & 15) != 0) return set_error(OZK_ERR_ARG, "slice buffer not 16-byte aligned");
  cuuint64_t dims[3] = {(cuuint64_t)k_pad, (cuuint64_t)rows, (cuuint64_t)depth};
  cuuint64_t strides[2] = {(cuuint64_t)(k_pad * 2), (cuuint64_t)(k_pad * 2 * rows)};
  cuuint32_t box[3] = {OZK_KB, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, (void*)base, dims, strides, box,
                        estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(OZK_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return OZK_OK;
}

template <int BN>
static int launch_bn(const CUtensorMap& ma, const CUtensorMap& mb, const PairList& pl,
                     const GemmArgs& ga, int dev, cudaStream_t stream) {
  using Cfg = GemmCfg<BN>;
  static int configured[64] = {0};
  if (!configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(k_slice_gemm<BN>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         Cfg::SMEM_BYTES);
    if (e != cudaSuccess) return set_cuda_error("cudaFuncSetAttribute(k_slice_gemm)", e);
    configured[dev] = 1;
  }
  int sms = device_sm_count(dev);
  int grid = ga.num_tiles < sms ? ga.num_tiles : sms;
  k_slice_gemm<BN><<<grid, kThreads, Cfg::SMEM_BYTES, stream>>>(ma, mb, pl, ga);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? OZK_OK : set_cuda_error("k_slice_gemm launch", e);
}

int launch_slice_gemm(const uint16_t* SA, const int32_t* eA, int nA, const uint16_t* SB,
                      const int32_t* eB, int nB, int64_t N, int64_t M, int64_t k_pad,
                      const uint8_t* pair_a, const uint8_t* pair_b, int n_pairs, int mode,
                      int symmetric, double alpha, double beta, const double* Cin, int64_t ldcin,
                      double* C, int64_t ldc, float* products, int32_t* status,
                      cudaStream_t stream) {
  if (N == 0 || M == 0) return OZK_OK;
  if (n_pairs < 1 || n_pairs > OZK_MAX_PAIRS) return set_error(OZK_ERR_ARG, "n_pairs out of range");
  if (k_pad <= 0 || k_pad % OZK_KB) return set_error(OZK_ERR_ARG, "k_pad must be a positive multiple of 64");
  if (nA < 1 || nA > OZK_MAX_SLICES || nB < 1 || nB > OZK_MAX_SLICES)
    return set_error(OZK_ERR_ARG, "slice counts out of range");
  for (int p = 0; p < n_pairs; ++p)
    if (pair_a[p] >= nA || pair_b[p] >= nB) return set_error(OZK_ERR_ARG, "pair index out of range");
  if (mode != OZK_ACC_F64 && mode != OZK_ACC_PRODUCTS) return set_error(OZK_ERR_ARG, "bad mode");
  if (mode == OZK_ACC_F64 && !C) return set_error(OZK_ERR_ARG, "C is NULL");
  if (mode == OZK_ACC_PRODUCTS && !products) return set_error(OZK_ERR_ARG, "products is NULL");
  if (beta != 0.0 && !Cin) return set_error(OZK_ERR_ARG, "Cin is NULL with beta != 0");
  if (symmetric && (N != M || SA != SB || eA != eB || mode != OZK_ACC_F64))
    return set_error(OZK_ERR_ARG, "symmetric mode needs one operand, N == M and FP64 output");
  if (N > (int64_t)1 << 31 || M > (int64_t)1 << 31) return set_error(OZK_ERR_ARG, "dimension too large");
  int rc = get_encode_fn();
  if (rc) return rc;
  int dev;
  cudaGetDevice(&dev);

  // Narrow outputs (e.g. residual right-hand sides) use a narrow tile.
  const int BN = M <= 16 ? 16 : (M <= 32 ? 32 : (M <= 64 ? 64 : 128));
  const int bn = symmetric ? 128 : BN;
  CUtensorMap ma, mb;
  if ((rc = make_slice_map(&ma, SA, k_pad, N, nA, kBM))) return rc;
  if ((rc = make_slice_map(&mb, SB, k_pad, M, nB, bn))) return rc;

  PairList pl;
  memset(&pl, 0, sizeof(pl));
  for (int p = 0; p < n_pairs; ++p) {
    pl.a[p] = pair_a[p];
    pl.b[p] = pair_b[p];
  }
  pl.n = n_pairs;
  GemmArgs ga;
  memset(&ga, 0, sizeof(ga));
  ga.eA = eA;
  ga.eB = eB;
  ga.N = N;
  ga.M = M;
  ga.num_kb = (int)(k_pad / OZK_KB);
  ga.nB = nB;
  ga.tiles_m = (int)((N + kBM - 1) / kBM);
  ga.tiles_n = (int)((M + bn - 1) / bn);
  ga.num_tiles = symmetric ? ga.tiles_m * (ga.tiles_m + 1) / 2 : ga.tiles_m * ga.tiles_n;
  ga.group_m = 8;
  ga.mode = mode;
  ga.symmetric = symmetric;
  ga.alpha = alpha;
  ga.beta = beta;
  ga.Cin = Cin;
  ga.ldcin = ldcin;
  ga.C = C;
  ga.ldc = ldc;
  ga.products = products;
  ga.status = status;
  ga.budget_ns = wait_budget_ns();
  switch (bn) {
    case 16: return launch_bn<16>(ma, mb, pl, ga, dev, stream);
    case 32: return launch_bn<32>(ma, mb, pl, ga, dev, stream);
    case 64: return launch_bn<64>(ma, mb, pl, ga, dev, stream);
    default: return launch_bn<128>(ma, mb, pl, ga, dev, stream);
  }
}

}  // namespace ozk
