// Skinny slice GEMM on int8 codes: C = alpha * (A @ X) + beta * Cin for an
// N x K matrix A and at most 16 right-hand sides X (K x M, M <= 16), with
// fixed-point sums (OZK_ACC_FIXED).  This is the shape of the reference's
// residual (_residual_ozaki_jit / _ozaki_matvec_f64, ozaki_jax/solve.py:38-53,
// :78-82: r = b - ozaki(A, x) with x of 16 columns), where reading A dominates.
//
// The wide slice GEMM walks the pair list with the K loop inside, so each A
// slice panel is read once per pair that uses it.  Here every pair product of
// a 128-row tile accumulates at once: the n_pairs accumulators of 128 x 16
// int32 take n_pairs * 16 <= 512 TMEM columns, and each pipeline stage holds
// one 128-element k-block of all nS slices of A and of X, so every A slice is
// read from DRAM exactly once.  The fixed-point combination (exactly the wide
// kernel's, so results are bit-identical to it) runs once per tile.
//
// Warp 0: TMA producer.  Warp 1: TMEM allocation and the MMA issuer (one
// thread, tcgen05.mma.cta_group::1.kind::i8, M = 128, K = 32).  Warps 2-5:
// epilogue, one output row per thread.
//
// The pairs are taken in (A slice, X slice) order, and the pairs of one A
// slice with consecutive X slices form a run: the X slices' 16-row tiles lie
// back to back in shared memory and their accumulators side by side in TMEM,
// so a run is ONE MMA of N = 16 * (run length).  For the preset (4, 1) that
// is 5 MMAs per k-step instead of 24, and each A tile is read from shared
// memory once per run rather than once per pair (at N = 16 the A operand's
// shared-memory reads, not the tensor math, bound an MMA).
//
// K split: when the tiles would leave SMs idle (fewer tiles than SMs, or a
// last wave less than half full), each tile's K range is cut into ksplit
// parts on different CTAs.  A part's int32 pair products are added into the
// tile's slot in a scratch with red.add -- integer adds, so the totals are
// exactly the products of the whole K range -- and the last of the tile's
// parts to arrive runs the fixed-point epilogue on them: bit-identical results.
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "ozk_device.cuh"
#include "ozk_fixed.cuh"
#include "ozk_internal.h"

namespace ozk {
namespace {

constexpr int kSkRows = 128;                 // rows of A per tile (MMA M)
constexpr int kSkCols = 16;                  // right-hand sides (MMA N)
constexpr int kSkMaxSlices = 6;              // nS limit: two stages must fit in shared memory
constexpr int kSkMaxPairs = 512 / kSkCols;   // TMEM columns / accumulator width
constexpr int kSkMaxStages = 4;
constexpr int kSkABytes = kSkRows * kS8KB;   // one slice's k-block of a tile: 16 KB
constexpr int kSkXBytes = kSkCols * kS8KB;   // one slice's k-block of X: 2 KB
constexpr int kSkThreads = 192;

struct SkPairs {
  uint8_t a[kSkMaxPairs];  // pairs sorted by (a, b); pair p accumulates in TMEM columns
  uint8_t b[kSkMaxPairs];  // [16 p, 16 p + 16)
  int n;
  uint8_t run_p0[kSkMaxPairs];   // first pair of each run
  uint8_t run_len[kSkMaxPairs];  // pairs in the run (<= 16: N <= 256)
  int n_runs;
};

struct SkArgs {
  const int32_t* eA;  // [nS][N]
  const int32_t* eX;  // [nS][M]
  int64_t N;
  int M;
  int nS;
  int stages;
  int num_kb;
  int num_tiles;
  double alpha, beta;
  const double* Cin;
  int64_t ldcin;
  double* C;
  int64_t ldc;
  int fix_scale;  // 2 (rho - 24) - kFixFrac
  int32_t* status;
  uint64_t budget_ns;
  const int32_t* gate;  // if set, the kernel runs only when (*gate != 0) == gate_want
  int gate_want;
  int ksplit;              // K parts per tile (1: no split)
  int32_t* sk_sum;         // ksplit > 1: [tile][pair * 16 + column][row in tile] int32
  unsigned int* sk_count;  // ksplit > 1: [tile] parts arrived
};

__global__ void __launch_bounds__(kSkThreads, 1)
    k_skinny_s8(const __grid_constant__ CUtensorMap mapA, const __grid_constant__ CUtensorMap mapX,
                const __grid_constant__ SkPairs pairs, const __grid_constant__ SkArgs g) {
  if (g.gate && ((*(volatile const int32_t*)g.gate != 0) != (g.gate_want != 0))) return;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const int nS = g.nS, ST = g.stages;
  const uint32_t stage_bytes = (uint32_t)nS * (kSkABytes + kSkXBytes);
  int32_t* s_eX = (int32_t*)(smem + ST * stage_bytes);           // [kSkMaxSlices][16]
  uint64_t* bars = (uint64_t*)(s_eX + kSkMaxSlices * kSkCols);
  uint64_t* full = bars;
  uint64_t* empty = bars + kSkMaxStages;
  uint64_t* accf = empty + kSkMaxStages;
  uint64_t* acce = accf + 1;
  uint64_t* mma_done = acce + 1;
  uint32_t* s_tmem = (uint32_t*)(mma_done + 1);
  volatile int* s_abort = (volatile int*)(s_tmem + 1);
  volatile int* s_sk_last = s_abort + 1;  // epilogue: this CTA completes a split tile
  auto a_tile = [&](int s, int a) { return smem + s * stage_bytes + a * kSkABytes; };
  auto x_tile = [&](int s, int b) { return smem + s * stage_bytes + nS * kSkABytes + b * kSkXBytes; };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Work items j: tile j / ksplit, k-blocks [kb0(j), kb1(j)) of it.
  const int n_items = g.num_tiles * g.ksplit;
  auto kb0 = [&](int j) { return (j % g.ksplit) * g.num_kb / g.ksplit; };
  auto kb1 = [&](int j) { return (j % g.ksplit + 1) * g.num_kb / g.ksplit; };
  if (threadIdx.x == 0) {
    for (int i = 0; i < kSkMaxStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(accf, 1);
    mbar_init(acce, 4);
    mbar_init(mma_done, 1);
    *s_abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(s_tmem, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&mapA);
      tma_prefetch_desc(&mapX);
      uint32_t it = 0;
      bool ok = true;
      for (int j = blockIdx.x; ok && j < n_items; j += gridDim.x) {
        const int t = j / g.ksplit;
        for (int kb = kb0(j); kb < kb1(j); ++kb) {
          const uint32_t s = it % ST, ph = (it / ST) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, s_abort, g.status, g.budget_ns)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], stage_bytes);
          for (int a = 0; a < nS; ++a)
            tma_load_3d(a_tile(s, a), &mapA, &full[s], kb * kS8KB, t * kSkRows, a);
          for (int b = 0; b < nS; ++b)
            tma_load_3d(x_tile(s, b), &mapX, &full[s], kb * kS8KB, 0, b);
          ++it;
        }
      }
      // Every issued copy lands before shared memory is released.
      const uint32_t first = it > (uint32_t)ST ? it - ST : 0;
      for (uint32_t j = first; j < it; ++j)
        mbar_wait(&full[j % ST], (j / ST) & 1, nullptr, g.status, g.budget_ns);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc0 = umma_idesc_s8(kSkRows, 0);
      uint32_t it = 0, tile_it = 0;
      bool ok = true;
      for (int j = blockIdx.x; ok && j < n_items; j += gridDim.x, ++tile_it) {
        if (!mbar_wait(acce, (tile_it & 1) ^ 1, s_abort, g.status, g.budget_ns)) break;
        tc_fence_after();
        const int kbf = kb0(j);
        for (int kb = kbf; kb < kb1(j); ++kb) {
          const uint32_t s = it % ST, ph = (it / ST) & 1;
          if (!mbar_wait(&full[s], ph, s_abort, g.status, g.budget_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          for (int r = 0; r < pairs.n_runs; ++r) {
            const int p0 = pairs.run_p0[r];
            const uint32_t a0 = smem_u32(a_tile(s, pairs.a[p0]));
            const uint32_t x0 = smem_u32(x_tile(s, pairs.b[p0]));
            // N = 16 * len: the N field holds N / 8
            const uint32_t idesc = idesc0 | ((uint32_t)(2 * pairs.run_len[r]) << 17);
#pragma unroll
            for (int kk = 0; kk < kS8KB / 32; ++kk)
              umma_s8(tmem + p0 * kSkCols, umma_desc_sw128(a0 + kk * 32),
                      umma_desc_sw128(x0 + kk * 32), idesc, ((kb - kbf) | kk) != 0);
          }
          umma_commit(&empty[s]);
          ++it;
        }
        if (!ok) break;
        umma_commit(accf);
      }
      // All MMAs issued by this thread complete before TMEM is released.
      umma_commit(mma_done);
      mbar_wait(mma_done, 0, nullptr, g.status, g.budget_ns);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quadrant of this warp
    const int et = threadIdx.x - 64;
    // Column exponents: slice 0 absolute, the others relative to slice 0.
    for (int e = et; e < nS * kSkCols; e += 128) {
      const int b = e / kSkCols, c = e % kSkCols;
      s_eX[e] = c < g.M ? g.eX[(int64_t)b * g.M + c] : 0;
    }
    named_bar(1, 128);
    for (int e = et + kSkCols; e < nS * kSkCols; e += 128) s_eX[e] -= s_eX[e % kSkCols];
    named_bar(1, 128);
    uint32_t tile_it = 0;
    for (int j = blockIdx.x; j < n_items; j += gridDim.x, ++tile_it) {
      const int t = j / g.ksplit;
      int got = 1;
      if (lane == 0) got = mbar_wait(accf, tile_it & 1, s_abort, g.status, g.budget_ns);
      got = __shfl_sync(0xffffffffu, got, 0);
      if (!got) break;
      tc_fence_after();
      const int rq = q * 32 + lane;  // row within the tile
      const int64_t row = (int64_t)t * kSkRows + rq;
      const bool rvalid = row < g.N;
      const bool split = g.ksplit > 1;
      int32_t* const slot = split ? g.sk_sum + (int64_t)t * pairs.n * kSkCols * kSkRows + rq : nullptr;
      if (split) {
        // This part's products into the tile's slot (exact int32 adds), the
        // accumulators released, then the count; the last part goes on.
        for (int p = 0; p < pairs.n; ++p) {
          uint32_t P[kSkCols];
          tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + p * kSkCols, P);
          tmem_wait_ld();
          if (rvalid) {
#pragma unroll
            for (int c = 0; c < kSkCols; ++c)
              if (c < g.M) atomicAdd(slot + (p * kSkCols + c) * kSkRows, (int)P[c]);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(acce);
        __threadfence();  // this thread's adds are performed before the count
        named_bar(1, 128);
        if (et == 0) *s_sk_last = (int)(atomicAdd(&g.sk_count[t], 1u) + 1 == (unsigned)g.ksplit);
        named_bar(1, 128);
        if (!*s_sk_last) continue;
        __threadfence();
      }
      const int eA0 = rvalid ? g.eA[row] : 0;
      long long acc[kSkCols];
#pragma unroll
      for (int c = 0; c < kSkCols; ++c) acc[c] = 0;
      for (int p = 0; p < pairs.n; ++p) {
        const int a = pairs.a[p], b = pairs.b[p];
        const int ta = (rvalid ? g.eA[(int64_t)a * g.N + row] : 0) - eA0 + kFixFrac;
        uint32_t P[kSkCols];
        if (split) {
#pragma unroll
          for (int c = 0; c < kSkCols; ++c) P[c] = (uint32_t)ld_cg_s32(slot + (p * kSkCols + c) * kSkRows);
        } else {
          tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + p * kSkCols, P);
          tmem_wait_ld();
        }
#pragma unroll
        for (int c = 0; c < kSkCols; ++c)
          acc[c] += fixed_term_s32((int32_t)P[c], ta + (b == 0 ? 0 : s_eX[b * kSkCols + c]));
      }
      if (!split) {
        // The accumulators are read: the next tile's MMAs may start.
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(acce);
      }
      if (rvalid) {
#pragma unroll
        for (int c = 0; c < kSkCols; ++c) {
          if (c < g.M) {
            double v = fixed_value(acc[c], eA0 + s_eX[c] + g.fix_scale);
            v = g.alpha * v;
            if (g.beta != 0.0) v = fma(g.beta, g.Cin[row * g.ldcin + c], v);
            g.C[row * g.ldc + c] = v;
          }
        }
      }
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

bool skinny_s8_eligible(int64_t N, int64_t M, int64_t k8, int nS, int n_pairs, int rho) {
  return s8_enabled() && M >= 1 && M <= kSkCols && N >= 1 && nS >= 1 && nS <= kSkMaxSlices &&
         n_pairs >= 1 && n_pairs <= kSkMaxPairs && rho >= kS8MinRho && k8 > 0 && k8 % kS8KB == 0 &&
         k8 <= 65536;
}

int launch_skinny_s8(const int8_t* SA, const int32_t* eA, const int8_t* SX, const int32_t* eX,
                     int nS, int64_t N, int64_t M, int64_t k8, const uint8_t* pair_a,
                     const uint8_t* pair_b, int n_pairs, double alpha, double beta,
                     const double* Cin, int64_t ldcin, double* C, int64_t ldc, int rho,
                     int32_t* status, const int32_t* gate, int gate_want, void* scratch,
                     size_t scratch_bytes, cudaStream_t stream) {
  if (N == 0 || M == 0) return OZK_OK;
  if (!skinny_s8_eligible(N, M, k8, nS, n_pairs, rho))
    return set_error(OZK_ERR_UNSUPPORTED,
                     "skinny int8 GEMM: needs M <= %d, nS <= %d, n_pairs <= %d, rho >= %d",
                     kSkCols, kSkMaxSlices, kSkMaxPairs, kS8MinRho);
  if (ldc < M || (beta != 0.0 && (!Cin || ldcin < M)))
    return set_error(OZK_ERR_ARG, "bad C / Cin leading dimension");
  for (int p = 0; p < n_pairs; ++p)
    if (pair_a[p] >= nS || pair_b[p] >= nS) return set_error(OZK_ERR_ARG, "pair index out of range");
  int dev;
  cudaGetDevice(&dev);
  CUtensorMap ma, mx;
  int rc;
  if ((rc = make_slice_map(&ma, SA, k8, N, nS, kSkRows, true))) return rc;
  if ((rc = make_slice_map(&mx, SX, k8, M, nS, kSkCols, true))) return rc;
  const size_t stage_bytes = (size_t)nS * (kSkABytes + kSkXBytes);
  const size_t tail = kSkMaxSlices * kSkCols * 4 + (2 * kSkMaxStages + 3) * 8 + 16;
  const size_t budget = 227 * 1024 - 1024 - tail;
  int stages = (int)(budget / stage_bytes);
  if (stages > kSkMaxStages) stages = kSkMaxStages;
  if (stages < 2) return set_error(OZK_ERR_UNSUPPORTED, "skinny int8 GEMM: stages do not fit");
  const size_t smem = 1024 + stages * stage_bytes + tail;
  static int configured[64] = {0};
  if (!configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(k_skinny_s8, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         227 * 1024);
    if (e != cudaSuccess) return set_cuda_error("cudaFuncSetAttribute(k_skinny_s8)", e);
    configured[dev] = 1;
  }
  // Pairs sorted by (a, b) (the fixed-point sum does not depend on the
  // order), then cut into runs of consecutive b under one a.
  SkPairs pl;
  memset(&pl, 0, sizeof(pl));
  int order[kSkMaxPairs];
  for (int p = 0; p < n_pairs; ++p) order[p] = p;
  for (int i = 1; i < n_pairs; ++i)
    for (int j = i; j > 0; --j) {
      const int u = order[j - 1], v = order[j];
      if (pair_a[u] < pair_a[v] || (pair_a[u] == pair_a[v] && pair_b[u] <= pair_b[v])) break;
      order[j - 1] = v;
      order[j] = u;
    }
  for (int p = 0; p < n_pairs; ++p) {
    pl.a[p] = pair_a[order[p]];
    pl.b[p] = pair_b[order[p]];
  }
  pl.n = n_pairs;
  for (int p = 0; p < n_pairs; ++p) {
    const int r = pl.n_runs - 1;
    if (p > 0 && pl.a[p] == pl.a[p - 1] && pl.b[p] == pl.b[p - 1] + 1 && pl.run_len[r] < 16) {
      ++pl.run_len[r];
    } else {
      pl.run_p0[pl.n_runs] = (uint8_t)p;
      pl.run_len[pl.n_runs] = 1;
      ++pl.n_runs;
    }
  }
  SkArgs ga;
  memset(&ga, 0, sizeof(ga));
  ga.eA = eA;
  ga.eX = eX;
  ga.N = N;
  ga.M = (int)M;
  ga.nS = nS;
  ga.stages = stages;
  ga.num_kb = (int)(k8 / kS8KB);
  ga.num_tiles = (int)((N + kSkRows - 1) / kSkRows);
  ga.alpha = alpha;
  ga.beta = beta;
  ga.Cin = Cin;
  ga.ldcin = ldcin;
  ga.C = C;
  ga.ldc = ldc;
  ga.fix_scale = 2 * (rho - 24) - kFixFrac;
  ga.status = status;
  ga.budget_ns = wait_budget_ns();
  ga.gate = gate;
  ga.gate_want = gate_want;
  // K split (exact, see the kernel) when the tiles would leave SMs idle: fewer
  // tiles than SMs, or a last wave under half full.  The k <= 8 parts (each
  // at least 4 k-blocks) minimise the rounds of work per part,
  // ceil(tiles k / SMs) / k, if that saves at least a tenth.  (A last wave
  // more than half full stays whole: the kernel streams from HBM, and the SMs
  // of such a wave already draw most of its bandwidth.)
  const int sms = device_sm_count(dev);
  const int T = ga.num_tiles;
  ga.ksplit = 1;
  if (T < sms || T % sms < sms / 2) {
    const double one = (double)((T + sms - 1) / sms);
    double best = one;
    int ks = 1;
    for (int k = 2; k <= 8 && ga.num_kb / k >= 4; ++k) {
      const double cost = (double)((T * k + sms - 1) / sms) / k;
      if (cost < best - 1e-9) {
        best = cost;
        ks = k;
      }
    }
    const size_t counts = ((size_t)T * sizeof(unsigned int) + 255) & ~(size_t)255;
    const size_t sums = (size_t)T * n_pairs * kSkCols * kSkRows * sizeof(int32_t);
    if (ks > 1 && best <= 0.9 * one && scratch && scratch_bytes >= counts + sums &&
        ((uintptr_t)scratch & 255) == 0) {
      ga.ksplit = ks;
      ga.sk_count = (unsigned int*)scratch;
      ga.sk_sum = (int32_t*)((char*)scratch + counts);
      cudaError_t e = cudaMemsetAsync(scratch, 0, counts + sums, stream);
      if (e != cudaSuccess) return set_cuda_error("cudaMemsetAsync(skinny split sums)", e);
    }
  }
  int grid = sms;
  if (grid > T * ga.ksplit) grid = T * ga.ksplit;
  k_skinny_s8<<<grid, kSkThreads, smem, stream>>>(ma, mx, pl, ga);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? OZK_OK : set_cuda_error("k_skinny_s8 launch", e);
}

}  // namespace ozk
