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
#include <stdlib.h>
#include <string.h>

#include "ozk_device.cuh"
#include "ozk_fixed.cuh"
#include "ozk_internal.h"

namespace ozk {

constexpr int kBM = 128;

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
  unsigned long long* stats;  // optional per-CTA wait-cycle counters (diagnostics)
  double* state;              // per-CTA FP64 running sums (BN = 256 tiles)
  int c_vec;                  // C is 32-byte aligned with ldc % 4 == 0
  int fixed;                  // 1: int64 fixed-point sums (OZK_ACC_FIXED), 0: FP64 sums
  int fix_off;                // -150 - G + kFixFrac, G = product-grid exponent 2 (rho - 24)
  int fix_scale;              // G - kFixFrac: output = sum * 2^(eA0 + eB0 + fix_scale)
  int prefetch;               // L2 prefetch distance in stages (0 = off)
  const int32_t* gate;        // if set, the kernel runs only when (*gate != 0) == gate_want
  int gate_want;
  // Pacing (optional): a unit's producer starts pair g of its walk only once
  // the units have issued pairs through g - pace_slack on average (counted in
  // *pace), waiting at most pace_budget_ns; keeps the units that share A and
  // B panels close enough in time for the panels to be reused from L2.
  unsigned long long* pace;
  int pace_slack;
  uint64_t pace_budget_ns;
  // Work split (int8 wide tiles): tiles below dp_tiles go round-robin, whole;
  // each of the r remaining tiles is cut into sk_chunks equal pair ranges, and
  // the r * sk_chunks items j = (chunk j / r of tile dp_tiles + j % r) go
  // round-robin too, so the units of a round run the same pairs of
  // neighbouring tiles at once (their panels are shared in L2, as in the
  // whole-tile waves).  A unit holding part of a tile's pairs adds its exact
  // int64 partial sums into sk_sum and counts itself in sk_count; the last of
  // the tile's sk_chunks contributors writes C.  dp_tiles == num_tiles: no
  // split.
  int dp_tiles, sk_chunks;
  long long* sk_sum;       // [tile - dp_tiles][rank][column][row in CTA]
  unsigned int* sk_count;  // [tile - dp_tiles][rank]
  // Raw output (int8 wide tiles, fixed-point sums): with C64 set, each
  // element's int64 sum is stored there (leading dimension ldc) as it is, in
  // units of 2^(eA0 + eB0 + fix_scale), instead of its FP64 value in C; a
  // symmetric launch stores only the upper triangle (column >= row).  Partial
  // sums of a split contraction add up exactly to the whole one's.
  long long* C64;
};

// PAIR = false: one CTA per output tile of 128 x BN.
// PAIR = true:  a cluster of two CTAs (a CTA pair on one TPC) per 256 x BN
//   tile with cta_group::2 MMAs (M = 256): each CTA stages its 128 rows of A
//   and half of B's BN rows, so a pair moves 3/4 of the shared-memory bytes
//   per FLOP that two single CTAs would; the even CTA issues the MMAs, its
//   full barriers count both CTAs' TMA bytes, stage releases and
//   accumulator-ready signals go to both CTAs, and both epilogues report to
//   the even CTA's accumulator-empty barriers.
template <int BN, bool PAIR>
struct GemmCfg {
  static constexpr int CTA_N = PAIR ? BN / 2 : BN;  // B rows staged per CTA
  static constexpr int TILE_M = PAIR ? 2 * kBM : kBM;
  static constexpr int A_BYTES = kBM * OZK_KB * 2;
  static constexpr int B_BYTES = CTA_N * OZK_KB * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = BN >= 256 ? 6 : (PAIR ? 8 : (BN >= 64 ? 6 : 8));
  // BN = 256: both TMEM accumulators take all 512 columns and the FP64 running
  // sum lives in a per-CTA global scratch; otherwise it is kept in TMEM.
  static constexpr bool GSTATE = BN >= 256;
  static constexpr int TMEM_COLS = GSTATE ? 2 * BN : (4 * BN < 32 ? 32 : 4 * BN);
  static constexpr int EPI_WARPS = GSTATE ? 8 : 4;  // 4 lane quadrants x column halves
  static constexpr int THREADS = 64 + 32 * EPI_WARPS;
  static constexpr int EPI_COLS = BN / (EPI_WARPS / 4);  // columns per epilogue thread
  static constexpr int CH = BN < 32 ? BN : 32;  // epilogue column chunk
  static constexpr int EB_BYTES = OZK_MAX_SLICES * BN * 4;
  static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + EB_BYTES + 256;
  static constexpr int64_t STATE_PER_CTA = (int64_t)kBM * BN;  // doubles
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

// The work items of a unit: its round-robin whole tiles (ndp), then its
// round-robin chunks of split tiles (nsk).
struct ItemRange {
  int ndp, nsk;
};

__device__ __forceinline__ ItemRange item_range(const GemmArgs& g, int unit, int n_units) {
  ItemRange r;
  r.ndp = g.dp_tiles > unit ? (g.dp_tiles - unit + n_units - 1) / n_units : 0;
  const int items = (g.num_tiles - g.dp_tiles) * g.sk_chunks;
  r.nsk = items > unit ? (items - unit + n_units - 1) / n_units : 0;
  return r;
}

// Item i: tile t and its pairs [p0, p1).
__device__ __forceinline__ void item_at(const GemmArgs& g, const ItemRange& r, int unit,
                                        int n_units, int np, int i, int& t, int& p0, int& p1) {
  if (i < r.ndp) {
    t = unit + i * n_units;
    p0 = 0;
    p1 = np;
    return;
  }
  const int rem = g.num_tiles - g.dp_tiles;
  const int j = unit + (i - r.ndp) * n_units;  // split item
  const int chunk = j / rem;
  t = g.dp_tiles + j % rem;
  p0 = chunk * np / g.sk_chunks;
  p1 = (chunk + 1) * np / g.sk_chunks;
}

// FP64 value of P * 2^e for the FP32 product bits u (exact), built with
// integer operations only: the FP32 exponent field moves to the FP64 one with
// e added, the mantissa shifts by 29.  Falls back to FP64 multiplies when the
// result would leave the normal FP64 range.  sign_flip = 0x80000000 negates.
__device__ __forceinline__ double scaled_term(uint32_t u, int e, uint32_t sign_flip) {
  const uint32_t ex = (u >> 23) & 0xFFu;
  if (ex == 0) return 0.0;  // products are 0 or normal
  const int E = (int)ex + e + (1023 - 127);
  if (E >= 1 && E <= 2046) {
    const uint32_t hi = ((u & 0x80000000u) ^ sign_flip) | ((uint32_t)E << 20) | ((u >> 3) & 0xFFFFFu);
    return __hiloint2double((int)hi, (int)(u << 29));
  }
  const double v = (double)__uint_as_float(u ^ sign_flip);
  return (v * pow2d(e / 2)) * pow2d(e - e / 2);
}

// S8 = true: int8 slice codes and kind::i8 MMAs into exact int32 accumulators
// (OZK_ACC_FIXED only, CTA pairs only); a pipeline stage then holds 128 K
// elements, the same bytes as 64 BF16 ones.
template <int BN, bool PAIR, bool S8>
__global__ void __launch_bounds__(GemmCfg<BN, PAIR>::THREADS, 1)
    k_slice_gemm(const __grid_constant__ CUtensorMap mapA, const __grid_constant__ CUtensorMap mapB,
                 const __grid_constant__ PairList pairs, const __grid_constant__ GemmArgs g) {
  static_assert(!S8 || PAIR, "int8 slices run on CTA pairs");
  using Cfg = GemmCfg<BN, PAIR>;
  constexpr int KBE = S8 ? kS8KB : OZK_KB;  // K elements per stage
  // Device-side choice between the int8 pass and its BF16 recomputation: every
  // CTA reads the same word, so the whole grid leaves before any setup.
  if (g.gate && ((*(volatile const int32_t*)g.gate != 0) != (g.gate_want != 0))) return;
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

  __shared__ int s_sk_last;  // epilogue: this CTA completes a split tile
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = PAIR ? cluster_ctarank() : 0;  // 0 = MMA-issuing CTA
  const int unit = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int n_units = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&accf[i], 1);
      mbar_init(&acce[i], (PAIR ? 2 : 1) * Cfg::EPI_WARPS);
    }
    mbar_init(mma_done, 1);
    *s_abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    if constexpr (PAIR) tmem_alloc_pair(s_tmem, Cfg::TMEM_COLS);
    else tmem_alloc(s_tmem, Cfg::TMEM_COLS);
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync();  // peer barriers initialised before any remote use
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
      long long w_empty = 0;
      bool pacer = g.pace != nullptr && (!PAIR || rank == 0);
      long long walk = 0;  // pairs this unit has issued
      const ItemRange ir = item_range(g, unit, n_units);
      for (int i = 0; ok && i < ir.ndp + ir.nsk; ++i) {
        int t, p0, p1, tm, tn;
        item_at(g, ir, unit, n_units, npairs, i, t, p0, p1);
        tile_coords(g, t, tm, tn);
        const int arow = tm * Cfg::TILE_M + (int)rank * kBM;
        const int brow = tn * BN + (int)rank * Cfg::CTA_N;
        for (int p = p0; ok && p < p1; ++p) {
          const int a = pairs.a[p], b = pairs.b[p];
          if (pacer && walk >= g.pace_slack) {
            const unsigned long long need =
                (unsigned long long)n_units * (unsigned long long)(walk - g.pace_slack + 1);
            const uint64_t t0 = global_ns();
            while (*(volatile unsigned long long*)g.pace < need) {
              if (global_ns() - t0 > g.pace_budget_ns) {
                // Some unit is not keeping up (not resident, or the GPU is
                // shared): stop pacing rather than wait again.
                pacer = false;
                break;
              }
              __nanosleep(256);
            }
          }
          for (int kb = 0; kb < g.num_kb; ++kb) {
            const uint32_t s = it % STAGES, ph = (it / STAGES) & 1;
            if (g.prefetch) {
              // Pull the stage `prefetch` steps ahead (same tile, possibly the
              // next pair) into L2 so pair boundaries do not wait on DRAM.
              int pk = kb + g.prefetch, pp = p;
              if (pk >= g.num_kb) {
                pk -= g.num_kb;
                ++pp;
              }
              if (pp < p1 && pk < g.num_kb) {
                tma_prefetch_3d(&mapA, pk * KBE, arow, pairs.a[pp]);
                tma_prefetch_3d(&mapB, pk * KBE, brow, pairs.b[pp]);
              }
            }
            long long c0 = clock64();
            if (!mbar_wait(&empty[s], ph ^ 1, s_abort, g.status, g.budget_ns)) {
              ok = false;
              break;
            }
            w_empty += clock64() - c0;
            if constexpr (PAIR) {
              if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * Cfg::STAGE_BYTES);
              const uint32_t fb = mapa_u32(&full[s], 0);
              tma_load_3d_pair(sA + s * Cfg::A_BYTES, &mapA, fb, kb * KBE, arow, a);
              tma_load_3d_pair(sB + s * Cfg::B_BYTES, &mapB, fb, kb * KBE, brow, b);
            } else {
              mbar_arrive_expect_tx(&full[s], Cfg::STAGE_BYTES);
              tma_load_3d(sA + s * Cfg::A_BYTES, &mapA, &full[s], kb * KBE, arow, a);
              tma_load_3d(sB + s * Cfg::B_BYTES, &mapB, &full[s], kb * KBE, brow, b);
            }
            ++it;
          }
          if (g.pace && (!PAIR || rank == 0)) atomicAdd(g.pace, 1ull);
          ++walk;
        }
      }
      if (g.pace && (!PAIR || rank == 0)) {
        // A unit with fewer tiles (or one that stopped) counts as done with
        // every pair the longest walk has, so no one waits for it.
        const int items = (g.num_tiles - g.dp_tiles) * g.sk_chunks;
        const long long longest =
            (long long)((g.dp_tiles + n_units - 1) / n_units) * npairs +
            (items ? (long long)((items + n_units - 1) / n_units) *
                         ((npairs + g.sk_chunks - 1) / g.sk_chunks)
                   : 0);
        if (longest > walk) atomicAdd(g.pace, (unsigned long long)(longest - walk));
      }
      if (g.stats) g.stats[8 * blockIdx.x + 2] = (unsigned long long)w_empty;
      // Drain: every issued copy must land before shared memory is released.
      // (In a pair only the even CTA's full barriers count the bytes.)
      if (!PAIR || rank == 0) {
        uint32_t first = it > (uint32_t)STAGES ? it - STAGES : 0;
        for (uint32_t j = first; j < it; ++j)
          mbar_wait(&full[j % STAGES], (j / STAGES) & 1, nullptr, g.status, g.budget_ns);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = S8 ? umma_idesc_s8(Cfg::TILE_M, BN) : umma_idesc_bf16(Cfg::TILE_M, BN);
      uint32_t it = 0, acc_it = 0;
      bool ok = true;
      long long w_acc = 0, w_full = 0, w_head = 0, t_start = clock64();
      const ItemRange ir = item_range(g, unit, n_units);
      for (int i = 0; ok && i < ir.ndp + ir.nsk; ++i) {
        int t, p0, p1;
        item_at(g, ir, unit, n_units, npairs, i, t, p0, p1);
        for (int p = p0; ok && p < p1; ++p) {
          const uint32_t buf = acc_it & 1, aph = (acc_it >> 1) & 1;
          long long c0 = clock64();
          if (!mbar_wait(&acce[buf], aph ^ 1, s_abort, g.status, g.budget_ns)) {
            ok = false;
            break;
          }
          w_acc += clock64() - c0;
          tc_fence_after();
          const uint32_t d = tmem + buf * BN;
          for (int kb = 0; kb < g.num_kb; ++kb) {
            const uint32_t s = it % STAGES, ph = (it / STAGES) & 1;
            long long c1 = clock64();
            if (!mbar_wait(&full[s], ph, s_abort, g.status, g.budget_ns)) {
              ok = false;
              break;
            }
            {
              const long long wf = clock64() - c1;
              w_full += wf;
              if (kb < STAGES) w_head += wf;
            }
            tc_fence_after();
            const uint32_t a0 = smem_u32(sA + s * Cfg::A_BYTES);
            const uint32_t b0 = smem_u32(sB + s * Cfg::B_BYTES);
#pragma unroll
            for (int kk = 0; kk < OZK_KB / 16; ++kk) {
              const uint64_t da = umma_desc_sw128(a0 + kk * 32);
              const uint64_t db = umma_desc_sw128(b0 + kk * 32);
              if constexpr (S8) umma_s8_pair(d, da, db, idesc, (kb | kk) != 0);
              else if constexpr (PAIR) umma_bf16_pair(d, da, db, idesc, (kb | kk) != 0);
              else umma_bf16(d, da, db, idesc, (kb | kk) != 0);
            }
            if constexpr (PAIR) umma_commit_pair(&empty[s], 0x3);
            else umma_commit(&empty[s]);
            ++it;
          }
          if (!ok) break;
          if constexpr (PAIR) umma_commit_pair(&accf[buf], 0x3);
          else umma_commit(&accf[buf]);
          ++acc_it;
        }
      }
      // All MMAs issued by this thread complete before TMEM is released.
      if constexpr (PAIR) umma_commit_pair(mma_done, 0x1);
      else umma_commit(mma_done);
      mbar_wait(mma_done, 0, nullptr, g.status, g.budget_ns);
      if (g.stats) {
        unsigned long long* st = g.stats + 8 * blockIdx.x;
        st[0] = (unsigned long long)w_acc;
        st[1] = (unsigned long long)w_full;
        st[3] = (unsigned long long)(clock64() - t_start);
        st[7] = (unsigned long long)w_head;
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    constexpr int NE = 32 * Cfg::EPI_WARPS;  // epilogue threads
    const int q = warp & 3;                 // TMEM lane quadrant of this warp
    const int half = (warp - 2) >> 2;       // column range of this warp
    const int cbeg = half * Cfg::EPI_COLS;  // first tile column of this thread
    const int etid = threadIdx.x - 64;      // 0..NE-1 among epilogue threads
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    // Column-major per-CTA FP64 state: a warp touches 32 consecutive rows of
    // one column (256 contiguous bytes) per access.
    double* const gst = Cfg::GSTATE ? g.state + (int64_t)blockIdx.x * Cfg::STATE_PER_CTA
                                      + q * 32 + lane : nullptr;
    const uint64_t l2keep = l2_policy_evict_last();  // the state is re-read every pair
    const uint32_t acce_leader = PAIR ? mapa_u32(&acce[0], 0) : 0;
    uint32_t acc_it = 0;
    bool ok = true;
    // (32-bit cycle sums: a launch lasts far fewer than 2^32 cycles)
    uint32_t ep_wait = 0, ep_busy = 0, ep_pairs = 0;
    long long Sa[16], Sb[16];  // running sums of two column chunks (int8 wide tiles)
    const ItemRange ir = item_range(g, unit, n_units);
    for (int i = 0; ok && i < ir.ndp + ir.nsk; ++i) {
      int t, p0, p1, tm, tn;
      item_at(g, ir, unit, n_units, npairs, i, t, p0, p1);
      tile_coords(g, t, tm, tn);
      // part of the tile's pairs: the sums go to the split slot, not to C
      const bool partial = p0 > 0 || p1 < npairs;
      auto sk_slot = [&]() {
        return g.sk_sum + ((int64_t)(t - g.dp_tiles) * 2 + rank) * (BN * kBM) + q * 32 + lane;
      };
      const int64_t col0 = (int64_t)tn * BN;
      named_bar(1, NE);
      for (int e = etid; e < g.nB * BN; e += NE) {
        int64_t c = col0 + (e % BN);
        s_eB[e] = c < g.M ? g.eB[(int64_t)(e / BN) * g.M + c] : 0;
      }
      named_bar(1, NE);
      if (g.fixed) {  // slices >= 1 hold eb - eB0 (read after the barrier below)
        for (int e = etid + BN; e < g.nB * BN; e += NE) s_eB[e] -= s_eB[e % BN];
        named_bar(1, NE);
      }
      const int64_t row = (int64_t)tm * Cfg::TILE_M + rank * kBM + q * 32 + lane;
      const bool rvalid = row < g.N;
      const int eA0 = rvalid ? g.eA[row] : 0;
      for (int p = p0; p < p1; ++p) {
        const uint32_t buf = acc_it & 1, aph = (acc_it >> 1) & 1;
        int got = 1;
        const uint32_t e0 = (uint32_t)clock64();
        if (lane == 0) got = mbar_wait(&accf[buf], aph, s_abort, g.status, g.budget_ns);
        got = __shfl_sync(0xffffffffu, got, 0);
        if (!got) {
          ok = false;
          break;
        }
        const uint32_t e1 = (uint32_t)clock64();
        tc_fence_after();
        const int a = pairs.a[p], b = pairs.b[p];
        const int ea = rvalid ? g.eA[(int64_t)a * g.N + row] : 0;
        const bool first = (p == p0), last = (p == p1 - 1);
        const uint32_t t_acc = tmem + lane_base + buf * BN;
        const uint32_t t_lo = tmem + lane_base + 2 * BN;
        const uint32_t t_hi = tmem + lane_base + 3 * BN;
        if constexpr (S8 && Cfg::GSTATE) {
          // int8 codes, fixed-point sums, running sums in the L2 scratch.  The
          // columns go in chunks of 16 with the next chunk's running sums in
          // flight while this one is computed, and chunk 0 of the next pair is
          // requested before this warp waits for that pair's accumulator.
          constexpr int C2 = 16;
          constexpr int NCH = Cfg::EPI_COLS / C2;
          const int ta = ea - eA0 + kFixFrac;
          auto load_state = [&](long long (&S)[C2], int c0) {
#pragma unroll
            for (int j = 0; j < C2; ++j)
              S[j] = ld_l2_hint((const long long*)(gst + (int64_t)(c0 + j) * kBM), l2keep);
          };
          // the FP64 results of a chunk's sums, alpha / beta applied, into C
          auto store_c = [&](const long long (&acc)[C2], int c0) {
            if (!rvalid) return;
            if (g.C64) {  // the raw sums
#pragma unroll
              for (int j = 0; j < C2; ++j) {
                const int64_t col = col0 + c0 + j;
                if (col < g.M && (!g.symmetric || col >= row)) g.C64[row * g.ldc + col] = acc[j];
              }
              return;
            }
            double V[C2];
#pragma unroll
            for (int j = 0; j < C2; ++j) {
              double v = g.alpha * fixed_value(acc[j], eA0 + s_eB[c0 + j] + g.fix_scale);
              if (g.beta != 0.0 && col0 + c0 + j < g.M)
                v = fma(g.beta, g.Cin[row * g.ldcin + col0 + c0 + j], v);
              V[j] = v;
            }
            const int64_t cb = col0 + c0;
            double* crow = g.C + row * g.ldc + cb;
            if (!g.symmetric && g.c_vec && cb + C2 <= g.M) {
#pragma unroll
              for (int j = 0; j < C2; j += 4) st_global_v4_f64(crow + j, V[j], V[j + 1], V[j + 2], V[j + 3]);
            } else {
#pragma unroll
              for (int j = 0; j < C2; ++j) {
                const int64_t col = cb + j;
                if (col < g.M) {
                  if (!g.symmetric) {
                    crow[j] = V[j];
                  } else if (tm != tn || col >= row) {
                    crow[j] = V[j];
                    g.C[col * g.ldc + row] = V[j];
                  }
                }
              }
            }
          };
          auto process = [&](const long long (&S)[C2], int c0) {
            uint32_t P[C2];
            tmem_ld16(t_acc + c0, P);
            tmem_wait_ld();
            long long acc[C2];
#pragma unroll
            for (int j = 0; j < C2; ++j) {
              const int db = b == 0 ? 0 : s_eB[b * BN + c0 + j];  // eb - eB0
              acc[j] = fixed_term_s32((int32_t)P[j], ta + db) + (first ? 0ll : S[j]);
            }
            if (!last) {
#pragma unroll
              for (int j = 0; j < C2; ++j)
                st_l2_hint((long long*)(gst + (int64_t)(c0 + j) * kBM), acc[j], l2keep);
              return;
            }
            if (partial) {  // exact integer adds: the order of the contributors is free
              if (rvalid) {
                long long* const sks = sk_slot();
#pragma unroll
                for (int j = 0; j < C2; ++j)
                  atomicAdd((unsigned long long*)(sks + (int64_t)(c0 + j) * kBM),
                            (unsigned long long)acc[j]);
              }
              return;
            }
            store_c(acc, c0);
          };
          // Sa holds chunk 0 of this pair when it is not the first (loaded at
          // the end of the previous pair); chunks alternate between Sa and Sb.
#pragma unroll 1
          for (int ci = 0; ci < NCH; ci += 2) {
            const int c0 = cbeg + ci * C2;
            if (!first) load_state(Sb, c0 + C2);
            process(Sa, c0);
            if (!first && ci + 2 < NCH) load_state(Sa, c0 + 2 * C2);
            process(Sb, c0 + C2);
          }
          // this thread's stores precede these loads of the same addresses
          if (!last) load_state(Sa, cbeg);
        } else {
#pragma unroll 1
        for (int c0 = cbeg; c0 < cbeg + Cfg::EPI_COLS; c0 += CH) {
          uint32_t P[CH], L[CH], H[CH];
          if constexpr (CH == 32) {
            tmem_ld32(t_acc + c0, P);
            if (!Cfg::GSTATE && g.mode != OZK_ACC_PRODUCTS && !first) {
              tmem_ld32(t_lo + c0, L);
              tmem_ld32(t_hi + c0, H);
            }
          } else {
            tmem_ld16(t_acc + c0, P);
            if (!Cfg::GSTATE && g.mode != OZK_ACC_PRODUCTS && !first) {
              tmem_ld16(t_lo + c0, L);
              tmem_ld16(t_hi + c0, H);
            }
          }
          double S[Cfg::GSTATE ? CH : 1];
          if constexpr (Cfg::GSTATE) {
            if (!first) {
#pragma unroll
              for (int j = 0; j < CH; ++j)
                S[j] = __longlong_as_double(
                    ld_l2_hint((const long long*)(gst + (int64_t)(c0 + j) * kBM), l2keep));
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
          if (g.fixed) {
            // ---- int64 fixed-point sums (integer pipes only until the last pair)
            const int ta = ea - eA0 + (S8 ? kFixFrac : g.fix_off);
#pragma unroll
            for (int j = 0; j < CH; ++j) {
              const int db = b == 0 ? 0 : s_eB[b * BN + c0 + j];  // eb - eB0
              long long acc;
              if constexpr (S8) acc = fixed_term_s32((int32_t)P[j], ta + db);
              else acc = fixed_term(P[j], ta + db);
              if (!first) {
                long long prev;
                if constexpr (Cfg::GSTATE) prev = __double_as_longlong(S[j]);
                else prev = (long long)(((unsigned long long)H[j] << 32) | L[j]);
                if constexpr (S8) acc += prev;  // int8 codes are finite by construction
                else acc = (acc == kFixNaN || prev == kFixNaN) ? kFixNaN : acc + prev;
              }
              if (!last) {
                if constexpr (Cfg::GSTATE) {
                  st_l2_hint((long long*)(gst + (int64_t)(c0 + j) * kBM), acc, l2keep);
                } else {
                  L[j] = (uint32_t)acc;
                  H[j] = (uint32_t)((unsigned long long)acc >> 32);
                }
              } else {
                double v = acc == kFixNaN ? __longlong_as_double(0x7ff8000000000000ll)
                                          : fixed_value(acc, eA0 + s_eB[c0 + j] + g.fix_scale);
                v = g.alpha * v;
                if (g.beta != 0.0 && rvalid && col0 + c0 + j < g.M)
                  v = fma(g.beta, g.Cin[row * g.ldcin + col0 + c0 + j], v);
                if constexpr (Cfg::GSTATE) {
                  S[j] = v;
                } else if (rvalid && col0 + c0 + j < g.M) {
                  const int64_t col = col0 + c0 + j;
                  if (!g.symmetric) {
                    g.C[row * g.ldc + col] = v;
                  } else if (tm != tn || col >= row) {
                    g.C[row * g.ldc + col] = v;
                    g.C[col * g.ldc + row] = v;
                  }
                }
              }
            }
          } else {
          // ---- FP64 sums (the same sums to FP64 rounding, pair order)
          const uint32_t sflip = g.alpha < 0.0 ? 0x80000000u : 0u;
#pragma unroll
          for (int j = 0; j < CH; ++j) {
            double acc;
            if (first) {
              acc = 0.0;
              if (g.beta != 0.0 && rvalid && col0 + c0 + j < g.M)
                acc = g.beta * g.Cin[row * g.ldcin + col0 + c0 + j];
            } else if constexpr (Cfg::GSTATE) {
              acc = S[j];
            } else {
              acc = __hiloint2double((int)H[j], (int)L[j]);
            }
            // one FP64 add per term; the term itself is built on the integer pipes
            acc += scaled_term(P[j], ea + s_eB[b * BN + c0 + j], sflip);
            if constexpr (Cfg::GSTATE) {
              if (!last)
                st_l2_hint((long long*)(gst + (int64_t)(c0 + j) * kBM), __double_as_longlong(acc),
                           l2keep);
              S[j] = acc;
            } else {
              L[j] = (uint32_t)__double2loint(acc);
              H[j] = (uint32_t)__double2hiint(acc);
            }
            if constexpr (!Cfg::GSTATE) {
              if (last && rvalid && col0 + c0 + j < g.M) {
                const int64_t col = col0 + c0 + j;
                if (!g.symmetric) {
                  g.C[row * g.ldc + col] = acc;
                } else if (tm != tn || col >= row) {
                  g.C[row * g.ldc + col] = acc;
                  g.C[col * g.ldc + row] = acc;
                }
              }
            }
          }
          }
          if constexpr (Cfg::GSTATE) {
            if (last && rvalid) {
              const int64_t cb = col0 + c0;
              double* crow = g.C + row * g.ldc + cb;
              if (!g.symmetric && g.c_vec && cb + CH <= g.M) {
#pragma unroll
                for (int j = 0; j < CH; j += 4) st_global_v4_f64(crow + j, S[j], S[j + 1], S[j + 2], S[j + 3]);
              } else {
#pragma unroll
                for (int j = 0; j < CH; ++j) {
                  const int64_t col = cb + j;
                  if (col < g.M) {
                    if (!g.symmetric) {
                      crow[j] = S[j];
                    } else if (tm != tn || col >= row) {
                      crow[j] = S[j];
                      g.C[col * g.ldc + row] = S[j];
                    }
                  }
                }
              }
            }
          }
          if (!Cfg::GSTATE && !last) {
            if constexpr (CH == 32) {
              tmem_st32(t_lo + c0, L);
              tmem_st32(t_hi + c0, H);
            } else {
              tmem_st16(t_lo + c0, L);
              tmem_st16(t_hi + c0, H);
            }
          }
        }
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if constexpr (PAIR) mbar_arrive_cluster(acce_leader + buf * sizeof(uint64_t));
          else mbar_arrive(&acce[buf]);
        }
        if (g.stats && warp == 2 && lane == 0) {
          const uint32_t e2 = (uint32_t)clock64();
          ep_wait += e1 - e0;
          ep_busy += e2 - e1;
          ++ep_pairs;
        }
        ++acc_it;
        if constexpr (S8 && Cfg::GSTATE) {
          if (partial && last) {
            // This CTA's share of the split tile is in sk_sum; the last of the
            // tile's contributors reads the total back and writes C.
            const int tr = t - g.dp_tiles;
            __threadfence();  // this thread's adds are performed before the count
            named_bar(1, NE);
            if (etid == 0) {
              const unsigned prev = atomicAdd(&g.sk_count[tr * 2 + rank], 1u);
              s_sk_last = (int)(prev + 1 == (unsigned)g.sk_chunks);
            }
            named_bar(1, NE);
            if (s_sk_last) {
              __threadfence();
              constexpr int C2 = 16;
              const long long* const sks = sk_slot();
              // (Sa is free here: the next item starts with its first pair.)
#pragma unroll 1
              for (int c0 = cbeg; c0 < cbeg + Cfg::EPI_COLS; c0 += C2) {
#pragma unroll
                for (int j = 0; j < C2; ++j) Sa[j] = ld_cg_s64(sks + (int64_t)(c0 + j) * kBM);
                if (!rvalid) continue;
#pragma unroll
                for (int j = 0; j < C2; ++j) {
                  const int64_t col = col0 + c0 + j;
                  if (col >= g.M) continue;
                  if (g.C64) {  // the raw sums
                    if (!g.symmetric || col >= row) g.C64[row * g.ldc + col] = Sa[j];
                    continue;
                  }
                  double v = g.alpha * fixed_value(Sa[j], eA0 + s_eB[c0 + j] + g.fix_scale);
                  if (g.beta != 0.0) v = fma(g.beta, g.Cin[row * g.ldcin + col], v);
                  if (!g.symmetric) {
                    g.C[row * g.ldc + col] = v;
                  } else if (tm != tn || col >= row) {
                    g.C[row * g.ldc + col] = v;
                    g.C[col * g.ldc + row] = v;
                  }
                }
              }
            }
          }
        }
      }
    }
    if (g.stats && warp == 2 && lane == 0) {
      unsigned long long* st = g.stats + 8 * blockIdx.x;
      st[4] = (unsigned long long)ep_wait;
      st[5] = (unsigned long long)ep_busy;
      st[6] = (unsigned long long)ep_pairs;
    }
  }

  __syncthreads();
  if constexpr (PAIR) cluster_sync();  // the pair finishes together before TMEM is freed
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR) tmem_dealloc_pair(tmem, Cfg::TMEM_COLS);
    else tmem_dealloc(tmem, Cfg::TMEM_COLS);
  }
}

// ---------------------------------------------------------------- host side

static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

// Diagnostics: with OZK_GEMM_STATS=1 each launch records, per CTA, the cycles
// its MMA thread waited for a free accumulator and for loaded stages, the
// cycles its producer waited for free stages, and the MMA thread's total;
// ozk_gemm_stats() returns the sums of the last launch.
static unsigned long long* g_stats_dev[64] = {nullptr};
static int g_stats_ctas[64] = {0};
static int g_stats_last_dev = -1;

static bool stats_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* s = getenv("OZK_GEMM_STATS");
    v = (s && s[0] == '1') ? 1 : 0;
  }
  return v == 1;
}

// L2 prefetch distance of the TMA producer, in stages (OZK_GEMM_PREFETCH;
// default 0 = off: measured on B200, prefetches issued by the producer thread
// delay its loads more than they save).
static int prefetch_distance() {
  static int v = -1;
  if (v < 0) {
    const char* s = getenv("OZK_GEMM_PREFETCH");
    v = s ? atoi(s) : 0;
    if (v < 0) v = 0;
  }
  return v;
}

// Tile rows per raster group (OZK_GEMM_GROUP_M, default 8): consecutive tiles
// walk down a group of this many tile rows before moving right, so the tiles
// in flight at once share few A and B panels in L2.
static int group_m_rows() {
  static int v = -1;
  if (v < 0) {
    const char* s = getenv("OZK_GEMM_GROUP_M");
    v = s ? atoi(s) : 8;
    if (v < 1) v = 8;
  }
  return v;
}

// Pair split of the last partial wave of int8 wide tiles (OZK_GEMM_SPLIT,
// default on; 0 deals whole tiles round-robin only).
static bool split_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* s = getenv("OZK_GEMM_SPLIT");
    v = (s && s[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

// CTA-pair tiles are the default for wide outputs; OZK_GEMM_PAIR=0 selects
// single-CTA tiles (kept for comparison and as a fallback).
static bool pair_mode_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* s = getenv("OZK_GEMM_PAIR");
    v = (s && s[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

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

// Tensor map over a [depth][rows][k_pad] slice stack (BF16, or int8 codes
// with s8), box of 128 bytes x box_rows.
int make_slice_map(CUtensorMap* map, const void* base, int64_t k_pad, int64_t rows, int depth,
                   int box_rows, bool s8) {
  if (((uintptr_t)base & 15) != 0) return set_error(OZK_ERR_ARG, "slice buffer not 16-byte aligned");
  int rc = get_encode_fn();
  if (rc) return rc;
  const int64_t esz = s8 ? 1 : 2;
  cuuint64_t dims[3] = {(cuuint64_t)k_pad, (cuuint64_t)rows, (cuuint64_t)depth};
  cuuint64_t strides[2] = {(cuuint64_t)(k_pad * esz), (cuuint64_t)(k_pad * esz * rows)};
  cuuint32_t box[3] = {(cuuint32_t)(s8 ? kS8KB : OZK_KB), (cuuint32_t)box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(map, s8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                        3, (void*)base, dims, strides, box,
                        estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(OZK_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return OZK_OK;
}

template <int BN, bool PAIR, bool S8 = false>
static int launch_bn(const CUtensorMap& ma, const CUtensorMap& mb, const PairList& pl,
                     const GemmArgs& ga, int dev, cudaStream_t stream) {
  using Cfg = GemmCfg<BN, PAIR>;
  static int configured[64] = {0};
  if (!configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(k_slice_gemm<BN, PAIR, S8>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         Cfg::SMEM_BYTES);
    if (e != cudaSuccess) return set_cuda_error("cudaFuncSetAttribute(k_slice_gemm)", e);
    configured[dev] = 1;
  }
  const int sms = device_sm_count(dev);
  const int per = PAIR ? 2 : 1;
  const int max_units = sms / per;
  const int units = (ga.num_tiles < max_units && ga.dp_tiles == ga.num_tiles) ? ga.num_tiles
                                                                             : max_units;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(units * per));
  cfg.blockDim = dim3(Cfg::THREADS);
  cfg.dynamicSmemBytes = Cfg::SMEM_BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = per;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  GemmArgs gl = ga;
  // Diagnostics allocate their counters on first use; calls without the state
  // scratch (the allocation-free entry point among them) record none.
  if (stats_enabled() && ga.state) {
    if (!g_stats_dev[dev]) cudaMalloc(&g_stats_dev[dev], 8 * 1024 * sizeof(unsigned long long));
    cudaMemsetAsync(g_stats_dev[dev], 0, 8 * 1024 * sizeof(unsigned long long), stream);
    gl.stats = g_stats_dev[dev];
    g_stats_ctas[dev] = units * per;
    g_stats_last_dev = dev;
  }
  cudaError_t e = cudaLaunchKernelEx(&cfg, k_slice_gemm<BN, PAIR, S8>, ma, mb, pl, gl);
  return e == cudaSuccess ? OZK_OK : set_cuda_error("k_slice_gemm launch", e);
}

// State scratch of the 256-wide tiles: the per-CTA running sums, a 4 KB
// header (the pacing counter at 0, the split tiles' counters from 256), then
// the split tiles' int64 sums, one 256 x 256 tile per CTA pair at most.  The
// wide kernel needs the first two parts; the pair split needs all three.
static size_t gemm_state_sums_bytes(int dev) {
  return (size_t)device_sm_count(dev) * GemmCfg<256, true>::STATE_PER_CTA * sizeof(double);
}
static constexpr size_t kStateHeader = 4096;
static constexpr size_t kSkCountOffset = 256;
static size_t gemm_split_bytes(int dev) {
  return (size_t)(device_sm_count(dev) / 2) * 2 * GemmCfg<256, true>::STATE_PER_CTA * sizeof(long long);
}
static size_t gemm_state_base_bytes(int dev) { return gemm_state_sums_bytes(dev) + kStateHeader; }

size_t gemm_state_bytes(int dev) { return gemm_state_base_bytes(dev) + gemm_split_bytes(dev); }

// Pacing slack in pairs (OZK_GEMM_PACE, default 1; 0 = off).  Measured on
// B200 at 8192^3 with int8 slices: slack 1 cuts the GEMM's DRAM reads from
// 43 GB to 11 GB per launch (tiles that share panels stay within about one
// pair of each other, so the panels are still in L2), which under the 1 kW
// power cap lets the clock rise: 13.5 ms -> 11.1 ms per launch.
static int pace_slack() {
  static int v = -1;
  if (v < 0) {
    const char* s = getenv("OZK_GEMM_PACE");
    v = s ? atoi(s) : 1;
    if (v < 0) v = 0;
  }
  return v;
}

// The running sums are marked evict_last; that priority applies inside the
// context's persisting-L2 set-aside.  The set-aside is a limit of the whole
// CUDA context, so the library leaves it as the caller has it: with the
// context's own limit (23.7 MB on this pool's B200s) the 8192^3 slice GEMM
// measured within 2.5% of a set-aside that holds all the sums, while changing
// the limit around each launch (and putting it back) stalled the overlapped
// copy pipelines (cudaDeviceSetLimit waits for the device).  Opt-ins:
// OZK_L2_PERSIST=sticky raises it once per device to hold the sums (about
// 46 MB) and keeps it, OZK_L2_PERSIST=<MB> raises it once to that size;
// ozk_set_l2_persisting sets it explicitly.
struct L2Scope {
  void raise(int dev, cudaStream_t stream, size_t sums_bytes) {
    static int done[64] = {0};
    const char* env = getenv("OZK_L2_PERSIST");
    if (!env || dev < 0 || dev >= 64 || done[dev]) return;
    size_t want = sums_bytes + (8u << 20);
    if (strcmp(env, "sticky") != 0) {
      const long mb = atol(env);
      if (mb <= 0) return;
      want = (size_t)mb << 20;
    }
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(stream, &cap) != cudaSuccess || cap != cudaStreamCaptureStatusNone)
      return;  // a limit change is not a capturable operation; try a later launch
    done[dev] = 1;
    size_t cur = 0;
    int mx = 0;
    if (cudaDeviceGetLimit(&cur, cudaLimitPersistingL2CacheSize) != cudaSuccess ||
        cudaDeviceGetAttribute(&mx, cudaDevAttrMaxPersistingL2CacheSize, dev) != cudaSuccess)
      return;
    if (want > (size_t)mx) want = (size_t)mx;
    if (cur < want) cudaDeviceSetLimit(cudaLimitPersistingL2CacheSize, want);
  }
};

int launch_slice_gemm(const uint16_t* SA, const int32_t* eA, int nA, const uint16_t* SB,
                      const int32_t* eB, int nB, int64_t N, int64_t M, int64_t k_pad,
                      const uint8_t* pair_a, const uint8_t* pair_b, int n_pairs, int mode,
                      int symmetric, double alpha, double beta, const double* Cin, int64_t ldcin,
                      double* C, int64_t ldc, float* products, double* state, size_t state_bytes,
                      int rho, int32_t* status, cudaStream_t stream) {
  return launch_slice_gemm_ex(SA, eA, nA, SB, eB, nB, N, M, k_pad, pair_a, pair_b, n_pairs, mode,
                              symmetric, alpha, beta, Cin, ldcin, C, ldc, products, state,
                              state_bytes, rho, status, false, nullptr, 0, stream);
}

bool slice_gemm_s8_eligible(int64_t N, int64_t M, int64_t k_pad, int mode, int rho,
                            size_t state_bytes) {
  int dev;
  cudaGetDevice(&dev);
  return mode == OZK_ACC_FIXED && rho >= kS8MinRho && N >= 256 && M >= 256 && k_pad > 0 &&
         k_pad % kS8KB == 0 && k_pad <= 65536 && state_bytes >= gemm_state_base_bytes(dev) &&
         pair_mode_enabled();
}

int launch_slice_gemm_ex(const void* SA, const int32_t* eA, int nA, const void* SB,
                         const int32_t* eB, int nB, int64_t N, int64_t M, int64_t k_pad,
                         const uint8_t* pair_a, const uint8_t* pair_b, int n_pairs, int mode,
                         int symmetric, double alpha, double beta, const double* Cin,
                         int64_t ldcin, double* C, int64_t ldc, float* products, double* state,
                         size_t state_bytes, int rho, int32_t* status, bool s8,
                         const int32_t* gate, int gate_want, cudaStream_t stream,
                         long long* C64) {
  if (N == 0 || M == 0) return OZK_OK;
  if (C64 && (!s8 || mode != OZK_ACC_FIXED))
    return set_error(OZK_ERR_UNSUPPORTED, "raw int64 sums come from the int8 fixed-point GEMM only");
  L2Scope l2;  // the persisting-L2 opt-ins (OZK_L2_PERSIST)
  if (n_pairs < 1 || n_pairs > OZK_MAX_PAIRS) return set_error(OZK_ERR_ARG, "n_pairs out of range");
  if (k_pad <= 0 || k_pad % OZK_KB) return set_error(OZK_ERR_ARG, "k_pad must be a positive multiple of 64");
  if (s8 && !slice_gemm_s8_eligible(N, M, k_pad, mode, rho, state_bytes))
    return set_error(OZK_ERR_UNSUPPORTED,
                     "int8 slices need OZK_ACC_FIXED, rho >= %d, N and M >= 256, k_pad a multiple of "
                     "%d up to 65536 and the GEMM state scratch", kS8MinRho, kS8KB);
  if (nA < 1 || nA > OZK_MAX_SLICES || nB < 1 || nB > OZK_MAX_SLICES)
    return set_error(OZK_ERR_ARG, "slice counts out of range");
  for (int p = 0; p < n_pairs; ++p)
    if (pair_a[p] >= nA || pair_b[p] >= nB) return set_error(OZK_ERR_ARG, "pair index out of range");
  if (mode != OZK_ACC_F64 && mode != OZK_ACC_PRODUCTS && mode != OZK_ACC_FIXED)
    return set_error(OZK_ERR_ARG, "bad mode");
  if (mode != OZK_ACC_PRODUCTS && !C && !C64) return set_error(OZK_ERR_ARG, "C is NULL");
  if (mode == OZK_ACC_FIXED && (rho < 1 || rho > 30))
    return set_error(OZK_ERR_ARG, "OZK_ACC_FIXED needs the extraction rho");
  if (mode == OZK_ACC_PRODUCTS && !products) return set_error(OZK_ERR_ARG, "products is NULL");
  if (beta != 0.0 && !Cin) return set_error(OZK_ERR_ARG, "Cin is NULL with beta != 0");
  if (symmetric && (N != M || SA != SB || eA != eB || mode == OZK_ACC_PRODUCTS))
    return set_error(OZK_ERR_ARG, "symmetric mode needs one operand, N == M and FP64 output");
  if (N > (int64_t)1 << 31 || M > (int64_t)1 << 31) return set_error(OZK_ERR_ARG, "dimension too large");
  int rc = get_encode_fn();
  if (rc) return rc;
  int dev;
  cudaGetDevice(&dev);

  // Tile choice: 256 x 256 on CTA pairs (FP64 sums in the per-CTA state
  // scratch) for large FP64 outputs; 256 x 128 on CTA pairs (sums in TMEM)
  // when no scratch is given; narrow single-CTA tiles for narrow outputs
  // (e.g. residual right-hand sides).
  const bool wide = s8 || (mode != OZK_ACC_PRODUCTS && N >= 256 && M >= 256 && state &&
                          state_bytes >= gemm_state_base_bytes(dev) && pair_mode_enabled());
  const int BN = wide ? 256 : (M <= 16 ? 16 : (M <= 32 ? 32 : (M <= 64 ? 64 : 128)));
  const int bn = (symmetric && !wide) ? 128 : BN;
  const bool pair = wide || (!symmetric && bn == 128 && pair_mode_enabled());
  const int tile_m = pair ? 2 * kBM : kBM;
  CUtensorMap ma, mb;
  if ((rc = make_slice_map(&ma, SA, k_pad, N, nA, kBM, s8))) return rc;
  if ((rc = make_slice_map(&mb, SB, k_pad, M, nB, pair ? bn / 2 : bn, s8))) return rc;

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
  ga.num_kb = (int)(k_pad / (s8 ? kS8KB : OZK_KB));
  ga.nB = nB;
  ga.tiles_m = (int)((N + tile_m - 1) / tile_m);
  ga.tiles_n = (int)((M + bn - 1) / bn);
  ga.num_tiles = symmetric ? ga.tiles_m * (ga.tiles_m + 1) / 2 : ga.tiles_m * ga.tiles_n;
  ga.group_m = group_m_rows();
  ga.mode = mode;
  ga.symmetric = symmetric;
  ga.alpha = alpha;
  ga.beta = beta;
  ga.Cin = Cin;
  ga.ldcin = ldcin;
  ga.C = C;
  ga.C64 = C64;
  ga.ldc = ldc;
  ga.products = products;
  ga.status = status;
  ga.budget_ns = wait_budget_ns();
  ga.state = state;
  ga.c_vec = C && ((uintptr_t)C % 32 == 0) && (ldc % 4 == 0);
  ga.fixed = mode == OZK_ACC_FIXED;
  ga.fix_off = -150 - 2 * (rho - 24) + kFixFrac;
  ga.fix_scale = 2 * (rho - 24) - kFixFrac;
  ga.prefetch = prefetch_distance();
  ga.gate = gate;
  ga.gate_want = gate_want;
  if (wide || s8) {
    l2.raise(dev, stream, gemm_state_sums_bytes(dev));
    // pairs long enough for the pacing handshake to be negligible
    if (pace_slack() > 0 && k_pad >= 2048) {
      ga.pace = reinterpret_cast<unsigned long long*>(reinterpret_cast<char*>(state) +
                                                      gemm_state_sums_bytes(dev));
      ga.pace_slack = pace_slack();
      ga.pace_budget_ns = 50000;  // a stalled peer costs at most 50 us per pair
      cudaError_t e = cudaMemsetAsync(ga.pace, 0, sizeof(unsigned long long), stream);
      if (e != cudaSuccess) return set_cuda_error("cudaMemsetAsync(pace)", e);
    }
  }
  ga.dp_tiles = ga.num_tiles;
  if (s8) {
    // Pair split of the last wave of tiles (exact: the partial sums are
    // integers), when the scratch holds the split tiles' sums.  With r tiles
    // left for U units, chunks of 1/k of a tile's pairs take ceil(r k / U) / k
    // of a tile's time instead of one: the k <= 8 that minimises it (the
    // smallest on ties), if that saves at least a tenth.  (Splitting every
    // tile into one chunk per pair-item share, with the units on different
    // pairs at once, lost 5% at the 65536 x 4096 gram: no panel reuse.)
    const int units = device_sm_count(dev) / 2;
    const int rem = ga.num_tiles % units;
    int chunks = 1;
    if (rem) {
      double best = 1.0;
      for (int k = 2; k <= 8 && k <= n_pairs; ++k) {
        const double cost = (double)((rem * k + units - 1) / units) / k;
        if (cost < best - 1e-9) {
          best = cost;
          chunks = k;
        }
      }
      if (best > 0.9) chunks = 1;
    }
    if (split_enabled() && chunks >= 2 && state_bytes >= gemm_state_bytes(dev)) {
      ga.dp_tiles = ga.num_tiles - rem;
      ga.sk_chunks = chunks;
      char* hdr = reinterpret_cast<char*>(state) + gemm_state_sums_bytes(dev);
      ga.sk_count = reinterpret_cast<unsigned int*>(hdr + kSkCountOffset);
      ga.sk_sum = reinterpret_cast<long long*>(hdr + kStateHeader);
      cudaError_t e = cudaMemsetAsync(ga.sk_count, 0, (size_t)rem * 2 * sizeof(unsigned int), stream);
      if (e == cudaSuccess)
        e = cudaMemsetAsync(ga.sk_sum, 0,
                            (size_t)rem * 2 * GemmCfg<256, true>::STATE_PER_CTA * sizeof(long long),
                            stream);
      if (e != cudaSuccess) return set_cuda_error("cudaMemsetAsync(split sums)", e);
    }
    return launch_bn<256, true, true>(ma, mb, pl, ga, dev, stream);
  }
  if (wide) return launch_bn<256, true>(ma, mb, pl, ga, dev, stream);
  switch (bn) {
    case 16: return launch_bn<16, false>(ma, mb, pl, ga, dev, stream);
    case 32: return launch_bn<32, false>(ma, mb, pl, ga, dev, stream);
    case 64: return launch_bn<64, false>(ma, mb, pl, ga, dev, stream);
    default:
      return pair ? launch_bn<128, true>(ma, mb, pl, ga, dev, stream)
                  : launch_bn<128, false>(ma, mb, pl, ga, dev, stream);
  }
}

}  // namespace ozk

extern "C" int ozk_gemm_stats(unsigned long long* out8) {
  using namespace ozk;
  if (!out8) return OZK_ERR_ARG;
  for (int i = 0; i < 8; ++i) out8[i] = 0;
  const int dev = g_stats_last_dev;
  if (dev < 0 || !g_stats_dev[dev]) return OZK_ERR_UNSUPPORTED;
  static unsigned long long h[8 * 1024];
  cudaDeviceSynchronize();
  cudaMemcpy(h, g_stats_dev[dev], sizeof(h), cudaMemcpyDeviceToHost);
  for (int c = 0; c < g_stats_ctas[dev] && c < 1024; ++c)
    for (int i = 0; i < 8; ++i) out8[i] += h[8 * c + i];
  return g_stats_ctas[dev];
}

// ---------------------------------------------------------------- self-test

namespace ozk {

// One CTA waits, through the same bounded wait every kernel uses, on an
// mbarrier that nothing arrives at; the wait gives up after budget_ns and
// raises OZK_FLAG_TIMEOUT.  Exercises the timeout path without a fault.
__global__ void k_selftest_timeout(int32_t* status, uint64_t budget_ns, int32_t* out_ok) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const bool ok = mbar_wait(&bar, 0, &abort_flag, status, budget_ns);
    *out_ok = ok ? 1 : 0;
  }
}

}  // namespace ozk

extern "C" int ozk_selftest_timeout(int budget_ms, int32_t* status_dev, int32_t* ok_dev,
                                    void* stream) {
  using namespace ozk;
  if (!status_dev || !ok_dev || budget_ms < 1 || budget_ms > 10000)
    return set_error(OZK_ERR_ARG, "bad self-test arguments");
  k_selftest_timeout<<<1, 32, 0, (cudaStream_t)stream>>>(status_dev, (uint64_t)budget_ms * 1000000ull,
                                                        ok_dev);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? OZK_OK : set_cuda_error("k_selftest_timeout launch", e);
}
