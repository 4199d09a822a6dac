// Multi-GPU Ozaki matmul behind the C ABI: ozk_context (one NCCL communicator
// per local GPU) and ozk_matmul_f64_multi.
//
// The reference has no multi-device code (its operators are single-device
// jitted functions, ozaki_jax/matmul.py:514-540); this is the partitioning of
// the on-device pipeline across the GPUs of one node.  Global rank r of P owns
// rows [r N / P, (r+1) N / P) of A and C.  Row extraction is row-local, so each
// rank's slices of A, and its rows of C, are bit-identical to the single-GPU
// ones.  Every rank needs the slices of all of B; they arrive in one of three
// ways (b_mode):
//   OZK_B_REPLICATED  every rank holds all of B and extracts it locally;
//   OZK_B_ROOT        rank 0 holds B, extracts it and broadcasts the slice
//                     stack and exponents over NCCL (NVLink);
//   OZK_B_COLUMNS     rank r holds the columns [r mc, min(M, (r+1) mc)) of B,
//                     mc = ceil(M / P), extracts them, and the slice stacks are
//                     all-gathered over NCCL.
// Column extraction is column-local too, so every variant gives every rank
// exactly the single-GPU slices of B.
//
// Flags: each rank's int8-code failure word and OZK_FLAG_* status word are
// all-gathered in the same NCCL group as B's slices, and every rank reduces
// them alike: the int8 GEMM is skipped on every rank if any code failed
// anywhere, and every rank reports any rank's non-finite input, as a single
// GPU would.  Then (blocking calls) every rank sees the same failure and runs
// the same BF16 pass, so all ranks always take the same collective steps.
//
// NCCL is loaded at run time (dlopen of libnccl.so.2, reusing an already
// loaded copy, such as PyTorch's), so the rest of the library does not depend
// on it.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <chrono>
#include <mutex>
#include <thread>
#include <vector>

#include "ozaki_b200.h"
#include "ozk_fixed.cuh"
#include "ozk_internal.h"

namespace ozk {
namespace {

struct NcclApi {
  decltype(&ncclGetUniqueId) GetUniqueId = nullptr;
  decltype(&ncclCommInitRank) CommInitRank = nullptr;
  decltype(&ncclCommInitAll) CommInitAll = nullptr;
  decltype(&ncclCommDestroy) CommDestroy = nullptr;
  decltype(&ncclCommAbort) CommAbort = nullptr;
  decltype(&ncclCommGetAsyncError) CommGetAsyncError = nullptr;
  decltype(&ncclGetErrorString) GetErrorString = nullptr;
  decltype(&ncclAllGather) AllGather = nullptr;
  decltype(&ncclBroadcast) Broadcast = nullptr;
  decltype(&ncclAllReduce) AllReduce = nullptr;
  decltype(&ncclGroupStart) GroupStart = nullptr;
  decltype(&ncclGroupEnd) GroupEnd = nullptr;
  bool ok = false;
  char why[256] = "";
};

const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    const char* names[] = {"libnccl.so.2", "libnccl.so"};
    void* h = nullptr;
    for (const char* n : names)
      if ((h = dlopen(n, RTLD_NOW | RTLD_NOLOAD))) break;
    if (!h)
      for (const char* n : names)
        if ((h = dlopen(n, RTLD_NOW | RTLD_GLOBAL))) break;
    if (!h) {
      const char* e = dlerror();
      snprintf(api.why, sizeof(api.why), "cannot load libnccl.so.2: %s", e ? e : "not found");
      return;
    }
#define OZK_SYM(f)                                                           \
  api.f = reinterpret_cast<decltype(api.f)>(dlsym(h, "nccl" #f));           \
  if (!api.f) {                                                              \
    snprintf(api.why, sizeof(api.why), "libnccl.so.2 lacks nccl%s", #f);     \
    return;                                                                  \
  }
    OZK_SYM(GetUniqueId)
    OZK_SYM(CommInitRank)
    OZK_SYM(CommInitAll)
    OZK_SYM(CommDestroy)
    OZK_SYM(CommAbort)
    OZK_SYM(CommGetAsyncError)
    OZK_SYM(GetErrorString)
    OZK_SYM(AllGather)
    OZK_SYM(Broadcast)
    OZK_SYM(AllReduce)
    OZK_SYM(GroupStart)
    OZK_SYM(GroupEnd)
#undef OZK_SYM
    api.ok = true;
  });
  return api;
}

int nccl_error(const char* what, ncclResult_t r) {
  return set_error(OZK_ERR_NCCL, "%s: %s", what, nccl().GetErrorString(r));
}

// One pass's flags: word 0 the int8-code failure, word 1 the OZK_FLAG_* bits.
// After the all-gather, every rank ORs all ranks' words: the gate (any code
// failed) and the status.  `redo` is OR-ed into the status when the int8 pass
// failed and the caller asked not to wait (its C was not written).
__global__ void k_reduce_flags(const int32_t* all, int nranks, int32_t* gate, int32_t* status_out,
                               int32_t redo) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  int32_t f = 0, st = 0;
  for (int r = 0; r < nranks; ++r) {
    f |= all[2 * r];
    st |= all[2 * r + 1];
  }
  *gate = f;
  const int32_t add = st | (f ? redo : 0);
  if (status_out && add) atomicOr(status_out, add);
}

// G = the FP64 values of the reduced int64 sums P (upper triangle, K x K):
// G[i][j] = G[j][i] = P[i][j] * 2^(e0[i] + e0[j] + fix_scale), 32 x 32 tiles
// I <= J through shared memory so both writes are coalesced.  Runs only when
// *gate == 0 (no int8 code failed on any rank).
__global__ void __launch_bounds__(256) k_gram_finalize(const long long* __restrict__ P,
                                                       int64_t K, const int32_t* __restrict__ e0,
                                                       int fix_scale, const int32_t* gate,
                                                       double* __restrict__ G, int64_t ldg) {
  if (*(volatile const int32_t*)gate) return;
  __shared__ double tile[32][33];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int64_t nt = (K + 31) / 32;
  for (int64_t b = blockIdx.x; b < nt * nt; b += gridDim.x) {
    const int64_t ti = b / nt, tj = b % nt;
    if (tj < ti) continue;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int64_t i = ti * 32 + ty + 8 * r, j = tj * 32 + tx;
      if (i < K && j < K && j >= i) {
        const double v = fixed_value(P[i * K + j], e0[i] + e0[j] + fix_scale);
        G[i * ldg + j] = v;
        tile[ty + 8 * r][tx] = v;
      }
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int64_t j = tj * 32 + ty + 8 * r, i = ti * 32 + tx;  // G[j][i] = G[i][j]
      if (i < K && j < K && j >= i) G[j * ldg + i] = tile[tx][ty + 8 * r];
    }
    __syncthreads();
  }
}

struct DevState {
  int device = 0;
  int rank = 0;
  ncclComm_t comm = nullptr;
  void* buf = nullptr;
  size_t buf_bytes = 0;
};

size_t a256(size_t x) { return (x + 255) & ~(size_t)255; }

}  // namespace
}  // namespace ozk

struct ozk_context {
  int nranks = 0;
  bool aborted = false;
  std::vector<ozk::DevState> dev;
};

namespace ozk {
namespace {

// Per-device workspace of one pass (elem = 1 for int8 codes, 2 for BF16).
struct MultiWs {
  char* SA;
  char* SB;      // [nS][Mp][kp]: Mp = P mc (columns mode) or M
  char* SBc;     // compact [nS][M][kp] when Mp != M (else == SB)
  int32_t* eA;
  int32_t* eB;   // [nS][Mp]
  int32_t* eBc;  // compact [nS][M]
  char* Bt;      // columns mode: this rank's [nS][mc][kp] (+ one slice of slack)
  int32_t* et;   // columns mode: [nS][mc] (+ slack)
  double* BT;    // FP64 transposed scratch of the extracted columns
  int32_t* flags_send;  // [2]
  int32_t* flags_all;   // [2 P]
  int32_t* gate;
  double* state;
  size_t state_bytes;
  size_t bytes;
};

MultiWs multi_layout(char* base, int64_t rows, int64_t K, int64_t M, int64_t Mp, int64_t mc,
                     int64_t kp, int elem, int nS, int P, int mode, int rank,
                     size_t state_bytes) {
  MultiWs w;
  size_t off = 0;
  auto take = [&](size_t n) {
    char* p = base ? base + off : nullptr;
    off += a256(n);
    return p;
  };
  w.SA = take((size_t)nS * rows * kp * elem);
  w.SB = take((size_t)nS * Mp * kp * elem);
  w.SBc = Mp != M ? take((size_t)nS * M * kp * elem) : w.SB;
  w.eA = (int32_t*)take((size_t)nS * rows * 4);
  w.eB = (int32_t*)take((size_t)nS * Mp * 4);
  w.eBc = Mp != M ? (int32_t*)take((size_t)nS * M * 4) : w.eB;
  const bool cols = mode == OZK_B_COLUMNS;
  w.Bt = cols ? take((size_t)(nS + 1) * mc * kp * elem) : nullptr;
  w.et = cols ? (int32_t*)take((size_t)(nS + 1) * mc * 4) : nullptr;
  // only ranks that extract columns of B need the transposed FP64 scratch
  const int64_t bt_lines = cols ? mc : (mode == OZK_B_ROOT && rank != 0 ? 0 : M);
  w.BT = (double*)take((size_t)bt_lines * K * 8);
  w.flags_send = (int32_t*)take(8);
  w.flags_all = (int32_t*)take((size_t)8 * P);
  w.gate = (int32_t*)take(4);
  w.state = state_bytes ? (double*)take(state_bytes) : nullptr;
  w.state_bytes = state_bytes;
  w.bytes = off;
  return w;
}

int grow(DevState& d, size_t need) {
  if (d.buf_bytes >= need) return OZK_OK;
  if (d.buf) cudaFree(d.buf);  // synchronises the device: no call still uses it
  d.buf = nullptr;
  d.buf_bytes = 0;
  cudaError_t e = cudaMalloc(&d.buf, need);
  if (e != cudaSuccess) return set_cuda_error("cudaMalloc(multi-GPU workspace)", e);
  d.buf_bytes = need;
  return OZK_OK;
}

struct MultiArgs {
  const double* const* A;
  const int64_t* lda;
  const double* const* B;
  const int64_t* ldb;
  double* const* C;
  const int64_t* ldc;
  int64_t N, K, M;
  int n_hi, n_lo, mode, rho;
  cudaStream_t* s;
  int32_t* const* status;
};

int64_t rows_of(int64_t N, int r, int P) { return (r + 1) * N / P - r * N / P; }

int64_t cols_of(int64_t M, int64_t mc, int r) {
  const int64_t c0 = r * mc;
  return c0 >= M ? 0 : (M - c0 < mc ? M - c0 : mc);
}

uint64_t multi_timeout_ms() {
  const char* s = getenv("OZK_NCCL_TIMEOUT_MS");
  const long v = s ? atol(s) : 0;
  return v > 0 ? (uint64_t)v : 300000ull;
}

// Waits for every local stream with a deadline, watching NCCL for
// asynchronous errors; on a failure or at the deadline every communicator of
// the context is aborted (the context is unusable afterwards).  The first
// 2 ms poll without sleeping, so a short step pays no sleep granularity.
int wait_all(ozk_context* ctx, cudaStream_t* s) {
  const auto t0 = std::chrono::steady_clock::now();
  const uint64_t budget = multi_timeout_ms();
  const NcclApi& api = nccl();
  for (size_t i = 0; i < ctx->dev.size(); ++i) {
    cudaSetDevice(ctx->dev[i].device);
    for (;;) {
      cudaError_t q = cudaStreamQuery(s[i]);
      if (q == cudaSuccess) break;
      if (q != cudaErrorNotReady) return set_cuda_error("cudaStreamQuery", q);
      ncclResult_t ar = ncclSuccess;
      api.CommGetAsyncError(ctx->dev[i].comm, &ar);
      const uint64_t ms = (uint64_t)std::chrono::duration_cast<std::chrono::milliseconds>(
                              std::chrono::steady_clock::now() - t0)
                              .count();
      if ((ar != ncclSuccess && ar != ncclInProgress) || ms > budget) {
        for (auto& d : ctx->dev)
          if (d.comm) api.CommAbort(d.comm);
        for (auto& d : ctx->dev) d.comm = nullptr;
        ctx->aborted = true;
        if (ar != ncclSuccess && ar != ncclInProgress) return nccl_error("collective failed", ar);
        return set_error(OZK_ERR_TIMEOUT,
                         "a collective did not finish within %llu ms (OZK_NCCL_TIMEOUT_MS); the "
                         "context was aborted",
                         (unsigned long long)budget);
      }
      if (ms < 2) std::this_thread::yield();
      else std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
  }
  return OZK_OK;
}

// One pass over all local devices: extraction, the NCCL group (B's slices and
// the flags), the flag reduction and the GEMM.  s8: int8 codes and the int8
// GEMM gated on the global failure word; else BF16 slices, ungated.
int run_pass(ozk_context* ctx, const MultiArgs& a, bool s8, int32_t redo) {
  const int P = ctx->nranks;
  const int nS = a.n_hi + a.n_lo;
  const int elem = s8 ? 1 : 2;
  const int64_t kp = s8 ? round_up(a.K, kS8KB) : round_up(a.K, OZK_KB);
  const int64_t mc = (a.M + P - 1) / P;
  const int64_t Mp = a.mode == OZK_B_COLUMNS ? mc * P : a.M;
  uint8_t pa[OZK_MAX_PAIRS], pb[OZK_MAX_PAIRS];
  const int np = ozk_pair_schedule_snake(a.n_hi, a.n_lo, pa, pb, OZK_MAX_PAIRS);
  if (np < 0) return np;
  const NcclApi& api = nccl();
  const int nl = (int)ctx->dev.size();
  std::vector<MultiWs> ws(nl);
  int rc;
  // 1. extraction on every local device
  for (int i = 0; i < nl; ++i) {
    DevState& d = ctx->dev[i];
    cudaSetDevice(d.device);
    const int r = d.rank;
    const int64_t rows = rows_of(a.N, r, P);
    const size_t sb = gemm_state_bytes(d.device);
    const size_t need =
        multi_layout(nullptr, rows, a.K, a.M, Mp, mc, kp, elem, nS, P, a.mode, r, sb).bytes;
    if ((rc = grow(d, need))) return rc;
    MultiWs& w = ws[i];
    w = multi_layout((char*)d.buf, rows, a.K, a.M, Mp, mc, kp, elem, nS, P, a.mode, r, sb);
    cudaStream_t s = a.s[i];
    cudaError_t e = cudaMemsetAsync(w.flags_send, 0, 8, s);
    if (e != cudaSuccess) return set_cuda_error("cudaMemsetAsync(flags)", e);
    int32_t* fail = w.flags_send;
    int32_t* st = w.flags_send + 1;
    if (rows > 0) {
      rc = s8 ? launch_extract_rows_s8(a.A[i], a.lda[i], rows, a.K, a.rho, a.n_hi, a.n_lo,
                                       (int8_t*)w.SA, kp, w.eA, st, fail, s)
              : launch_extract_rows(a.A[i], a.lda[i], rows, a.K, a.rho, a.n_hi, a.n_lo,
                                    (uint16_t*)w.SA, kp, w.eA, st, s);
      if (rc) return rc;
    }
    const bool whole_b = a.mode == OZK_B_REPLICATED || (a.mode == OZK_B_ROOT && r == 0);
    if (whole_b) {
      rc = s8 ? launch_extract_cols_s8(a.B[i], a.ldb[i], a.K, a.M, a.rho, a.n_hi, a.n_lo,
                                       (int8_t*)w.SB, kp, w.eB, st, fail, w.BT, s)
              : launch_extract_cols(a.B[i], a.ldb[i], a.K, a.M, a.rho, a.n_hi, a.n_lo,
                                    (uint16_t*)w.SB, kp, w.eB, st, w.BT, s);
      if (rc) return rc;
    } else if (a.mode == OZK_B_COLUMNS) {
      const int64_t mr = cols_of(a.M, mc, r);
      if (mr > 0) {
        rc = s8 ? launch_extract_cols_s8(a.B[i], a.ldb[i], a.K, mr, a.rho, a.n_hi, a.n_lo,
                                         (int8_t*)w.Bt, kp, w.et, st, fail, w.BT, s)
                : launch_extract_cols(a.B[i], a.ldb[i], a.K, mr, a.rho, a.n_hi, a.n_lo,
                                      (uint16_t*)w.Bt, kp, w.et, st, w.BT, s);
        if (rc) return rc;
      }
    }
  }
  // 2. B's slices and every rank's flags, in one group
  ncclResult_t nr = api.GroupStart();
  if (nr != ncclSuccess) return nccl_error("ncclGroupStart", nr);
  for (int i = 0; i < nl && nr == ncclSuccess; ++i) {
    DevState& d = ctx->dev[i];
    MultiWs& w = ws[i];
    cudaStream_t s = a.s[i];
    if (a.mode == OZK_B_ROOT) {
      nr = api.Broadcast(w.SB, w.SB, (size_t)nS * a.M * kp * elem, ncclInt8, 0, d.comm, s);
      if (nr == ncclSuccess)
        nr = api.Broadcast(w.eB, w.eB, (size_t)nS * a.M, ncclInt32, 0, d.comm, s);
    } else if (a.mode == OZK_B_COLUMNS) {
      // this rank's extracted columns are [nS][mr][kp]; each slice's chunk has
      // mc lines (a short last rank sends slack, which lands beyond column M)
      const int64_t mr = cols_of(a.M, mc, d.rank);
      for (int t = 0; t < nS && nr == ncclSuccess; ++t) {
        nr = api.AllGather(w.Bt + (size_t)t * mr * kp * elem, w.SB + (size_t)t * Mp * kp * elem,
                           (size_t)mc * kp * elem, ncclInt8, d.comm, s);
        if (nr == ncclSuccess)
          nr = api.AllGather(w.et + (size_t)t * mr, w.eB + (size_t)t * Mp, (size_t)mc, ncclInt32,
                             d.comm, s);
      }
    }
    if (nr == ncclSuccess) nr = api.AllGather(w.flags_send, w.flags_all, 2, ncclInt32, d.comm, s);
  }
  ncclResult_t ge = api.GroupEnd();
  if (nr != ncclSuccess) return nccl_error("enqueueing B's slices", nr);
  if (ge != ncclSuccess) return nccl_error("ncclGroupEnd", ge);
  // 3. flags, compaction of a ragged column split, the GEMM
  for (int i = 0; i < nl; ++i) {
    DevState& d = ctx->dev[i];
    cudaSetDevice(d.device);
    MultiWs& w = ws[i];
    cudaStream_t s = a.s[i];
    const int64_t rows = rows_of(a.N, d.rank, P);
    k_reduce_flags<<<1, 32, 0, s>>>(w.flags_all, P, w.gate, a.status ? a.status[i] : nullptr,
                                    redo);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_cuda_error("k_reduce_flags launch", e);
    if (Mp != a.M) {
      e = cudaMemcpy2DAsync(w.SBc, (size_t)a.M * kp * elem, w.SB, (size_t)Mp * kp * elem,
                            (size_t)a.M * kp * elem, (size_t)nS, cudaMemcpyDeviceToDevice, s);
      if (e == cudaSuccess)
        e = cudaMemcpy2DAsync(w.eBc, (size_t)a.M * 4, w.eB, (size_t)Mp * 4, (size_t)a.M * 4,
                              (size_t)nS, cudaMemcpyDeviceToDevice, s);
      if (e != cudaSuccess) return set_cuda_error("compacting B's slices", e);
    }
    if (rows == 0) continue;
    rc = launch_slice_gemm_ex(w.SA, w.eA, nS, w.SBc, w.eBc, nS, rows, a.M, kp, pa, pb, np,
                              OZK_ACC_FIXED, 0, 1.0, 0.0, nullptr, 0, a.C[i], a.ldc[i], nullptr,
                              w.state, w.state_bytes, a.rho, a.status ? a.status[i] : nullptr, s8,
                              s8 ? w.gate : nullptr, 0, s);
    if (rc) return rc;
  }
  return OZK_OK;
}

}  // namespace
}  // namespace ozk

using namespace ozk;

extern "C" {

int ozk_nccl_unique_id(void* id_out, size_t len) {
  if (!id_out || len < sizeof(ncclUniqueId))
    return set_error(OZK_ERR_ARG, "the id buffer needs %zu bytes", sizeof(ncclUniqueId));
  const NcclApi& api = nccl();
  if (!api.ok) return set_error(OZK_ERR_NCCL, "%s", api.why);
  ncclUniqueId id;
  ncclResult_t r = api.GetUniqueId(&id);
  if (r != ncclSuccess) return nccl_error("ncclGetUniqueId", r);
  memcpy(id_out, &id, sizeof(id));
  return OZK_OK;
}

int ozk_context_create_rank(ozk_context** ctx, int nranks, int rank, const void* nccl_id,
                            size_t id_len, int device) {
  if (!ctx || !nccl_id || id_len < sizeof(ncclUniqueId) || nranks < 1 || rank < 0 ||
      rank >= nranks || device < 0)
    return set_error(OZK_ERR_ARG, "bad context arguments");
  *ctx = nullptr;
  const NcclApi& api = nccl();
  if (!api.ok) return set_error(OZK_ERR_NCCL, "%s", api.why);
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return set_cuda_error("cudaSetDevice", e);
  ncclUniqueId id;
  memcpy(&id, nccl_id, sizeof(id));
  ncclComm_t comm = nullptr;
  ncclResult_t r = api.CommInitRank(&comm, nranks, id, rank);
  if (r != ncclSuccess) return nccl_error("ncclCommInitRank", r);
  ozk_context* c = new ozk_context;
  c->nranks = nranks;
  DevState d;
  d.device = device;
  d.rank = rank;
  d.comm = comm;
  c->dev.push_back(d);
  *ctx = c;
  return OZK_OK;
}

int ozk_context_create_local(ozk_context** ctx, int ndev, const int* devices) {
  if (!ctx || ndev < 1 || !devices) return set_error(OZK_ERR_ARG, "bad context arguments");
  *ctx = nullptr;
  const NcclApi& api = nccl();
  if (!api.ok) return set_error(OZK_ERR_NCCL, "%s", api.why);
  std::vector<ncclComm_t> comms(ndev, nullptr);
  ncclResult_t r = api.CommInitAll(comms.data(), ndev, devices);
  if (r != ncclSuccess) return nccl_error("ncclCommInitAll", r);
  ozk_context* c = new ozk_context;
  c->nranks = ndev;
  for (int i = 0; i < ndev; ++i) {
    DevState d;
    d.device = devices[i];
    d.rank = i;
    d.comm = comms[i];
    c->dev.push_back(d);
  }
  *ctx = c;
  return OZK_OK;
}

int ozk_context_destroy(ozk_context* ctx) {
  if (!ctx) return OZK_OK;
  const NcclApi& api = nccl();
  int rc = OZK_OK;
  for (auto& d : ctx->dev) {
    cudaSetDevice(d.device);
    if (d.buf) {
      cudaDeviceSynchronize();
      cudaFree(d.buf);
    }
    if (d.comm && api.ok) {
      ncclResult_t r = api.CommDestroy(d.comm);
      if (r != ncclSuccess && !rc) rc = nccl_error("ncclCommDestroy", r);
    }
  }
  delete ctx;
  return rc;
}

int ozk_context_wait(ozk_context* ctx, void* const* streams) {
  if (!ctx) return set_error(OZK_ERR_ARG, "NULL context");
  if (ctx->aborted) return set_error(OZK_ERR_NCCL, "the context was aborted after a failure");
  if (!nccl().ok) return set_error(OZK_ERR_NCCL, "%s", nccl().why);
  std::vector<cudaStream_t> s(ctx->dev.size());
  for (size_t i = 0; i < s.size(); ++i) s[i] = streams ? (cudaStream_t)streams[i] : nullptr;
  return wait_all(ctx, s.data());
}

int ozk_context_info(const ozk_context* ctx, int* nranks, int* first_rank, int* nlocal) {
  if (!ctx) return set_error(OZK_ERR_ARG, "NULL context");
  if (nranks) *nranks = ctx->nranks;
  if (first_rank) *first_rank = ctx->dev.empty() ? -1 : ctx->dev[0].rank;
  if (nlocal) *nlocal = (int)ctx->dev.size();
  return OZK_OK;
}

int ozk_matmul_f64_multi(ozk_context* ctx, const double* const* A, const int64_t* lda,
                         const double* const* B, const int64_t* ldb, double* const* C,
                         const int64_t* ldc, int64_t N, int64_t K, int64_t M, int n_hi, int n_lo,
                         int b_mode, int flags, void* const* streams, int32_t* const* status_dev) {
  if (!ctx) return set_error(OZK_ERR_ARG, "NULL context");
  if (ctx->aborted) return set_error(OZK_ERR_NCCL, "the context was aborted after a failure");
  if (!A || !lda || !C || !ldc) return set_error(OZK_ERR_ARG, "NULL pointer array");
  if (N < 0 || M < 1 || K < 1) return set_error(OZK_ERR_ARG, "bad shape (K, M must be >= 1)");
  if (b_mode != OZK_B_REPLICATED && b_mode != OZK_B_ROOT && b_mode != OZK_B_COLUMNS)
    return set_error(OZK_ERR_ARG, "bad b_mode");
  if (n_hi < 1 || n_lo < 0 || n_hi > OZK_MAX_SIDE || n_lo > OZK_MAX_SIDE)
    return set_error(OZK_ERR_ARG, "n_hi must be in [1,%d] and n_lo in [0,%d]", OZK_MAX_SIDE,
                     OZK_MAX_SIDE);
  const int P = ctx->nranks;
  const int nl = (int)ctx->dev.size();
  const int64_t mc = (M + P - 1) / P;
  for (int i = 0; i < nl; ++i) {
    const int r = ctx->dev[i].rank;
    const int64_t rows = rows_of(N, r, P);
    if (rows > 0 && (!A[i] || lda[i] < K)) return set_error(OZK_ERR_ARG, "A[%d] / lda", i);
    if (rows > 0 && (!C[i] || ldc[i] < M)) return set_error(OZK_ERR_ARG, "C[%d] / ldc", i);
    const bool needs_b = b_mode == OZK_B_REPLICATED || b_mode == OZK_B_COLUMNS ||
                         (b_mode == OZK_B_ROOT && r == 0);
    const int64_t bcols = b_mode == OZK_B_COLUMNS ? cols_of(M, mc, r) : M;
    if (needs_b && bcols > 0 && (!B || !ldb || !B[i] || ldb[i] < bcols))
      return set_error(OZK_ERR_ARG, "B[%d] / ldb", i);
  }
  const int rho = ozk_compute_rho_f32(K);
  int rc = check_bound(K, 24 - rho);
  if (rc) return rc;
  std::vector<cudaStream_t> s(nl);
  for (int i = 0; i < nl; ++i) s[i] = streams ? (cudaStream_t)streams[i] : nullptr;
  MultiArgs a{A, lda, B, ldb, C, ldc, N, K, M, n_hi, n_lo, b_mode, rho, s.data(), status_dev};
  // int8 codes when every rank's GEMM can take them (the same decision on
  // every rank: it depends only on the global shapes)
  const int64_t min_rows = N / P;
  const int64_t k8 = round_up(K, kS8KB);
  cudaSetDevice(ctx->dev[0].device);
  const bool s8 = !(flags & OZK_MULTI_BF16) && s8_enabled() &&
                  slice_gemm_s8_eligible(min_rows, M, k8, OZK_ACC_FIXED, rho,
                                         gemm_state_bytes(ctx->dev[0].device));
  const bool nowait = (flags & OZK_MULTI_NOWAIT) != 0;
  if ((rc = run_pass(ctx, a, s8, nowait ? OZK_FLAG_REDO : 0))) return rc;
  if (nowait) return OZK_OK;
  if ((rc = wait_all(ctx, s.data()))) return rc;
  if (!s8) return OZK_OK;
  // blocking: run the BF16 pass on every rank if any int8 code failed (the
  // gate of the pass, in the first local device's workspace, is global)
  int32_t gate = 0;
  {
    cudaSetDevice(ctx->dev[0].device);
    const int64_t rows = rows_of(N, ctx->dev[0].rank, P);
    const int nS = n_hi + n_lo;
    const int64_t Mp = b_mode == OZK_B_COLUMNS ? mc * P : M;
    MultiWs w = multi_layout((char*)ctx->dev[0].buf, rows, K, M, Mp, mc, k8, 1, nS, P, b_mode,
                             ctx->dev[0].rank, gemm_state_bytes(ctx->dev[0].device));
    cudaError_t e = cudaMemcpy(&gate, w.gate, 4, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return set_cuda_error("reading the gate", e);
  }
  if (!gate) return OZK_OK;
  if ((rc = run_pass(ctx, a, false, 0))) return rc;
  return wait_all(ctx, s.data());
}


int ozk_gram_f64_multi(ozk_context* ctx, const double* const* A, const int64_t* lda, double* const* G,
                       const int64_t* ldg, int64_t N, int64_t K, int n_hi, int n_lo, int flags,
                       void* const* streams, int32_t* const* status_dev) {
  if (!ctx) return set_error(OZK_ERR_ARG, "NULL context");
  if (ctx->aborted) return set_error(OZK_ERR_NCCL, "the context was aborted after a failure");
  if (!A || !lda || !G || !ldg) return set_error(OZK_ERR_ARG, "NULL pointer array");
  if (N < 1 || K < 1) return set_error(OZK_ERR_ARG, "bad shape (N, K must be >= 1)");
  if (n_hi < 1 || n_lo < 0 || n_hi > OZK_MAX_SIDE || n_lo > OZK_MAX_SIDE)
    return set_error(OZK_ERR_ARG, "n_hi must be in [1,%d] and n_lo in [0,%d]", OZK_MAX_SIDE,
                     OZK_MAX_SIDE);
  const NcclApi& api = nccl();
  const int P = ctx->nranks;
  const int nl = (int)ctx->dev.size();
  for (int i = 0; i < nl; ++i) {
    const int64_t rows = rows_of(N, ctx->dev[i].rank, P);
    if (rows > 0 && (!A[i] || lda[i] < K)) return set_error(OZK_ERR_ARG, "A[%d] / lda", i);
    if (!G[i] || ldg[i] < K) return set_error(OZK_ERR_ARG, "G[%d] / ldg", i);
  }
  const int rho = ozk_compute_rho_f32(N);  // the contraction is over all N rows
  int rc = check_bound(N, 24 - rho);
  if (rc) return rc;
  // int8 codes and the int8 GEMM's raw sums, decided from the global shapes
  // (the same on every rank)
  const int64_t rmax = (N + P - 1) / P;
  const int64_t k8 = round_up(rmax > 0 ? rmax : 1, kS8KB);
  cudaSetDevice(ctx->dev[0].device);
  if (!(s8_enabled() && k8 <= 65536 &&
        slice_gemm_s8_eligible(K, K, k8, OZK_ACC_FIXED, rho, gemm_state_bytes(ctx->dev[0].device))))
    return set_error(OZK_ERR_UNSUPPORTED,
                     "the multi-GPU gram needs int8 codes (rho >= %d: N > 4096), K >= 256 and at "
                     "most 65536 rows per rank",
                     kS8MinRho);
  const int nS = n_hi + n_lo;
  const int npass = n_hi > n_lo ? n_hi : n_lo;
  uint8_t pa[OZK_MAX_PAIRS], pb[OZK_MAX_PAIRS];
  const int np = ozk_pair_schedule_snake(n_hi, n_lo, pa, pb, OZK_MAX_PAIRS);
  if (np < 0) return np;
  std::vector<cudaStream_t> s(nl);
  for (int i = 0; i < nl; ++i) s[i] = streams ? (cudaStream_t)streams[i] : nullptr;
  struct Ws {
    double* AT;    // [K][rows]: this rank's part of each line (column of A)
    int8_t* S;     // [nS][K][k8] codes of the part
    int32_t* e;    // [nS][K]
    float* pmax;   // [2][K] this rank's maxima
    float* gmax;   // [2][K] all ranks' maxima
    long long* P;  // [K][K] int64 sums (upper triangle)
    int32_t* flags_send;
    int32_t* flags_all;
    int32_t* gate;
    double* state;
    size_t state_bytes;
  };
  std::vector<Ws> ws(nl);
  for (int i = 0; i < nl; ++i) {
    DevState& d = ctx->dev[i];
    cudaSetDevice(d.device);
    const int64_t rows = rows_of(N, d.rank, P);
    const size_t sb = gemm_state_bytes(d.device);
    size_t off = 0;
    auto take = [&](size_t n) { size_t o = off; off += a256(n); return o; };
    const size_t oAT = take((size_t)K * (rows > 0 ? rows : 1) * 8), oS = take((size_t)nS * K * k8),
                 oe = take((size_t)nS * K * 4), opm = take((size_t)2 * K * 4),
                 ogm = take((size_t)2 * K * 4), oP = take((size_t)K * K * 8), ofs = take(8),
                 ofa = take((size_t)8 * P), og = take(4), ost = take(sb);
    if ((rc = grow(d, off))) return rc;
    char* b = (char*)d.buf;
    Ws& w = ws[i];
    w.AT = (double*)(b + oAT);
    w.S = (int8_t*)(b + oS);
    w.e = (int32_t*)(b + oe);
    w.pmax = (float*)(b + opm);
    w.gmax = (float*)(b + ogm);
    w.P = (long long*)(b + oP);
    w.flags_send = (int32_t*)(b + ofs);
    w.flags_all = (int32_t*)(b + ofa);
    w.gate = (int32_t*)(b + og);
    w.state = (double*)(b + ost);
    w.state_bytes = sb;
    cudaError_t e = cudaMemsetAsync(w.flags_send, 0, 8, s[i]);
    if (e == cudaSuccess) e = cudaMemsetAsync(w.pmax, 0, (size_t)2 * K * 4, s[i]);
    if (e != cudaSuccess) return set_cuda_error("cudaMemsetAsync", e);
    // the rank's rows of A as lines (columns of A), then the split's maxima
    if (rows > 0) {
      if ((rc = launch_transpose_f64(A[i], lda[i], rows, K, w.AT, s[i]))) return rc;
      if ((rc = launch_line_pass_s8(w.AT, rows, K, rows, -1, npass, rho, n_hi, n_lo, nullptr,
                                    w.pmax, w.S, k8, w.e, w.flags_send + 1, w.flags_send, s[i])))
        return rc;
    }
  }
  // the slice passes: the lines' maxima over all ranks, then this rank's codes
  for (int t = 0; t < npass; ++t) {
    ncclResult_t nr = api.GroupStart();
    for (int i = 0; i < nl && nr == ncclSuccess; ++i)
      nr = api.AllReduce(ws[i].pmax, ws[i].gmax, (size_t)2 * K, ncclFloat32, ncclMax,
                         ctx->dev[i].comm, s[i]);
    ncclResult_t ge = api.GroupEnd();
    if (nr != ncclSuccess) return nccl_error("all-reduce of the line maxima", nr);
    if (ge != ncclSuccess) return nccl_error("ncclGroupEnd", ge);
    for (int i = 0; i < nl; ++i) {
      cudaSetDevice(ctx->dev[i].device);
      const int64_t rows = rows_of(N, ctx->dev[i].rank, P);
      Ws& w = ws[i];
      if (rows > 0) {
        rc = launch_line_pass_s8(w.AT, rows, K, rows, t, npass, rho, n_hi, n_lo, w.gmax, w.pmax,
                                 w.S, k8, w.e, w.flags_send + 1, w.flags_send, s[i]);
      } else {
        // no rows here: zero codes; the exponents follow from gmax as anywhere
        rc = launch_line_pass_s8(w.AT, 0, K, 0, t, npass, rho, n_hi, n_lo, w.gmax, w.pmax, w.S,
                                 k8, w.e, w.flags_send + 1, w.flags_send, s[i]);
      }
      if (rc) return rc;
    }
  }
  // every rank's flags; then the raw sums of this rank's rows (gated), their
  // all-reduce, and the FP64 values with the mirror
  ncclResult_t nr = api.GroupStart();
  for (int i = 0; i < nl && nr == ncclSuccess; ++i)
    nr = api.AllGather(ws[i].flags_send, ws[i].flags_all, 2, ncclInt32, ctx->dev[i].comm, s[i]);
  ncclResult_t ge = api.GroupEnd();
  if (nr != ncclSuccess) return nccl_error("all-gather of the flags", nr);
  if (ge != ncclSuccess) return nccl_error("ncclGroupEnd", ge);
  const bool nowait = (flags & OZK_MULTI_NOWAIT) != 0;
  for (int i = 0; i < nl; ++i) {
    cudaSetDevice(ctx->dev[i].device);
    Ws& w = ws[i];
    k_reduce_flags<<<1, 32, 0, s[i]>>>(w.flags_all, P, w.gate, status_dev ? status_dev[i] : nullptr,
                                       OZK_FLAG_REDO);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaMemsetAsync(w.P, 0, (size_t)K * K * 8, s[i]);
    if (e != cudaSuccess) return set_cuda_error("k_reduce_flags / memset", e);
    const int64_t rows = rows_of(N, ctx->dev[i].rank, P);
    if (rows > 0 &&
        (rc = launch_slice_gemm_ex(w.S, w.e, nS, w.S, w.e, nS, K, K, k8, pa, pb, np, OZK_ACC_FIXED,
                                   1, 1.0, 0.0, nullptr, 0, nullptr, K, nullptr, w.state,
                                   w.state_bytes, rho, status_dev ? status_dev[i] : nullptr, true,
                                   w.gate, 0, s[i], w.P)))
      return rc;
  }
  nr = api.GroupStart();
  for (int i = 0; i < nl && nr == ncclSuccess; ++i)
    nr = api.AllReduce(ws[i].P, ws[i].P, (size_t)K * K, ncclInt64, ncclSum, ctx->dev[i].comm, s[i]);
  ge = api.GroupEnd();
  if (nr != ncclSuccess) return nccl_error("all-reduce of the sums", nr);
  if (ge != ncclSuccess) return nccl_error("ncclGroupEnd", ge);
  for (int i = 0; i < nl; ++i) {
    cudaSetDevice(ctx->dev[i].device);
    Ws& w = ws[i];
    const int64_t tiles = ((K + 31) / 32) * ((K + 31) / 32);
    const unsigned grid = (unsigned)(tiles < 65535 ? tiles : 65535);
    k_gram_finalize<<<grid, 256, 0, s[i]>>>(w.P, K, w.e, 2 * (rho - 24) - kFixFrac, w.gate, G[i],
                                            ldg[i]);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_cuda_error("k_gram_finalize launch", e);
  }
  return nowait ? OZK_OK : wait_all(ctx, s.data());
}

}  // extern "C"
