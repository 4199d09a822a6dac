// Device-side building blocks for sm_100a: exact FP32 helpers of the Ozaki
// extraction, mbarriers with bounded waits, TMA tile loads and tcgen05
// (UMMA / TMEM) wrappers written as inline PTX.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "ozaki_b200.h"

namespace ozk {

// ---------------------------------------------------------------- exact FP32

// 2^n as FP32 with the semantics of ldexp(1.0f, n): +inf above 127, subnormal
// below -126, 0 below -149 (2^-150 rounds to even = 0).
__device__ __forceinline__ float pow2f(int n) {
  if (n > 127) return __int_as_float(0x7f800000);
  if (n >= -126) return __int_as_float((n + 127) << 23);
  if (n >= -149) return __int_as_float(1 << (n + 149));
  return 0.0f;
}

// 2^n as FP64 (inf above 1023, subnormal below -1022, 0 below -1074).
__device__ __forceinline__ double pow2d(int n) {
  if (n > 1023) return __longlong_as_double(0x7ff0000000000000LL);
  if (n >= -1022) return __longlong_as_double((long long)(n + 1023) << 52);
  if (n >= -1074) return __longlong_as_double(1LL << (n + 1074));
  return 0.0;
}

// floor(RN32(log2(m))) for finite m > 0, from the per-binade threshold table
// (thr[e + 149] = bits of the smallest m of binade e whose rounded log2 is e+1,
// e in [-149, 127]).  An infinite or NaN m (a line the caller flags as
// non-finite) gives 128, and m = 0 (which callers treat as a zero line
// before asking) -150, without reading outside the table.
__device__ __forceinline__ int floor_log2_rn32(float m, const uint32_t* thr) {
  uint32_t b = __float_as_uint(m);
  int e = (b >= 0x00800000u) ? (int)(b >> 23) - 127 : -149 + (31 - __clz(b));
  if (e > 127) return 128;
  if (e < -149) return -150;
  return e + (b >= thr[e + 149] ? 1 : 0);
}

// BF16 bit pattern of an FP32 value that is exactly representable in BF16.
__device__ __forceinline__ uint16_t bf16_bits_exact(float v) {
  return (uint16_t)(__float_as_uint(v) >> 16);
}

// ---------------------------------------------------------------- flags

__device__ __forceinline__ void raise_flag(int32_t* status, int32_t bits) {
  if (status) atomicOr(status, bits);
}

// ---------------------------------------------------------------- smem/mbarrier

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
          smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait for the phase of `bar` with the given parity to complete.
// Gives up (returns false) when *abort becomes non-zero (abort may be NULL:
// then only the clock ends it) or when `budget_ns` of wall time pass; on a
// timeout it sets *abort and OZK_FLAG_TIMEOUT in *status.  Every device-side
// wait in this library goes through here.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort,
                                          int32_t* status, uint64_t budget_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  uint64_t t0 = global_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63) == 0) {
      if (abort && *abort) return false;
      if (global_ns() - t0 > budget_ns) {
        if (abort) *abort = 1;
        raise_flag(status, OZK_FLAG_TIMEOUT);
        return false;
      }
    }
  }
}

// ---------------------------------------------------------------- TMA

// Untiled bulk copy global -> shared (this CTA), completion counted on `bar`
// in bytes.  dst and src 16-byte aligned, bytes a multiple of 16.  No multicast.
__device__ __forceinline__ void bulk_load_g2s(void* dst, const void* src, uint32_t bytes,
                                              uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(smem_u32(dst)), "l"((uint64_t)src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Untiled bulk copy shared (this CTA) -> global, tracked by this thread's bulk
// groups.  dst and src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_store_s2g(void* dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;"
               ::"l"((uint64_t)dst), "r"(smem_u32(src)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Every committed bulk store of this thread has read its shared-memory source.
__device__ __forceinline__ void bulk_wait_read_all() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// Every committed bulk store of this thread is complete.
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// Orders this thread's earlier generic-proxy shared-memory accesses before
// its later async-proxy ones (a bulk copy into a buffer just read, or out of
// a buffer just written).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)map) : "memory");
}

// 3D tiled bulk tensor load global -> shared (this CTA), completion counted
// on `bar` in bytes.  No multicast.
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(smem_dst)),
      "l"((uint64_t)map), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

// 3D tiled load for a CTA pair (cta_group::2): the data lands in this CTA's
// shared memory, completion is counted on `bar_cluster`, an mbarrier of either
// CTA of the pair given by its shared::cluster address.  No multicast.
__device__ __forceinline__ void tma_load_3d_pair(void* smem_dst, const CUtensorMap* map,
                                                 uint32_t bar_cluster, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(smem_dst)),
      "l"((uint64_t)map), "r"(x), "r"(y), "r"(z), "r"(bar_cluster)
      : "memory");
}

// Prefetch a 3D tile into L2 (no shared-memory destination, no completion).
__device__ __forceinline__ void tma_prefetch_3d(const CUtensorMap* map, int x, int y, int z) {
  asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(
                   (uint64_t)map),
               "r"(x), "r"(y), "r"(z)
               : "memory");
}

// L2 cache policy that keeps lines resident (evict_last) for data re-read soon.
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// 32-bit load served by L2, not L1: for data other SMs wrote with atomics.
__device__ __forceinline__ int ld_cg_s32(const int* p) {
  int v;
  asm volatile("ld.global.cg.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// 64-bit load served by L2, not L1: for data other SMs wrote with atomics.
__device__ __forceinline__ long long ld_cg_s64(const long long* p) {
  long long v;
  asm volatile("ld.global.cg.s64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ long long ld_l2_hint(const long long* p, uint64_t pol) {
  long long v;
  asm volatile("ld.global.L1::no_allocate.L2::cache_hint.b64 %0, [%1], %2;"
               : "=l"(v)
               : "l"(p), "l"(pol)
               : "memory");
  return v;
}

__device__ __forceinline__ void st_l2_hint(long long* p, long long v, uint64_t pol) {
  asm volatile("st.global.L2::cache_hint.b64 [%0], %1, %2;" ::"l"(p), "l"(v), "l"(pol) : "memory");
}

// 32-byte vector store (sm_100): p must be 32-byte aligned.
__device__ __forceinline__ void st_global_v4_f64(double* p, double a, double b, double c, double d) {
  asm volatile("st.global.v4.f64 [%0], {%1, %2, %3, %4};" ::"l"(p), "d"(a), "d"(b), "d"(c), "d"(d)
               : "memory");
}

// shared::cluster address of the object at local address `p` in CTA `rank`.
__device__ __forceinline__ uint32_t mapa_u32(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}

// Arrive on an mbarrier given by its shared::cluster address (possibly in a
// peer CTA).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster)
               : "memory");
}

// ---------------------------------------------------------------- tcgen05

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Whole-warp TMEM allocation; the base address is written to *dst_smem.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// CTA-pair variants: one warp of each CTA of the pair (same warp index, same
// destination offset) executes them.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// Shared-memory matrix descriptor for a K-major BF16 tile written by TMA with
// 128-byte swizzle: rows of 64 elements (128 B), 8-row atoms 1024 B apart.
//   bits  0-13 start address >> 4     bits 16-29 leading byte offset >> 4 (unused)
//   bits 32-45 stride byte offset >> 4 bits 46-47 descriptor version (1)
//   bits 61-63 layout (2 = 128-byte swizzle)
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFF) >> 4);
  d |= (uint64_t)(16 >> 4) << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor: BF16 x BF16 -> FP32, both operands K-major.
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int M, int N) {
  return (1u << 4)      // D format FP32
         | (1u << 7)    // A format BF16
         | (1u << 10)   // B format BF16
         | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// kind::i8 instruction descriptor: signed 8-bit A and B, signed 32-bit D,
// both operands K-major.
__host__ __device__ constexpr uint32_t umma_idesc_s8(int M, int N) {
  return (2u << 4)      // D format S32
         | (1u << 7)    // A format S8
         | (1u << 10)   // B format S8
         | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// D[tmem] (+)= A[smem] * B[smem]^T, issued by one thread.
__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A * B^T over a CTA pair (M = 256: rows 0-127 from this CTA's
// A tile, 128-255 from the peer's at the same shared-memory offset; B's
// N columns split in halves the same way).  Issued by one thread of the
// even CTA of the pair.
__device__ __forceinline__ void umma_bf16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                               uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A * B^T on int8 operands with an exact int32 accumulator,
// one CTA (K = 32 per instruction).
__device__ __forceinline__ void umma_s8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// The same over int8 operands with an exact int32 accumulator (K = 32 per
// instruction: the same 32 bytes of each row as a BF16 instruction).
__device__ __forceinline__ void umma_s8_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on the mbarrier at the same offset in each CTA of `cta_mask` once all
// pair MMAs issued so far by this thread have completed.
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(smem_u32(bar)),
      "h"(cta_mask)
      : "memory");
}

// Arrive on `bar` once all tcgen05 operations issued so far by this thread
// have completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread t of the warp receives
// lane (taddr.lane + t), columns taddr.col .. +31.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// ---------------------------------------------------------------- clusters

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %cluster_ctarank;" : "=r"(r));
  return r;
}

// Full cluster barrier (all threads of all CTAs), release/acquire ordering of
// shared memory across the cluster.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}

// Load a float from the shared memory of CTA `rank` of this cluster at the
// offset of the local object `p`.
__device__ __forceinline__ float ld_dsmem_f32(const float* p, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(p)), "r"(rank));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
  return v;
}

// Relaxed 64-bit store to this CTA's shared memory: one single-copy-atomic word.
__device__ __forceinline__ void st_smem_relaxed_u64(uint64_t* p, uint64_t v) {
  asm volatile("st.relaxed.cluster.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(p)), "l"(v) : "memory");
}

// Relaxed 64-bit load from the shared memory of CTA `rank` of this cluster (this
// CTA included) at the offset of the local object `p`.
__device__ __forceinline__ uint64_t ld_dsmem_relaxed_u64(const uint64_t* p, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(p)), "r"(rank));
  uint64_t v;
  asm volatile("ld.relaxed.cluster.shared::cluster.b64 %0, [%1];" : "=l"(v) : "r"(remote) : "memory");
  return v;
}

// Bounded wait for a tagged word of CTA `rank`: (tag << 32) | value, written
// with st_smem_relaxed_u64.  Tag and value travel in one atomic word, so a
// matching tag proves the value current without release/acquire ordering.
// Returns the value; gives up like mbar_wait (returns false, sets *abort and
// OZK_FLAG_TIMEOUT in *status) after budget_ns or once *abort is set.
__device__ __forceinline__ bool tag_wait(const uint64_t* p, uint32_t rank, uint32_t tag,
                                         uint32_t& val, volatile int* abort, int32_t* status,
                                         uint64_t budget_ns) {
  uint64_t w = ld_dsmem_relaxed_u64(p, rank);
  if ((uint32_t)(w >> 32) == tag) {
    val = (uint32_t)w;
    return true;
  }
  val = 0;
  if (*abort) return false;
  const uint64_t t0 = global_ns();
  for (uint32_t i = 1;; ++i) {
    w = ld_dsmem_relaxed_u64(p, rank);
    if ((uint32_t)(w >> 32) == tag) {
      val = (uint32_t)w;
      return true;
    }
    if ((i & 31) == 0) {
      if (*abort) return false;
      if (global_ns() - t0 > budget_ns) {
        *abort = 1;
        raise_flag(status, OZK_FLAG_TIMEOUT);
        return false;
      }
    }
  }
}

// Relaxed 64-bit store into the shared memory of CTA `rank` of this cluster
// (this CTA included) at the offset of the local object `p`: one
// single-copy-atomic word, sent without waiting for it to land.
__device__ __forceinline__ void st_dsmem_relaxed_u64(uint64_t* p, uint32_t rank, uint64_t v) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(p)), "r"(rank));
  asm volatile("st.relaxed.cluster.shared::cluster.b64 [%0], %1;" ::"r"(remote), "l"(v) : "memory");
}

// Bounded wait for a tagged word in this CTA's own shared memory, (tag << 32)
// | value, which a peer CTA of the cluster stored with st_dsmem_relaxed_u64.
// The poll is a local load, so waiting costs no round trip to the peer.
// Returns like tag_wait.
__device__ __forceinline__ bool tag_wait_local(const uint64_t* p, uint32_t tag, uint32_t& val,
                                               volatile int* abort, int32_t* status,
                                               uint64_t budget_ns) {
  const uint32_t a = smem_u32(p);
  uint64_t w;
  asm volatile("ld.relaxed.cluster.shared::cta.b64 %0, [%1];" : "=l"(w) : "r"(a) : "memory");
  if ((uint32_t)(w >> 32) == tag) {
    val = (uint32_t)w;
    return true;
  }
  val = 0;
  if (*abort) return false;
  const uint64_t t0 = global_ns();
  for (uint32_t i = 1;; ++i) {
    asm volatile("ld.relaxed.cluster.shared::cta.b64 %0, [%1];" : "=l"(w) : "r"(a) : "memory");
    if ((uint32_t)(w >> 32) == tag) {
      val = (uint32_t)w;
      return true;
    }
    if ((i & 255) == 0) {
      if (*abort) return false;
      if (global_ns() - t0 > budget_ns) {
        *abort = 1;
        raise_flag(status, OZK_FLAG_TIMEOUT);
        return false;
      }
    }
  }
}

// Cluster barrier without memory ordering (arrive.relaxed): the data that
// crosses it carries tags instead (tag_wait).
__device__ __forceinline__ void cluster_sync_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;\n\tbarrier.cluster.wait.aligned;" ::
                   : "memory");
}

// Named barrier among `nthreads` threads (multiple of 32).
__device__ __forceinline__ void named_bar(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

}  // namespace ozk
