// Host-memory staging for copies between pageable host memory and the device.
//
// A copy from ordinary (pageable) host memory goes through the driver's own
// staging, which moved about 11 GB/s on this pool's B200 hosts, against
// 55 GB/s of PCIe Gen5 from page-locked memory; page-locking the caller's
// buffer in place (cudaHostRegister) ran at about 11 GB/s as well.  Host
// memcpy, on the other hand, reached 73-87 GB/s with 8-12 threads.  So a
// pageable operand is moved through a small ring of page-locked slots: host
// threads copy chunk c into a free slot while the DMA engine moves chunk c-1,
// and each slot is reused once the event recorded after its DMA has completed.
//
// Resources (kept for the life of the process, created on first pageable use):
// per device and direction, kSlots page-locked slots of kSlotBytes and their
// events; two pools of memcpy threads (one per direction, so the copy-out of
// C can run while A is still being copied in).
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <condition_variable>
#include <functional>
#include <mutex>
#include <thread>
#include <vector>

#include "ozaki_b200.h"
#include "ozk_internal.h"

namespace ozk {
namespace {

constexpr int kSlots = 3;
constexpr size_t kSlotBytes = 32u << 20;

// A pool of worker threads that run one job at a time: run(f) calls f(t, n)
// for t = 0..n-1, t = 0 on the calling thread, and returns when all are done.
class CopyPool {
 public:
  explicit CopyPool(int n) : n_(n < 1 ? 1 : n) {
    for (int t = 1; t < n_; ++t) th_.emplace_back([this, t] { loop(t); });
  }
  ~CopyPool() {
    {
      std::lock_guard<std::mutex> lk(mu_);
      stop_ = true;
    }
    cv_.notify_all();
    for (auto& t : th_) t.join();
  }
  void run(const std::function<void(int, int)>& f) {
    std::lock_guard<std::mutex> serial(run_mu_);
    {
      std::lock_guard<std::mutex> lk(mu_);
      job_ = &f;
      pending_ = n_ - 1;
      ++gen_;
    }
    cv_.notify_all();
    f(0, n_);
    std::unique_lock<std::mutex> lk(mu_);
    done_cv_.wait(lk, [this] { return pending_ == 0; });
    job_ = nullptr;
  }

 private:
  void loop(int t) {
    uint64_t seen = 0;
    for (;;) {
      const std::function<void(int, int)>* f;
      {
        std::unique_lock<std::mutex> lk(mu_);
        cv_.wait(lk, [&] { return stop_ || gen_ != seen; });
        if (stop_) return;
        seen = gen_;
        f = job_;
      }
      (*f)(t, n_);
      std::lock_guard<std::mutex> lk(mu_);
      if (--pending_ == 0) done_cv_.notify_all();
    }
  }
  int n_;
  std::vector<std::thread> th_;
  std::mutex mu_, run_mu_;
  std::condition_variable cv_, done_cv_;
  const std::function<void(int, int)>* job_ = nullptr;
  int pending_ = 0;
  uint64_t gen_ = 0;
  bool stop_ = false;
};

CopyPool& pool(int dir) {
  static std::once_flag once;
  static CopyPool* pools[2];
  std::call_once(once, [] {
    const int hc = (int)std::max(1u, std::thread::hardware_concurrency());
    pools[0] = new CopyPool(std::min(12, std::max(1, hc / 2)));      // host -> device
    pools[1] = new CopyPool(std::min(8, std::max(1, hc * 3 / 8)));   // device -> host
  });
  return *pools[dir];
}

struct Ring {
  std::mutex mu;  // one staged copy at a time per device and direction
  char* slot[kSlots] = {};
  cudaEvent_t ev[kSlots] = {};
  bool busy[kSlots] = {};
  bool ready = false;
};

Ring g_rings[64][2];
std::mutex g_ring_init_mu;

int ring_for(int dir, Ring** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_cuda_error("cudaGetDevice", e);
  if (dev < 0 || dev >= 64) return set_error(OZK_ERR_ARG, "device index %d out of range", dev);
  Ring& r = g_rings[dev][dir];
  std::lock_guard<std::mutex> lk(g_ring_init_mu);
  if (!r.ready) {
    for (int i = 0; i < kSlots; ++i) {
      if ((e = cudaHostAlloc((void**)&r.slot[i], kSlotBytes, cudaHostAllocPortable)) != cudaSuccess)
        return set_cuda_error("cudaHostAlloc(staging slot)", e);
      if ((e = cudaEventCreateWithFlags(&r.ev[i], cudaEventDisableTiming)) != cudaSuccess)
        return set_cuda_error("cudaEventCreate(staging)", e);
    }
    r.ready = true;
  }
  *out = &r;
  return OZK_OK;
}

// Copies `rows` rows of `width` bytes between a strided source and a strided
// destination with all threads of the pool.
void parallel_rows(CopyPool& p, char* dst, size_t dpitch, const char* src, size_t spitch,
                   size_t width, size_t rows) {
  if (rows == 0 || width == 0) return;
  const size_t total = rows * width;
  if (dpitch == width && spitch == width) {
    p.run([&](int t, int n) {
      const size_t a = total * t / n, b = total * (t + 1) / n;
      memcpy(dst + a, src + a, b - a);
    });
    return;
  }
  p.run([&](int t, int n) {
    const size_t a = rows * t / n, b = rows * (t + 1) / n;
    for (size_t r = a; r < b; ++r) memcpy(dst + r * dpitch, src + r * spitch, width);
  });
}

}  // namespace

bool is_pageable(const void* p) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return true;
  }
  return a.type == cudaMemoryTypeUnregistered;
}

// Host (pageable) -> device, rows x width bytes, enqueued on `s`.  Returns once
// every byte has left `src` (the caller may reuse it); the DMAs may still be in
// flight on `s`.
int staged_h2d_2d(void* dst, size_t dpitch, const void* src, size_t spitch, size_t width,
                  size_t rows, cudaStream_t s) {
  if (rows == 0 || width == 0) return OZK_OK;
  if (width > kSlotBytes) {
    cudaError_t e = cudaMemcpy2DAsync(dst, dpitch, src, spitch, width, rows, cudaMemcpyDefault, s);
    return e == cudaSuccess ? OZK_OK : set_cuda_error("cudaMemcpy2DAsync", e);
  }
  Ring* r = nullptr;
  int rc = ring_for(0, &r);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(r->mu);
  const size_t per = kSlotBytes / width;
  CopyPool& p = pool(0);
  int slot = 0;
  for (size_t r0 = 0; r0 < rows; r0 += per) {
    const size_t nr = std::min(per, rows - r0);
    if (r->busy[slot]) {
      cudaError_t e = cudaEventSynchronize(r->ev[slot]);
      if (e != cudaSuccess) return set_cuda_error("cudaEventSynchronize(staging)", e);
    }
    parallel_rows(p, r->slot[slot], width, (const char*)src + r0 * spitch, spitch, width, nr);
    cudaError_t e = cudaMemcpy2DAsync((char*)dst + r0 * dpitch, dpitch, r->slot[slot], width,
                                      width, nr, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaEventRecord(r->ev[slot], s);
    if (e != cudaSuccess) return set_cuda_error("staged copy to the device", e);
    r->busy[slot] = true;
    slot = (slot + 1) % kSlots;
  }
  return OZK_OK;
}

// Device -> host (pageable), rows x width bytes, ordered on `s`.  Blocking:
// returns when every byte is in `dst`.
int staged_d2h_2d(void* dst, size_t dpitch, const void* src, size_t spitch, size_t width,
                  size_t rows, cudaStream_t s) {
  if (rows == 0 || width == 0) return OZK_OK;
  if (width > kSlotBytes) {
    cudaError_t e = cudaMemcpy2DAsync(dst, dpitch, src, spitch, width, rows, cudaMemcpyDefault, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    return e == cudaSuccess ? OZK_OK : set_cuda_error("cudaMemcpy2DAsync", e);
  }
  Ring* r = nullptr;
  int rc = ring_for(1, &r);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(r->mu);
  const size_t per = kSlotBytes / width;
  const size_t nchunk = (rows + per - 1) / per;
  CopyPool& p = pool(1);
  auto issue = [&](size_t c) -> cudaError_t {
    const int slot = (int)(c % kSlots);
    const size_t r0 = c * per, nr = std::min(per, rows - r0);
    cudaError_t e = cudaMemcpy2DAsync(r->slot[slot], width, (const char*)src + r0 * spitch, spitch,
                                      width, nr, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaEventRecord(r->ev[slot], s);
    return e;
  };
  for (size_t c = 0; c < nchunk && c < (size_t)kSlots; ++c) {
    cudaError_t e = issue(c);
    if (e != cudaSuccess) return set_cuda_error("staged copy from the device", e);
  }
  for (size_t c = 0; c < nchunk; ++c) {
    const int slot = (int)(c % kSlots);
    const size_t r0 = c * per, nr = std::min(per, rows - r0);
    cudaError_t e = cudaEventSynchronize(r->ev[slot]);
    if (e != cudaSuccess) return set_cuda_error("cudaEventSynchronize(staging)", e);
    parallel_rows(p, (char*)dst + r0 * dpitch, dpitch, r->slot[slot], width, width, nr);
    if (c + kSlots < nchunk && (e = issue(c + kSlots)) != cudaSuccess)
      return set_cuda_error("staged copy from the device", e);
  }
  for (int i = 0; i < kSlots; ++i) r->busy[i] = false;
  return OZK_OK;
}

}  // namespace ozk

extern "C" int ozk_memcpy_staged(void* dst, const void* src, size_t bytes, void* stream) {
  using namespace ozk;
  if (!dst || !src) return set_error(OZK_ERR_ARG, "NULL pointer");
  if (!bytes) return OZK_OK;
  cudaStream_t s = (cudaStream_t)stream;
  cudaPointerAttributes ad, as;
  cudaError_t e = cudaPointerGetAttributes(&ad, dst);
  if (e == cudaSuccess) e = cudaPointerGetAttributes(&as, src);
  if (e != cudaSuccess) return set_cuda_error("cudaPointerGetAttributes", e);
  const bool dst_dev = ad.type == cudaMemoryTypeDevice || ad.type == cudaMemoryTypeManaged;
  const bool src_dev = as.type == cudaMemoryTypeDevice || as.type == cudaMemoryTypeManaged;
  // a flat copy as rows of 1 MiB plus a tail row
  const size_t W = 1u << 20, rows = bytes / W, tail = bytes % W;
  const char* sc = (const char*)src;
  char* dc = (char*)dst;
  int rc = OZK_OK;
  if (dst_dev && !src_dev && as.type == cudaMemoryTypeUnregistered) {
    if ((rc = staged_h2d_2d(dc, W, sc, W, W, rows, s))) return rc;
    if (tail && (rc = staged_h2d_2d(dc + rows * W, tail, sc + rows * W, tail, tail, 1, s)))
      return rc;
    e = cudaStreamSynchronize(s);
    return e == cudaSuccess ? OZK_OK : set_cuda_error("cudaStreamSynchronize", e);
  }
  if (src_dev && !dst_dev && ad.type == cudaMemoryTypeUnregistered) {
    if ((rc = staged_d2h_2d(dc, W, sc, W, W, rows, s))) return rc;
    if (tail) rc = staged_d2h_2d(dc + rows * W, tail, sc + rows * W, tail, tail, 1, s);
    return rc;
  }
  e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  return e == cudaSuccess ? OZK_OK : set_cuda_error("cudaMemcpyAsync", e);
}
