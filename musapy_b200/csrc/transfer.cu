// Host <-> device copies of pageable host memory at PCIe speed.
//
// musapy moves host data with list-based ms.array / tolist (O(n) in Python,
// rust/musapy-python/src/ops.rs:354-625, array.rs:451-488) and plain
// musaMemcpy; a copy from pageable memory is staged by the driver through a
// small bounce buffer one chunk at a time, and a fresh pageable destination
// first has to be faulted in page by page (a 1 GiB numpy() ran at ~2 GB/s).
// Here a ring of pinned staging slots (4 x 32 MiB, allocated once, portable
// across devices) pipelines the two halves of every copy:
//   H2D  host threads copy chunk k into a free slot while the DMA engine moves
//        chunk k-1 to the device (cudaMemcpyAsync on the caller's stream);
//   D2H  the DMA engine fills slot k+S while host threads copy slot k out.
// The host-side memcpy of each chunk is split across a small pool of worker
// threads, which also spreads the first-touch page faults of a fresh
// destination over several cores. One cudaMemcpyAsync per chunk; the ring
// is a process-wide resource guarded by a mutex, so concurrent calls take
// turns. Host memory that is already page-locked (cudaHostAlloc,
// cudaHostRegister, torch's pin_memory) needs no staging: it is moved by one
// DMA straight from or to the caller's buffer, and the call waits for that
// DMA, so both kinds of host memory give the same return contract.
#include <condition_variable>
#include <cstring>
#include <functional>
#include <mutex>
#include <thread>
#include <vector>
#include "internal.h"
#include "musapy_b200.h"

namespace mpb {
namespace {

constexpr size_t kSlotBytes = 32u << 20;
constexpr int kSlots = 4;
constexpr int kMaxDevices = 64;

// Fixed pool of worker threads running index-range jobs. It is created on
// first use and intentionally never destroyed: its threads wait on a
// condition variable and end with the process.
class Pool {
 public:
  explicit Pool(int n) {
    for (int i = 0; i < n; ++i) threads_.emplace_back([this] { loop(); });
    for (auto& t : threads_) t.detach();
  }
  int size() const { return (int)threads_.size() + 1; }
  // Runs fn(part) for part in [0, parts) on the workers and the caller.
  void run(int parts, const std::function<void(int)>& fn) {
    {
      std::lock_guard<std::mutex> lk(mu_);
      job_ = &fn;
      parts_ = parts;
      next_ = 0;
      done_ = 0;
      ++gen_;
    }
    cv_.notify_all();
    work();
    std::unique_lock<std::mutex> lk(mu_);
    done_cv_.wait(lk, [&] { return done_ == parts_; });
    job_ = nullptr;
  }

 private:
  void work() {
    for (;;) {
      int p;
      const std::function<void(int)>* job;
      {
        std::lock_guard<std::mutex> lk(mu_);
        if (job_ == nullptr || next_ >= parts_) return;
        p = next_++;
        job = job_;
      }
      (*job)(p);
      {
        std::lock_guard<std::mutex> lk(mu_);
        if (++done_ == parts_) done_cv_.notify_all();
      }
    }
  }
  void loop() {
    unsigned seen = 0;
    for (;;) {
      {
        std::unique_lock<std::mutex> lk(mu_);
        cv_.wait(lk, [&] { return gen_ != seen; });
        seen = gen_;
      }
      work();
    }
  }
  std::vector<std::thread> threads_;
  std::mutex mu_;
  std::condition_variable cv_, done_cv_;
  const std::function<void(int)>* job_ = nullptr;
  int parts_ = 0, next_ = 0, done_ = 0;
  unsigned gen_ = 0;
};

Pool& pool() {
  static Pool* p = [] {
    unsigned hw = std::thread::hardware_concurrency();
    int n = hw > 1 ? (int)(hw < 8 ? hw : 8) - 1 : 0;
    return new Pool(n);
  }();
  return *p;
}

// memcpy split into 1 MiB-aligned parts over the pool
void par_memcpy(void* dst, const void* src, size_t n) {
  Pool& pl = pool();
  if (n < (4u << 20) || pl.size() == 1) {
    std::memcpy(dst, src, n);
    return;
  }
  const size_t unit = 1u << 20;
  int parts = pl.size() * 2;
  size_t per = (n + parts - 1) / parts;
  per = (per + unit - 1) / unit * unit;
  parts = (int)((n + per - 1) / per);
  pl.run(parts, [&](int i) {
    const size_t off = (size_t)i * per;
    const size_t len = off + per <= n ? per : n - off;
    std::memcpy(static_cast<char*>(dst) + off, static_cast<const char*>(src) + off, len);
  });
}

struct Ring {
  std::mutex mu;
  char* host = nullptr;                // kSlots * kSlotBytes pinned, portable
  cudaEvent_t ev[kMaxDevices][kSlots];  // per device: slot s free / filled
  cudaEvent_t direct[kMaxDevices];      // per device: end of a direct DMA
  bool ev_made[kMaxDevices] = {false};
};

Ring& ring() {
  static Ring* r = new Ring();
  return *r;
}

// This device's events (lock held by the caller).
int events_ready(Ring& r, int dev) {
  if (dev < 0 || dev >= kMaxDevices) return fail(MPB_ERR_INVALID, "copy: device %d out of range", dev);
  if (!r.ev_made[dev]) {
    for (int s = 0; s < kSlots; ++s) {
      int rc = cuda_check(cudaEventCreateWithFlags(&r.ev[dev][s], cudaEventDisableTiming), "copy: cudaEventCreate");
      if (rc != MPB_OK) return rc;
    }
    int rc = cuda_check(cudaEventCreateWithFlags(&r.direct[dev], cudaEventDisableTiming), "copy: cudaEventCreate");
    if (rc != MPB_OK) return rc;
    r.ev_made[dev] = true;
  }
  return MPB_OK;
}

// The pinned slots, allocated on the first staged copy (a copy between
// page-locked memory and the device never needs them) - lock held.
int ring_ready(Ring& r) {
  if (r.host == nullptr) {
    void* p = nullptr;
    int rc = cuda_check(cudaHostAlloc(&p, (size_t)kSlots * kSlotBytes, cudaHostAllocPortable), "copy: cudaHostAlloc");
    if (rc != MPB_OK) return rc;
    r.host = static_cast<char*>(p);
  }
  return MPB_OK;
}

int current_device(int* dev) { return cuda_check(cudaGetDevice(dev), "copy: cudaGetDevice"); }

// True when both ends of [p, p + bytes) are page-locked host memory known to
// CUDA. Pageable memory reports cudaMemoryTypeUnregistered (no error).
bool page_locked(const void* p, size_t bytes) {
  const char* ends[2] = {static_cast<const char*>(p), static_cast<const char*>(p) + bytes - 1};
  for (const char* e : ends) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, e) != cudaSuccess) {
      cudaGetLastError();
      return false;
    }
    if (a.type != cudaMemoryTypeHost) return false;
  }
  return true;
}

// One DMA between page-locked host memory and the device on `s`, then a wait
// for it (lock held by the caller).
int direct_copy(Ring& r, int dev, void* dst, const void* src, size_t bytes, cudaMemcpyKind kind, cudaStream_t s) {
  int rc = cuda_check(cudaMemcpyAsync(dst, src, bytes, kind, s), "copy: cudaMemcpyAsync (page-locked)");
  if (rc != MPB_OK) return rc;
  if ((rc = cuda_check(cudaEventRecord(r.direct[dev], s), "copy: cudaEventRecord")) != MPB_OK) return rc;
  return cuda_check(cudaEventSynchronize(r.direct[dev]), "copy: page-locked DMA wait");
}

}  // namespace
}  // namespace mpb

using namespace mpb;

extern "C" {

int mpb_copy_h2d(void* dst, const void* src, size_t bytes, mpb_stream_t stream) {
  if (bytes == 0) return MPB_OK;
  if (!dst || !src) return fail(MPB_ERR_INVALID, "mpb_copy_h2d: null pointer");
  cudaStream_t s = (cudaStream_t)stream;
  int dev = 0;
  int rc = current_device(&dev);
  if (rc != MPB_OK) return rc;
  Ring& r = ring();
  std::lock_guard<std::mutex> lk(r.mu);
  if ((rc = events_ready(r, dev)) != MPB_OK) return rc;
  if (page_locked(src, bytes)) return direct_copy(r, dev, dst, src, bytes, cudaMemcpyHostToDevice, s);
  if ((rc = ring_ready(r)) != MPB_OK) return rc;
  // slots may still be read by DMAs of a previous call: wait per slot below
  const size_t nchunks = (bytes + kSlotBytes - 1) / kSlotBytes;
  for (size_t k = 0; k < nchunks; ++k) {
    const int slot = (int)(k % kSlots);
    const size_t off = k * kSlotBytes;
    const size_t len = off + kSlotBytes <= bytes ? kSlotBytes : bytes - off;
    char* stage = r.host + (size_t)slot * kSlotBytes;
    if ((rc = cuda_check(cudaEventSynchronize(r.ev[dev][slot]), "copy: slot wait")) != MPB_OK) return rc;
    par_memcpy(stage, static_cast<const char*>(src) + off, len);
    if ((rc = cuda_check(cudaMemcpyAsync(static_cast<char*>(dst) + off, stage, len, cudaMemcpyHostToDevice, s),
                         "copy: cudaMemcpyAsync H2D")) != MPB_OK)
      return rc;
    if ((rc = cuda_check(cudaEventRecord(r.ev[dev][slot], s), "copy: cudaEventRecord")) != MPB_OK) return rc;
  }
  return MPB_OK;
}

int mpb_copy_d2h(void* dst, const void* src, size_t bytes, mpb_stream_t stream) {
  if (bytes == 0) return MPB_OK;
  if (!dst || !src) return fail(MPB_ERR_INVALID, "mpb_copy_d2h: null pointer");
  cudaStream_t s = (cudaStream_t)stream;
  int dev = 0;
  int rc = current_device(&dev);
  if (rc != MPB_OK) return rc;
  Ring& r = ring();
  std::lock_guard<std::mutex> lk(r.mu);
  if ((rc = events_ready(r, dev)) != MPB_OK) return rc;
  if (page_locked(dst, bytes)) return direct_copy(r, dev, dst, src, bytes, cudaMemcpyDeviceToHost, s);
  if ((rc = ring_ready(r)) != MPB_OK) return rc;
  const size_t nchunks = (bytes + kSlotBytes - 1) / kSlotBytes;
  auto issue = [&](size_t k) -> int {
    const int slot = (int)(k % kSlots);
    const size_t off = k * kSlotBytes;
    const size_t len = off + kSlotBytes <= bytes ? kSlotBytes : bytes - off;
    int e = cuda_check(cudaMemcpyAsync(r.host + (size_t)slot * kSlotBytes, static_cast<const char*>(src) + off, len,
                                       cudaMemcpyDeviceToHost, s),
                       "copy: cudaMemcpyAsync D2H");
    if (e != MPB_OK) return e;
    return cuda_check(cudaEventRecord(r.ev[dev][slot], s), "copy: cudaEventRecord");
  };
  // a previous H2D may still read the slots: the stream orders our DMAs after
  // the caller's earlier work, but not after other streams' copies
  for (int slot = 0; slot < kSlots; ++slot)
    if ((rc = cuda_check(cudaEventSynchronize(r.ev[dev][slot]), "copy: slot wait")) != MPB_OK) return rc;
  for (size_t k = 0; k < nchunks && k < (size_t)kSlots; ++k)
    if ((rc = issue(k)) != MPB_OK) return rc;
  for (size_t k = 0; k < nchunks; ++k) {
    const int slot = (int)(k % kSlots);
    const size_t off = k * kSlotBytes;
    const size_t len = off + kSlotBytes <= bytes ? kSlotBytes : bytes - off;
    if ((rc = cuda_check(cudaEventSynchronize(r.ev[dev][slot]), "copy: D2H wait")) != MPB_OK) return rc;
    par_memcpy(static_cast<char*>(dst) + off, r.host + (size_t)slot * kSlotBytes, len);
    if (k + kSlots < nchunks && (rc = issue(k + kSlots)) != MPB_OK) return rc;
  }
  return MPB_OK;
}

}  // extern "C"
