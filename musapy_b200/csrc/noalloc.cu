// mpb_reduce_noalloc: the reduction entry point for callers that cannot
// allocate device memory.
//
// mpb_reduce asks its caller for scratch (the partial results of reductions
// split across several CTAs). Some callers of this library cannot provide
// it: an application that embeds the library and owns the whole device
// memory budget through its own pool (a cudaMalloc from inside the library
// would fail, or silently break the host's accounting), and latency-critical
// loops in which cudaMalloc / cudaFree must not run because they can
// synchronise the whole device. This entry point takes the same arguments as
// mpb_reduce minus the scratch, and uses instead a fixed array that lives in
// this library's device image (kNoAllocScratchBytes per GPU, held from the
// moment the library's module is loaded on that GPU until the process exits).
//
// Rules:
//  * Requests are never refused for their size. The plan is limited to splits
//    whose partials fit in kNoAllocScratchBytes; a reduction too wide to split
//    within it (more than 16384 outputs) runs unsplit, as mpb_reduce does when
//    splitting is off, which needs no scratch at all. When the limit changes
//    the split count, sums and means may differ from mpb_reduce's in the last
//    bits (another grouping of the same additions); when it does not, the two
//    entry points run the same plan and agree bit for bit.
//  * Nothing here allocates: no cudaMalloc, no cudaFree, no allocating
//    library routine.
//  * Every call shares the one array per GPU and the array keeps whatever the
//    last call wrote. The split reduction writes every partial it later reads,
//    so nothing in it has to start at zero. Two calls that can run at the same
//    time on the GPU (different streams, no ordering between them) race on
//    the array: order them on one stream or through events.
//  * The first call on each device looks up the array's device address with
//    cudaGetSymbolAddress while that device is current. That first call must
//    come before any stream capture on the device. Later calls made while
//    their stream is not being captured look the address up again (a
//    cudaDeviceReset unloads this library's module, which may come back at
//    another address); calls made under capture use the last address found.
#include <mutex>

#include "internal.h"
#include "reduce.h"

namespace mpb {
namespace {

// 256 KiB: a full reduction splits into 4 CTAs per SM (592 partials on B200,
// 16 bytes each at most), so one output uses under 10 KiB.
constexpr size_t kNoAllocScratchBytes = 256 * 1024;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

void* g_scratch_addr[kMaxDevices] = {nullptr};
std::mutex g_scratch_mu;

// Device address of g_noalloc_scratch on the current device. In host code the
// name g_noalloc_scratch is only a host-side stand-in, never a device address.
int noalloc_scratch(cudaStream_t stream, void** out) {
  int dev = 0;
  int rc = cuda_check(cudaGetDevice(&dev), "mpb_reduce_noalloc: cudaGetDevice");
  if (rc) return rc;
  if (dev < 0 || dev >= kMaxDevices) return fail(MPB_ERR_INVALID, "mpb_reduce_noalloc: device %d out of range", dev);
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  rc = cuda_check(cudaStreamIsCapturing(stream, &cap), "mpb_reduce_noalloc: cudaStreamIsCapturing");
  if (rc) return rc;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (cap == cudaStreamCaptureStatusNone) {
    void* p = nullptr;
    rc = cuda_check(cudaGetSymbolAddress(&p, g_noalloc_scratch), "mpb_reduce_noalloc: cudaGetSymbolAddress");
    if (rc) return rc;
    g_scratch_addr[dev] = p;
  } else if (g_scratch_addr[dev] == nullptr) {
    return fail(MPB_ERR_INVALID,
                "mpb_reduce_noalloc: the first call on device %d ran under stream capture; make one call on the "
                "device before capturing",
                dev);
  }
  *out = g_scratch_addr[dev];
  return MPB_OK;
}

}  // namespace
}  // namespace mpb

using namespace mpb;

extern "C" int mpb_reduce_noalloc(int op, int ndim, const int64_t* shape, const int64_t* strides, const void* a,
                                  int in_dtype, uint64_t axes_mask, void* out, int out_dtype, int compute_dtype,
                                  int nan_first_rule, cudaStream_t stream) {
  RedReq r{};
  r.op = op;
  r.ndim = ndim;
  r.shape = shape;
  r.strides = strides;
  r.a = a;
  r.in_dt = in_dtype;
  r.axes_mask = axes_mask;
  r.out = out;
  r.out_dt = out_dtype;
  r.compute_dt = compute_dtype;
  r.nan_first_rule = nan_first_rule;
  r.allow_split = 1;
  r.scratch_cap = kNoAllocScratchBytes;  // split only as far as the built-in array holds
  r.out_stride = 1;
  const size_t need = red_scratch_bytes(r);
  if (need > kNoAllocScratchBytes)  // the capped planner never asks for more; kept as a guard
    return fail(MPB_ERR_SCRATCH,
                "mpb_reduce_noalloc: this reduction needs %zu bytes of scratch but the built-in scratch holds %zu "
                "bytes; call mpb_reduce with caller-provided scratch instead",
                need, kNoAllocScratchBytes);
  if (need > 0) {
    void* p = nullptr;
    const int rc = noalloc_scratch(stream, &p);
    if (rc) return rc;
    r.scratch = p;
    r.scratch_bytes = kNoAllocScratchBytes;
  }
  return red_run(r, stream);
}
