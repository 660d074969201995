// Entry point of the elementwise engine: validates the request and routes it
// to the op family (arithmetic, comparison, unary/clamp, cast/fill).
//
// The reference picks one of four kernel shapes inside each C wrapper
// (scalar-a / scalar-b / contiguous-vec4 / nd; kernels/elementwise.mu:
// 581-659). Here the choice is made once per call from the collapsed
// geometry (ew_host.cuh), for every dtype combination, and type promotion is
// fused into the loads instead of materialising a cast temporary
// (rust/musapy-ops/src/op_builder.rs:410-417).
#include <cuda.h>
#include <atomic>
#include <map>
#include <mutex>
#include <utility>
#include "internal.h"
#include "musapy_b200.h"
#include "plan.h"

namespace mpb {
namespace ew {
int arith(const EwReq& r, cudaStream_t s);
int compare(const EwReq& r, cudaStream_t s);
int unary(const EwReq& r, cudaStream_t s);
int cast(const EwReq& r, cudaStream_t s);
int fill(const EwReq& r, cudaStream_t s);

// Resident blocks per SM of `kernel` at `threads` threads per block, per
// device, queried once (cudaOccupancyMaxActiveBlocksPerMultiprocessor).
int blocks_per_sm_cached(const void* kernel, int threads) {
  static std::mutex mu;
  static std::map<std::pair<int, const void*>, int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    (void)cudaGetLastError();
    return 1;
  }
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find({dev, kernel});
  if (it != cache.end()) return it->second;
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, 0) != cudaSuccess || per_sm < 1) {
    (void)cudaGetLastError();
    per_sm = 1;
  }
  cache[{dev, kernel}] = per_sm;
  return per_sm;
}

int blocks_per_sm_smem(const void* kernel, int threads, int smem) {
  static std::mutex mu;
  static std::map<std::pair<int, const void*>, int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    (void)cudaGetLastError();
    return 1;
  }
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find({dev, kernel});
  if (it != cache.end()) return it->second;
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem) != cudaSuccess || per_sm < 1) {
    (void)cudaGetLastError();
    per_sm = 1;
  }
  cache[{dev, kernel}] = per_sm;
  return per_sm;
}

// cuTensorMapEncodeTiled, reached through the runtime's driver entry point
// (no link against the driver library).
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      (void)cudaGetLastError();
      p = nullptr;
    }
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

// Tensor map of a (p, q[, batch]) view with unit stride along p: boxes of
// box_p x box_q elements, no swizzle, zero fill outside the array.
int tma_encode(CUtensorMap* m, const void* base, int elem_bytes, int64_t dp, int64_t dq, int64_t nb, int64_t sq_bytes,
               int64_t sb_bytes, int box_p, int box_q) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return -1;
  CUtensorMapDataType dt;
  switch (elem_bytes) {
    case 2: dt = CU_TENSOR_MAP_DATA_TYPE_UINT16; break;
    case 4: dt = CU_TENSOR_MAP_DATA_TYPE_UINT32; break;
    case 8: dt = CU_TENSOR_MAP_DATA_TYPE_INT64; break;
    default: return -1;
  }
  const cuuint32_t rank = nb > 1 ? 3 : 2;
  const cuuint64_t dims[3] = {(cuuint64_t)dp, (cuuint64_t)dq, (cuuint64_t)(nb > 1 ? nb : 1)};
  const cuuint64_t strides[2] = {(cuuint64_t)sq_bytes, (cuuint64_t)(nb > 1 ? sb_bytes : sq_bytes * dq)};
  const cuuint32_t box[3] = {(cuuint32_t)box_p, (cuuint32_t)box_q, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = fn(m, dt, rank, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -1;
}

// One device int per GPU, set by a tiled-TMA warp whose wait ran out.
int* tiled_wait_flag() {
  static std::mutex mu;
  static std::map<int, int*> flags;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    (void)cudaGetLastError();
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  auto it = flags.find(dev);
  if (it != flags.end()) return it->second;
  int* p = nullptr;
  if (cudaMalloc(&p, sizeof(int)) != cudaSuccess || cudaMemset(p, 0, sizeof(int)) != cudaSuccess) {
    (void)cudaGetLastError();
    if (p) cudaFree(p);
    return nullptr;
  }
  flags[dev] = p;  // held until the process exits
  return p;
}

static std::atomic<int> g_tiled_tma{1};
static std::atomic<unsigned long long> g_tma_launches{0};
bool tiled_tma_enabled() { return g_tiled_tma.load(std::memory_order_relaxed) != 0; }

void count_tma_launch() { g_tma_launches.fetch_add(1, std::memory_order_relaxed); }

}  // namespace ew

int ew_run(const EwReq& r, cudaStream_t s) {
  if (r.ndim < 0 || r.ndim > MPB_MAX_DIMS) return fail(MPB_ERR_INVALID, "elementwise: ndim %d out of range", r.ndim);
  for (int i = 0; i < r.ndim; ++i)
    if (r.shape[i] < 0) return fail(MPB_ERR_SHAPE, "elementwise: negative extent");
  if (r.op == MPB_FILL) return r.out ? ew::fill(r, s) : fail(MPB_ERR_INVALID, "fill: null output");
  int64_t n = 1;
  for (int i = 0; i < r.ndim; ++i) n *= r.shape[i];
  if (n == 0) return MPB_OK;
  if (!r.a || !r.out) return fail(MPB_ERR_INVALID, "elementwise: null pointer");
  for (int dt : {r.a_dt, r.out_dt, r.compute_dt})
    if (dt < 0 || dt >= MPB_NUM_DTYPES) return fail(MPB_ERR_DTYPE, "elementwise: bad dtype tag %d", dt);
  if (r.op <= MPB_GE) {
    if (!r.b) return fail(MPB_ERR_INVALID, "elementwise: binary op without second operand");
    if (r.b_dt < 0 || r.b_dt >= MPB_NUM_DTYPES) return fail(MPB_ERR_DTYPE, "elementwise: bad dtype tag %d", r.b_dt);
  }
  if (r.op <= MPB_POW) return ew::arith(r, s);
  if (r.op >= MPB_EQ && r.op <= MPB_GE) return ew::compare(r, s);
  if ((r.op >= MPB_SIN && r.op <= MPB_NEG) || r.op == MPB_CLAMP) return ew::unary(r, s);
  if (r.op == MPB_CAST) return ew::cast(r, s);
  return fail(MPB_ERR_INVALID, "elementwise: unknown op %d", r.op);
}

}  // namespace mpb

using namespace mpb;

extern "C" {

int mpb_ew_set_tma(int enable) {
  const int prev = ew::g_tiled_tma.load();
  if (enable >= 0) ew::g_tiled_tma.store(enable ? 1 : 0);
  return prev;
}

uint64_t mpb_ew_tma_launches(void) { return ew::g_tma_launches.load(); }

int mpb_ew_wait_status(int* timed_out) {
  if (!timed_out) return fail(MPB_ERR_INVALID, "mpb_ew_wait_status: null pointer");
  *timed_out = 0;
  int* f = ew::tiled_wait_flag();
  if (!f) return fail(MPB_ERR_CUDA, "mpb_ew_wait_status: no flag on this device");
  int v = 0;
  int rc = cuda_check(cudaMemcpy(&v, f, sizeof(int), cudaMemcpyDeviceToHost), "mpb_ew_wait_status");
  if (rc) return rc;
  if (v) {
    const int zero = 0;
    rc = cuda_check(cudaMemcpy(f, &zero, sizeof(int), cudaMemcpyHostToDevice), "mpb_ew_wait_status");
  }
  *timed_out = v;
  return rc;
}

}  // extern "C"
