// Entry point of the elementwise engine: validates the request and routes it
// to the op family (arithmetic, comparison, unary/clamp, cast/fill).
//
// The reference picks one of four kernel shapes inside each C wrapper
// (scalar-a / scalar-b / contiguous-vec4 / nd; kernels/elementwise.mu:
// 581-659). Here the choice is made once per call from the collapsed
// geometry (ew_host.cuh), for every dtype combination, and type promotion is
// fused into the loads instead of materialising a cast temporary
// (rust/musapy-ops/src/op_builder.rs:410-417).
#include <map>
#include <mutex>
#include <utility>
#include "internal.h"
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
