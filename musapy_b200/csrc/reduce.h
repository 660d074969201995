// Reduction / scan request and plan types shared by the engine and the C-ABI.
#pragma once
#include <stddef.h>
#include <stdint.h>
#include "mpb_types.h"
#include "plan.h"

namespace mpb {

struct RedReq {
  int op;  // mpb_red_op
  int ndim;
  const int64_t* shape;
  const int64_t* strides;  // elements, may be 0 or negative
  const void* a;           // logical element [0, ..., 0]
  int in_dt;
  uint64_t axes_mask;  // bit d set -> dim d reduced
  void* out;           // C-contiguous over the kept dims
  int out_dt;
  int compute_dt;
  int nan_first_rule;  // 1: a NaN first element decides max/min/arg (CPU rule)
  void* scratch;
  size_t scratch_bytes;
  int allow_split;     // 0: never pick a plan that needs scratch
  size_t scratch_cap;  // > 0: pick no split whose partials exceed this many bytes
  int64_t out_stride;  // elements between consecutive outputs (0 or 1: contiguous)
};

enum RedKind { RK_EMPTY = 0, RK_ROW_WARP, RK_ROW_BLOCK, RK_ROW_SPLIT, RK_COL, RK_COL_SPLIT, RK_GEN };

struct RedPlan {
  int kind = RK_EMPTY;
  int K = 0, R = 0;
  int64_t M = 0, L = 0, Li = 0, Lo = 0;
  int64_t ks[kMaxCollapsed], kst[kMaxCollapsed];
  int64_t rs[kMaxCollapsed], rst[kMaxCollapsed], rw[kMaxCollapsed];
  int vec = 1;
  bool vectorized = false;
  int64_t splits = 1;
  int64_t chunk = 0;
  int colv = 1;  // COL kinds: adjacent outputs per thread (one 8- or 16-byte load per reduced step)
};

int red_plan(const RedReq& r, RedPlan& pl);
size_t red_scratch_bytes(const RedReq& r);
int red_run(const RedReq& r, cudaStream_t s);

struct ScanReq {
  int ndim;
  const int64_t* shape;
  const int64_t* strides;
  const void* a;
  int in_dt;
  int axis;
  void* out;  // C-contiguous, same shape
  int out_dt; // compute dtype: i64 for integers, else the float type
  void* scratch;
  size_t scratch_bytes;
  int* status;  // optional device word: set non-zero when a bounded wait gives up
};

size_t scan_scratch_bytes(const ScanReq& r);
int scan_run(const ScanReq& r, cudaStream_t s);

}  // namespace mpb
