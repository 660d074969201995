// Internal host helpers: error reporting and device queries.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include "mpb_types.h"

namespace mpb {

// Records a message for mpb_last_error() (thread-local) and returns `code`.
int fail(int code, const char* fmt, ...);
// MPB_OK when `e` is cudaSuccess, otherwise records the CUDA error.
int cuda_check(cudaError_t e, const char* what);
// Checks the CUDA error state after a launch: cleared (cudaGetLastError) for
// the extended API, which reports it as a status; left in place
// (cudaPeekAtLastError) while a reference-ABI wrapper runs, so the caller's own
// cudaGetLastError() still sees it as with musapy's kernels.
int launch_check(const char* what);
// launch_check for a launch made through cudaLaunchKernelEx, whose own return
// code `e` is checked as well.
int launch_check_pdl(cudaError_t e, const char* what);
void set_preserve_last_error(bool on);
// Multiprocessor count of the current device (cached per device).
int sm_count();

struct EwReq {
  int op;
  int ndim;
  const int64_t* shape;
  const void* a;
  int a_dt;
  const int64_t* a_st;
  const void* b;  // null for unary ops
  int b_dt;
  const int64_t* b_st;
  void* out;  // C-contiguous with `shape`
  int out_dt;
  int compute_dt;
  double p0, p1;  // clamp bounds / fill value
};

int ew_run(const EwReq& r, cudaStream_t stream);

}  // namespace mpb
