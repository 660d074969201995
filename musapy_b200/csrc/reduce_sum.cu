// sum / mean instantiations. Accumulator follows musapy's compute dtype
// (rust/musapy-ops/src/op_builder.rs:2209-2225): f32 (also for f16/bf16
// inputs) -> f32, f64 -> f64, integers -> wrapping i64 (f64 for mean),
// complex -> f64 parts as the CPU loop does (op_builder.rs:3439-3492).
#include "reduce_kernels.cuh"

namespace mpb {
namespace red {

int run_sum(const RedReq& r, const RedPlan& pl, RedOut ro, cudaStream_t s) {
  switch (r.compute_dt) {
    case MPB_F32:
      if (r.in_dt == MPB_F32) return launch_policy<PSum<float, float>>(r, pl, ro, s);
      if (r.in_dt == MPB_F16) return launch_policy<PSum<__half, float>>(r, pl, ro, s);
      if (r.in_dt == MPB_BF16) return launch_policy<PSum<__nv_bfloat16, float>>(r, pl, ro, s);
      break;
    case MPB_F64:
      if (r.in_dt == MPB_F64) return launch_policy<PSum<double, double>>(r, pl, ro, s);
      if (r.in_dt == MPB_I64) return launch_policy<PSum<int64_t, double>>(r, pl, ro, s);
      if (r.in_dt == MPB_U64) return launch_policy<PSum<uint64_t, double>>(r, pl, ro, s);
      break;
    case MPB_I64:
      if (r.in_dt == MPB_I64) return launch_policy<PSum<int64_t, uint64_t>>(r, pl, ro, s);
      if (r.in_dt == MPB_U64) return launch_policy<PSum<uint64_t, uint64_t>>(r, pl, ro, s);
      break;
    case MPB_C64:
    case MPB_C128:
      if (r.in_dt == MPB_C64) return launch_policy<PSum<c64, c128>>(r, pl, ro, s);
      if (r.in_dt == MPB_C128) return launch_policy<PSum<c128, c128>>(r, pl, ro, s);
      break;
    default: break;
  }
  return fail(MPB_ERR_DTYPE, "sum/mean: input dtype %d with compute dtype %d not supported (narrow integers are widened to int64 by the caller)", r.in_dt, r.compute_dt);
}

}  // namespace red
}  // namespace mpb
