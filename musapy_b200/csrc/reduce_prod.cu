// prod instantiations (same accumulator rules as sum).
#include "reduce_kernels.cuh"

namespace mpb {
namespace red {

int run_prod(const RedReq& r, const RedPlan& pl, RedOut ro, cudaStream_t s) {
  switch (r.compute_dt) {
    case MPB_F32:
      if (r.in_dt == MPB_F32) return launch_policy<PProd<float, float>>(r, pl, ro, s);
      if (r.in_dt == MPB_F16) return launch_policy<PProd<__half, float>>(r, pl, ro, s);
      if (r.in_dt == MPB_BF16) return launch_policy<PProd<__nv_bfloat16, float>>(r, pl, ro, s);
      break;
    case MPB_F64:
      if (r.in_dt == MPB_F64) return launch_policy<PProd<double, double>>(r, pl, ro, s);
      break;
    case MPB_I64:
      if (r.in_dt == MPB_I64) return launch_policy<PProd<int64_t, uint64_t>>(r, pl, ro, s);
      if (r.in_dt == MPB_U64) return launch_policy<PProd<uint64_t, uint64_t>>(r, pl, ro, s);
      break;
    case MPB_C64:
    case MPB_C128:
      if (r.in_dt == MPB_C64) return launch_policy<PProd<c64, c128>>(r, pl, ro, s);
      if (r.in_dt == MPB_C128) return launch_policy<PProd<c128, c128>>(r, pl, ro, s);
      break;
    default: break;
  }
  return fail(MPB_ERR_DTYPE, "prod: input dtype %d with compute dtype %d not supported (narrow integers are widened to int64 by the caller)", r.in_dt, r.compute_dt);
}

}  // namespace red
}  // namespace mpb
