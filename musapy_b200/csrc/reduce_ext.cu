// max / min value instantiations: value-only accumulators (no index), the
// CPU NaN rule and the first-zero sign rule (op_builder.rs:3543-3578).
// Unsigned 64-bit inputs compare as int64, as musapy's cast to i64 does.
#include "reduce_kernels.cuh"

namespace mpb {
namespace red {

template <class TIn, class V>
int ext_typed(const RedReq& r, const RedPlan& pl, RedOut ro, bool is_max, cudaStream_t s) {
  if (is_max) return launch_policy<PExt<TIn, V, true>>(r, pl, ro, s);
  return launch_policy<PExt<TIn, V, false>>(r, pl, ro, s);
}

int run_ext(const RedReq& r, const RedPlan& pl, RedOut ro, bool is_max, cudaStream_t s) {
  switch (r.in_dt) {
    case MPB_F32: return ext_typed<float, float>(r, pl, ro, is_max, s);
    case MPB_F64: return ext_typed<double, double>(r, pl, ro, is_max, s);
    case MPB_F16: return ext_typed<__half, float>(r, pl, ro, is_max, s);
    case MPB_BF16: return ext_typed<__nv_bfloat16, float>(r, pl, ro, is_max, s);
    case MPB_I64: return ext_typed<int64_t, int64_t>(r, pl, ro, is_max, s);
    case MPB_U64: return ext_typed<uint64_t, int64_t>(r, pl, ro, is_max, s);
    default:
      return fail(MPB_ERR_DTYPE, "max/min: input dtype %d not supported (narrow integers are widened to int64 by the caller)", r.in_dt);
  }
}

}  // namespace red
}  // namespace mpb
