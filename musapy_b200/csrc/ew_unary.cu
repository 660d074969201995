// Unary math (sin/cos/exp/log/abs/sign/neg) and clamp of the elementwise
// engine. The input dtype is the compute dtype (no promotion), as in
// rust/musapy-ops/src/op_builder.rs:561-582 and :752-763.
#include "ew_host.cuh"

namespace mpb {
namespace ew {
namespace {

template <class Op>
int unary_real(const Op& op, const EwReq& r, cudaStream_t s) {
  switch (r.compute_dt) {
    case MPB_F32: return run_typed<Op, float, float, float, float, 1>(op, r, s);
    case MPB_F64: return run_typed<Op, double, double, double, double, 1>(op, r, s);
    case MPB_F16: return run_generic<Op, float, __half, 1>(op, r, s);
    case MPB_BF16: return run_generic<Op, float, __nv_bfloat16, 1>(op, r, s);
    default: return fail(MPB_ERR_DTYPE, "unary: dtype %d not supported", r.compute_dt);
  }
}

int clamp(const EwReq& r, cudaStream_t s) {
  switch (r.compute_dt) {
    case MPB_F32: {
      // lo/hi narrowed to f32 like `lo as f32` (op_builder.rs:851).
      OpClamp<float> op{(float)r.p0, (float)r.p1};
      return run_typed<OpClamp<float>, float, float, float, float, 1>(op, r, s);
    }
    case MPB_F64: {
      OpClamp<double> op{r.p0, r.p1};
      return run_typed<OpClamp<double>, double, double, double, double, 1>(op, r, s);
    }
    case MPB_F16: {
      OpClamp<float> op{__half2float(__double2half(r.p0)), __half2float(__double2half(r.p1))};
      return run_generic<OpClamp<float>, float, __half, 1>(op, r, s);
    }
    case MPB_BF16: {
      OpClamp<float> op{__bfloat162float(__double2bfloat16(r.p0)), __bfloat162float(__double2bfloat16(r.p1))};
      return run_generic<OpClamp<float>, float, __nv_bfloat16, 1>(op, r, s);
    }
    default: return fail(MPB_ERR_DTYPE, "clamp: dtype %d not supported", r.compute_dt);
  }
}

}  // namespace

int unary(const EwReq& r, cudaStream_t s) {
  if (r.a_dt != r.compute_dt) return fail(MPB_ERR_DTYPE, "unary: input dtype %d != compute dtype %d", r.a_dt, r.compute_dt);
  const int cd = r.compute_dt;
  switch (r.op) {
    case MPB_SIN: return unary_real(OpSin{}, r, s);
    case MPB_COS: return unary_real(OpCos{}, r, s);
    case MPB_EXP: return unary_real(OpExp{}, r, s);
    case MPB_LOG: return unary_real(OpLog{}, r, s);
    case MPB_SIGN: return unary_real(OpSign{}, r, s);
    case MPB_NEG:
      if (cd == MPB_C64) return run_typed<OpNeg, c64, c64, c64, c64, 1>(OpNeg{}, r, s);
      if (cd == MPB_C128) return run_typed<OpNeg, c128, c128, c128, c128, 1>(OpNeg{}, r, s);
      return unary_real(OpNeg{}, r, s);
    case MPB_ABS:
      // |complex| is real (op_builder.rs:584-589)
      if (cd == MPB_C64) return run_typed<OpAbs, c64, c64, c64, float, 1>(OpAbs{}, r, s);
      if (cd == MPB_C128) return run_typed<OpAbs, c128, c128, c128, double, 1>(OpAbs{}, r, s);
      return unary_real(OpAbs{}, r, s);
    case MPB_CLAMP: return clamp(r, s);
    default: return fail(MPB_ERR_INVALID, "unary: unknown op %d", r.op);
  }
}

}  // namespace ew
}  // namespace mpb
