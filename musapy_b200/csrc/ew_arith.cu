// Binary arithmetic (add/sub/mul/div/pow) of the elementwise engine.
// Same-dtype operands and the int64 (x) float64 promotion pair get dedicated
// instantiations; any other promotion pair reads through runtime-dtype loads.
#include "ew_host.cuh"

namespace mpb {
namespace ew {
namespace {

#define SAME2(DT) (r.a_dt == (DT) && r.b_dt == (DT))

template <class Op>
int arith_real(const Op& op, const EwReq& r, cudaStream_t s) {
  switch (r.compute_dt) {
    case MPB_F32:
      if (SAME2(MPB_F32)) return run_typed<Op, float, float, float, float, 2, true>(op, r, s);
      return run_generic<Op, float, float, 2>(op, r, s);
    case MPB_F64:
      if (SAME2(MPB_F64)) return run_typed<Op, double, double, double, double, 2, true>(op, r, s);
      if (r.a_dt == MPB_I64 && r.b_dt == MPB_F64) return run_typed<Op, double, int64_t, double, double, 2, true>(op, r, s);
      if (r.a_dt == MPB_F64 && r.b_dt == MPB_I64) return run_typed<Op, double, double, int64_t, double, 2, true>(op, r, s);
      return run_generic<Op, double, double, 2>(op, r, s);
    case MPB_F16:
      if (SAME2(MPB_F16)) return run_typed<Op, float, __half, __half, __half, 2>(op, r, s);
      return run_generic<Op, float, __half, 2>(op, r, s);
    case MPB_BF16:
      if (SAME2(MPB_BF16)) return run_typed<Op, float, __nv_bfloat16, __nv_bfloat16, __nv_bfloat16, 2>(op, r, s);
      return run_generic<Op, float, __nv_bfloat16, 2>(op, r, s);
    default:
      return fail(MPB_ERR_DTYPE, "arithmetic: compute dtype %d not supported", r.compute_dt);
  }
}

template <class Op>
int arith_cplx(const Op& op, const EwReq& r, cudaStream_t s) {
  if (r.compute_dt == MPB_C64) {
    if (SAME2(MPB_C64)) return run_typed<Op, c64, c64, c64, c64, 2>(op, r, s);
    return run_generic<Op, c64, c64, 2>(op, r, s);
  }
  if (SAME2(MPB_C128)) return run_typed<Op, c128, c128, c128, c128, 2>(op, r, s);
  return run_generic<Op, c128, c128, 2>(op, r, s);
}

int arith_pow(const EwReq& r, cudaStream_t s) {
  switch (r.compute_dt) {
    case MPB_F32:
      if (SAME2(MPB_F32)) return run_typed<OpPow, float, float, float, float, 2>(OpPow{}, r, s);
      return run_generic<OpPow, float, float, 2>(OpPow{}, r, s);
    case MPB_F64:
      if (SAME2(MPB_F64)) return run_typed<OpPow, double, double, double, double, 2>(OpPow{}, r, s);
      return run_generic<OpPow, double, double, 2>(OpPow{}, r, s);
    case MPB_F16:
      if (SAME2(MPB_F16)) return run_typed<OpPowLow, float, __half, __half, __half, 2>(OpPowLow{}, r, s);
      return run_generic<OpPowLow, float, __half, 2>(OpPowLow{}, r, s);
    case MPB_BF16:
      return run_generic<OpPowLow, float, __nv_bfloat16, 2>(OpPowLow{}, r, s);
    default:
      return fail(MPB_ERR_DTYPE, "pow: compute dtype %d not supported", r.compute_dt);
  }
}

}  // namespace

int arith(const EwReq& r, cudaStream_t s) {
  const bool cplx = is_complex(r.compute_dt);
  if (r.out_dt != r.compute_dt) return fail(MPB_ERR_DTYPE, "arithmetic: output dtype %d != compute dtype %d", r.out_dt, r.compute_dt);
  switch (r.op) {
    case MPB_ADD: return cplx ? arith_cplx(OpAdd{}, r, s) : arith_real(OpAdd{}, r, s);
    case MPB_SUB: return cplx ? arith_cplx(OpSub{}, r, s) : arith_real(OpSub{}, r, s);
    case MPB_MUL: return cplx ? arith_cplx(OpMul{}, r, s) : arith_real(OpMul{}, r, s);
    case MPB_DIV: return cplx ? arith_cplx(OpDiv{}, r, s) : arith_real(OpDiv{}, r, s);
    case MPB_POW:
      if (cplx) return fail(MPB_ERR_DTYPE, "pow: complex dtypes are not supported");
      return arith_pow(r, s);
    default: return fail(MPB_ERR_INVALID, "arithmetic: unknown op %d", r.op);
  }
}

}  // namespace ew
}  // namespace mpb
