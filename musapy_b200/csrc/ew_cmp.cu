// Comparisons (eq/ne/lt/gt/le/ge) of the elementwise engine: bool (u8 0/1)
// output, compare in the promoted dtype (16-bit floats widen exactly to f32).
#include "ew_host.cuh"

namespace mpb {
namespace ew {
namespace {

#define SAME2(DT) (r.a_dt == (DT) && r.b_dt == (DT))

template <class Op>
int cmp_real(const Op& op, const EwReq& r, cudaStream_t s) {
  switch (r.compute_dt) {
    case MPB_F32:
      if (SAME2(MPB_F32)) return run_typed<Op, float, float, float, boolean, 2>(op, r, s);
      return run_generic<Op, float, boolean, 2>(op, r, s);
    case MPB_F64:
      if (SAME2(MPB_F64)) return run_typed<Op, double, double, double, boolean, 2>(op, r, s);
      return run_generic<Op, double, boolean, 2>(op, r, s);
    case MPB_F16:
      if (SAME2(MPB_F16)) return run_typed<Op, float, __half, __half, boolean, 2>(op, r, s);
      return run_generic<Op, float, boolean, 2>(op, r, s);
    case MPB_BF16: return run_generic<Op, float, boolean, 2>(op, r, s);
    case MPB_I64:
      if (SAME2(MPB_I64)) return run_typed<Op, int64_t, int64_t, int64_t, boolean, 2>(op, r, s);
      return run_generic<Op, int64_t, boolean, 2>(op, r, s);
    case MPB_I32: return run_generic<Op, int32_t, boolean, 2>(op, r, s);
    case MPB_I16: return run_generic<Op, int16_t, boolean, 2>(op, r, s);
    case MPB_I8: return run_generic<Op, int8_t, boolean, 2>(op, r, s);
    case MPB_U64: return run_generic<Op, uint64_t, boolean, 2>(op, r, s);
    case MPB_U32: return run_generic<Op, uint32_t, boolean, 2>(op, r, s);
    case MPB_U16: return run_generic<Op, uint16_t, boolean, 2>(op, r, s);
    case MPB_U8:
    case MPB_BOOL: return run_generic<Op, uint8_t, boolean, 2>(op, r, s);
    default: return fail(MPB_ERR_DTYPE, "compare: compute dtype %d not supported", r.compute_dt);
  }
}

template <class Op>
int cmp_cplx(const Op& op, const EwReq& r, cudaStream_t s) {
  if (r.compute_dt == MPB_C64) {
    if (SAME2(MPB_C64)) return run_typed<Op, c64, c64, c64, boolean, 2>(op, r, s);
    return run_generic<Op, c64, boolean, 2>(op, r, s);
  }
  if (SAME2(MPB_C128)) return run_typed<Op, c128, c128, c128, boolean, 2>(op, r, s);
  return run_generic<Op, c128, boolean, 2>(op, r, s);
}

}  // namespace

int compare(const EwReq& r, cudaStream_t s) {
  if (r.out_dt != MPB_BOOL) return fail(MPB_ERR_DTYPE, "compare: output dtype must be bool");
  const bool cplx = is_complex(r.compute_dt);
  switch (r.op) {
    case MPB_EQ: return cplx ? cmp_cplx(OpEqC{}, r, s) : cmp_real(OpEq{}, r, s);
    case MPB_NE: return cplx ? cmp_cplx(OpNeC{}, r, s) : cmp_real(OpNe{}, r, s);
    default: break;
  }
  if (cplx) return fail(MPB_ERR_DTYPE, "ordering comparison not supported for complex dtypes");
  switch (r.op) {
    case MPB_LT: return cmp_real(OpLt{}, r, s);
    case MPB_GT: return cmp_real(OpGt{}, r, s);
    case MPB_LE: return cmp_real(OpLe{}, r, s);
    case MPB_GE: return cmp_real(OpGe{}, r, s);
    default: return fail(MPB_ERR_INVALID, "compare: unknown op %d", r.op);
  }
}

}  // namespace ew
}  // namespace mpb
