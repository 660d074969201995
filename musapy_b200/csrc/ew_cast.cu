// Casts, strided copies (same dtype, any layout -> contiguous) and fills of
// the elementwise engine. Cast semantics are musapy's (Rust `as`:
// rust/musapy-ops/src/op_builder.rs:2052-2097) plus IEEE round-to-nearest-even
// for f16/bf16, which the reference rejects (op_builder.rs:904-962).
#include "ew_host.cuh"

namespace mpb {
namespace ew {
namespace {

template <class T>
__global__ void __launch_bounds__(kEwThreads) k_fill(T* __restrict__ out, int64_t n, T v) {
  const int64_t gtid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t gs = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = gtid; i < n; i += gs) out[i] = v;
}

template <class T>
int fill_as(const EwReq& r, T v, cudaStream_t s) {
  int64_t n = 1;
  for (int i = 0; i < r.ndim; ++i) n *= r.shape[i];
  if (n == 0) return MPB_OK;
  k_fill<T><<<grid_for(n, kEwThreads * 4), kEwThreads, 0, s>>>(static_cast<T*>(r.out), n, v);
  return launch_check("fill");
}

}  // namespace

int fill(const EwReq& r, cudaStream_t s) {
  const double v = r.p0;
  switch (r.out_dt) {
    case MPB_BOOL: return fill_as<uint8_t>(r, (uint8_t)(v != 0.0), s);
    case MPB_I8: return fill_as<int8_t>(r, (int8_t)v, s);
    case MPB_I16: return fill_as<int16_t>(r, (int16_t)v, s);
    case MPB_I32: return fill_as<int32_t>(r, (int32_t)v, s);
    case MPB_I64: return fill_as<int64_t>(r, (int64_t)v, s);
    case MPB_U8: return fill_as<uint8_t>(r, (uint8_t)v, s);
    case MPB_U16: return fill_as<uint16_t>(r, (uint16_t)v, s);
    case MPB_U32: return fill_as<uint32_t>(r, (uint32_t)v, s);
    case MPB_U64: return fill_as<uint64_t>(r, (uint64_t)v, s);
    case MPB_F16: return fill_as<__half>(r, __double2half(v), s);
    case MPB_F32: return fill_as<float>(r, (float)v, s);
    case MPB_F64: return fill_as<double>(r, v, s);
    case MPB_BF16: return fill_as<__nv_bfloat16>(r, __double2bfloat16(v), s);
    case MPB_C64: return fill_as<c64>(r, c64{(float)v, (float)r.p1}, s);
    case MPB_C128: return fill_as<c128>(r, c128{v, r.p1}, s);
    default: return fail(MPB_ERR_DTYPE, "fill: dtype %d not supported", r.out_dt);
  }
}

int cast(const EwReq& r, cudaStream_t s) {
  const OpIdentity id{};
  const int a = r.a_dt, o = r.out_dt;
  if (a == o) {  // bit copy into a contiguous buffer
    switch (dtype_size(a)) {
      case 1: return run_typed<OpIdentity, uint8_t, uint8_t, uint8_t, uint8_t, 1, true>(id, r, s);
      case 2: return run_typed<OpIdentity, uint16_t, uint16_t, uint16_t, uint16_t, 1, true>(id, r, s);
      case 4: return run_typed<OpIdentity, uint32_t, uint32_t, uint32_t, uint32_t, 1, true>(id, r, s);
      case 8: return run_typed<OpIdentity, uint64_t, uint64_t, uint64_t, uint64_t, 1, true>(id, r, s);
      default: return run_typed<OpIdentity, c128, c128, c128, c128, 1, true>(id, r, s);
    }
  }
#define CAST_PAIR(SRC, DST, TS, TD) \
  if (a == SRC && o == DST) return run_typed<OpIdentity, TD, TS, TS, TD, 1>(id, r, s);
  CAST_PAIR(MPB_F32, MPB_BF16, float, __nv_bfloat16)
  CAST_PAIR(MPB_BF16, MPB_F32, __nv_bfloat16, float)
  CAST_PAIR(MPB_F32, MPB_F16, float, __half)
  CAST_PAIR(MPB_F16, MPB_F32, __half, float)
  CAST_PAIR(MPB_F32, MPB_F64, float, double)
  CAST_PAIR(MPB_F64, MPB_F32, double, float)
  CAST_PAIR(MPB_I64, MPB_F64, int64_t, double)
  CAST_PAIR(MPB_I64, MPB_F32, int64_t, float)
  CAST_PAIR(MPB_F64, MPB_I64, double, int64_t)
  CAST_PAIR(MPB_F32, MPB_I64, float, int64_t)
#undef CAST_PAIR
  switch (o) {
    case MPB_BOOL: return run_generic<OpIdentity, boolean, boolean, 1>(id, r, s);
    case MPB_I8: return run_generic<OpIdentity, int8_t, int8_t, 1>(id, r, s);
    case MPB_I16: return run_generic<OpIdentity, int16_t, int16_t, 1>(id, r, s);
    case MPB_I32: return run_generic<OpIdentity, int32_t, int32_t, 1>(id, r, s);
    case MPB_I64: return run_generic<OpIdentity, int64_t, int64_t, 1>(id, r, s);
    case MPB_U8: return run_generic<OpIdentity, uint8_t, uint8_t, 1>(id, r, s);
    case MPB_U16: return run_generic<OpIdentity, uint16_t, uint16_t, 1>(id, r, s);
    case MPB_U32: return run_generic<OpIdentity, uint32_t, uint32_t, 1>(id, r, s);
    case MPB_U64: return run_generic<OpIdentity, uint64_t, uint64_t, 1>(id, r, s);
    case MPB_F16: return run_generic<OpIdentity, __half, __half, 1>(id, r, s);
    case MPB_F32: return run_generic<OpIdentity, float, float, 1>(id, r, s);
    case MPB_F64: return run_generic<OpIdentity, double, double, 1>(id, r, s);
    case MPB_BF16: return run_generic<OpIdentity, __nv_bfloat16, __nv_bfloat16, 1>(id, r, s);
    case MPB_C64: return run_generic<OpIdentity, c64, c64, 1>(id, r, s);
    case MPB_C128: return run_generic<OpIdentity, c128, c128, 1>(id, r, s);
    default: return fail(MPB_ERR_DTYPE, "cast: target dtype %d not supported", o);
  }
}

}  // namespace ew
}  // namespace mpb
