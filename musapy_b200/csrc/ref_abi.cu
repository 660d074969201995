// musapy's kernel C-ABI (rust/musapy-ops/src/kernels.rs:16-343), symbol for
// symbol, routed to the sm_100a engine. Declarations and per-symbol citations:
// include/musapy_kernels_v2.h.
//
// Each wrapper converts musapy's (size_t shape, ssize_t strides) arguments and
// calls the engine entry that the extended API uses. The wrappers return void
// like musapy's; a launch failure stays visible to the caller's
// cudaGetLastError() (the engine peeks instead of clearing while a wrapper
// runs), and requests the engine rejects are described by mpb_last_error().
#include <stddef.h>
#include <stdint.h>
#include <string.h>

#include "common.cuh"
#include "internal.h"
#include "reduce.h"

namespace mpb {
namespace ref {

// Keeps CUDA's last error for the caller while a reference wrapper runs.
struct PeekGuard {
  PeekGuard() { set_preserve_last_error(true); }
  ~PeekGuard() { set_preserve_last_error(false); }
};

struct Dims {
  int nd = 0;
  int64_t shape[MPB_MAX_DIMS];
  int64_t sa[MPB_MAX_DIMS];
  int64_t sb[MPB_MAX_DIMS];
};

bool load(int ndim, const size_t* shape, const ptrdiff_t* sa, const ptrdiff_t* sb, Dims& d) {
  if (ndim < 0 || ndim > MPB_MAX_DIMS) {
    fail(MPB_ERR_INVALID, "musapy kernel ABI: ndim %d out of range", ndim);
    return false;
  }
  d.nd = ndim;
  for (int i = 0; i < ndim; ++i) {
    d.shape[i] = (int64_t)shape[i];
    d.sa[i] = sa ? (int64_t)sa[i] : 0;
    d.sb[i] = sb ? (int64_t)sb[i] : 0;
  }
  return true;
}

void ew(int op, int a_dt, int b_dt, int out_dt, int cd, const void* a, const void* b, void* c, int ndim,
        const size_t* shape, const ptrdiff_t* as, const ptrdiff_t* bs, double p0, double p1, cudaStream_t s) {
  PeekGuard g;
  Dims d;
  if (!load(ndim, shape, as, bs, d)) return;
  EwReq r;
  r.op = op;
  r.ndim = d.nd;
  r.shape = d.shape;
  r.a = a;
  r.a_dt = a_dt;
  r.a_st = d.sa;
  r.b = b;
  r.b_dt = b_dt;
  r.b_st = d.sb;
  r.out = c;
  r.out_dt = out_dt;
  r.compute_dt = cd;
  r.p0 = p0;
  r.p1 = p1;
  ew_run(r, s);
}

// One reduction over `axis` (no scratch: musapy's one-launch wrappers take
// none), output written with stride `ostride`.
int reduce_axis(int op, int dt, int out_dt, const void* a, void* c, int ndim, const size_t* in_shape,
                const ptrdiff_t* in_strides, int axis, int64_t ostride, cudaStream_t s) {
  Dims d;
  if (!load(ndim, in_shape, in_strides, nullptr, d)) return MPB_ERR_INVALID;
  if (axis < 0 || axis >= (ndim > 0 ? ndim : 1)) return fail(MPB_ERR_INVALID, "musapy kernel ABI: axis %d", axis);
  RedReq r{};
  r.op = op;
  r.ndim = d.nd;
  r.shape = d.shape;
  r.strides = d.sa;
  r.a = a;
  r.in_dt = dt;
  r.axes_mask = 1ull << axis;
  r.out = c;
  r.out_dt = out_dt;
  r.compute_dt = dt;
  r.nan_first_rule = 1;
  r.allow_split = 0;
  r.out_stride = ostride;
  return red_run(r, s);
}

void reduce_v2(int op, int dt, int out_dt, const void* a, void* c, int ndim, const size_t* in_shape,
               const ptrdiff_t* in_strides, int axis, cudaStream_t s) {
  PeekGuard g;
  reduce_axis(op, dt, out_dt, a, c, ndim, in_shape, in_strides, axis, 1, s);
}

// ---------------------------------------------------------------- stages
// Fill tiles 1..tiles-1 of each output with the identity (fill_mode 0: zero,
// 1: one) or with a copy of tile 0 (fill_mode 2).
template <class T>
__global__ void k_spread_tiles(T* __restrict__ p, int64_t out_size, int64_t tiles, int fill_mode, T zero, T one) {
  const int64_t n = out_size * tiles;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i % tiles;
    if (t == 0) continue;
    p[i] = fill_mode == 0 ? zero : (fill_mode == 1 ? one : p[i - t]);
  }
}

template <class T>
int spread(T* p, int64_t out_size, int64_t tiles, int mode, T zero, T one, cudaStream_t s) {
  if (tiles <= 1 || out_size == 0) return MPB_OK;
  int64_t blocks = (out_size * tiles + 255) / 256;
  if (blocks > (int64_t)sm_count() * 16) blocks = (int64_t)sm_count() * 16;
  k_spread_tiles<T><<<(unsigned)blocks, 256, 0, s>>>(p, out_size, tiles, mode, zero, one);
  return launch_check("musapy partial stage");
}

template <class T>
void partial_v2(int op, int dt, const T* a, T* partials, int ndim, const size_t* in_shape, const ptrdiff_t* in_strides,
                int axis, size_t out_size, size_t tiles, T zero, T one, cudaStream_t s) {
  PeekGuard g;
  const int red = op == MPB_R_MEAN ? MPB_R_SUM : op;  // a mean partial is a sum partial
  if (reduce_axis(red, dt, dt, a, partials, ndim, in_shape, in_strides, axis, (int64_t)tiles, s)) return;
  const int mode = (op == MPB_R_MAX || op == MPB_R_MIN) ? 2 : (op == MPB_R_PROD ? 1 : 0);
  spread<T>(partials, (int64_t)out_size, (int64_t)tiles, mode, zero, one, s);
}

template <class T>
void arg_partial_v2(bool is_max, int dt, const T* a, T* pv, int64_t* pi, int ndim, const size_t* in_shape,
                    const ptrdiff_t* in_strides, int axis, size_t out_size, size_t tiles, cudaStream_t s) {
  PeekGuard g;
  if (reduce_axis(is_max ? MPB_R_MAX : MPB_R_MIN, dt, dt, a, pv, ndim, in_shape, in_strides, axis, (int64_t)tiles, s))
    return;
  if (reduce_axis(is_max ? MPB_R_ARGMAX : MPB_R_ARGMIN, dt, MPB_I64, a, pi, ndim, in_shape, in_strides, axis,
                  (int64_t)tiles, s))
    return;
  if (spread<T>(pv, (int64_t)out_size, (int64_t)tiles, 2, T(), T(), s)) return;
  spread<int64_t>(pi, (int64_t)out_size, (int64_t)tiles, 2, 0, 0, s);
}

// (value, index) candidate rule of musapy's CPU path: strictly better value,
// or equal value with a lower index; a NaN is taken only as the first element
// (index 0).
template <class T> MPB_D bool nan_of(T v) { return v != v; }
template <> MPB_D bool nan_of<int64_t>(int64_t) { return false; }

template <class T>
MPB_D void arg_take(bool is_max, T v, int64_t i, T& bv, int64_t& bi, bool& have, bool& nan0) {
  if (nan0) return;
  if (nan_of(v)) {
    if (i == 0) {
      bv = v;
      bi = 0;
      have = true;
      nan0 = true;
    }
    return;
  }
  if (!have || (is_max ? v > bv : v < bv) || (v == bv && i < bi)) {
    bv = v;
    bi = i;
    have = true;
  }
}

// Mid stage: pairs [o][tiles] -> [o][ceil(tiles/1024)], one thread per output group.
template <class T>
__global__ void k_arg_mid(const T* __restrict__ pv, const int64_t* __restrict__ pi, T* __restrict__ ov,
                          int64_t* __restrict__ oi, int64_t out_size, int64_t tiles, int is_max) {
  const int64_t groups = (tiles + 1023) / 1024;
  const int64_t n = out_size * groups;
  for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < n; k += (int64_t)gridDim.x * blockDim.x) {
    const int64_t o = k / groups, gidx = k % groups;
    const int64_t t0 = gidx * 1024, t1 = t0 + 1024 < tiles ? t0 + 1024 : tiles;
    T bv = pv[o * tiles + t0];
    int64_t bi = pi[o * tiles + t0];
    bool have = false, nan0 = false;
    for (int64_t t = t0; t < t1; ++t) arg_take<T>(is_max != 0, pv[o * tiles + t], pi[o * tiles + t], bv, bi, have, nan0);
    ov[k] = bv;
    oi[k] = bi;
  }
}

template <class T>
__global__ void k_arg_final(const T* __restrict__ pv, const int64_t* __restrict__ pi, int64_t* __restrict__ c,
                            int64_t num_partials, int64_t out_size, int is_max) {
  for (int64_t o = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; o < out_size; o += (int64_t)gridDim.x * blockDim.x) {
    T bv = pv[o * num_partials];
    int64_t bi = pi[o * num_partials];
    bool have = false, nan0 = false;
    for (int64_t t = 0; t < num_partials; ++t)
      arg_take<T>(is_max != 0, pv[o * num_partials + t], pi[o * num_partials + t], bv, bi, have, nan0);
    c[o] = bi;
  }
}

inline unsigned grid_of(int64_t n) {
  int64_t b = (n + 255) / 256;
  if (b > (int64_t)sm_count() * 16) b = (int64_t)sm_count() * 16;
  return (unsigned)(b < 1 ? 1 : b);
}

template <class T>
void arg_mid_v2(bool is_max, const T* pv, const int64_t* pi, T* ov, int64_t* oi, size_t out_size, size_t tiles,
                cudaStream_t s) {
  PeekGuard g;
  const int64_t n = (int64_t)out_size * (((int64_t)tiles + 1023) / 1024);
  if (n == 0) return;
  k_arg_mid<T><<<grid_of(n), 256, 0, s>>>(pv, pi, ov, oi, (int64_t)out_size, (int64_t)tiles, is_max);
  launch_check("musapy arg mid stage");
}

template <class T>
void arg_final_v2(bool is_max, const T* pv, const int64_t* pi, int64_t* c, size_t num_partials, size_t out_size,
                  cudaStream_t s) {
  PeekGuard g;
  if (out_size == 0 || num_partials == 0) return;
  k_arg_final<T><<<grid_of((int64_t)out_size), 256, 0, s>>>(pv, pi, c, (int64_t)num_partials, (int64_t)out_size,
                                                             is_max);
  launch_check("musapy arg final stage");
}

// Final stage of sum/prod/max/min/mean (and complex sum/prod/mean): each
// output folds its num_partials partials in order; mean divides by axis_len.
template <class T> struct FinalAcc { using type = T; };
template <> struct FinalAcc<c64> { using type = c128; };

MPB_D c128 cadd(c128 a, c128 b) { return c128{a.re + b.re, a.im + b.im}; }
MPB_D c128 cmul(c128 a, c128 b) {
  return c128{__dsub_rn(__dmul_rn(a.re, b.re), __dmul_rn(a.im, b.im)),
              __dadd_rn(__dmul_rn(a.re, b.im), __dmul_rn(a.im, b.re))};
}

template <class T> MPB_D T wadd(T a, T b) { return a + b; }
template <> MPB_D int64_t wadd<int64_t>(int64_t a, int64_t b) { return (int64_t)((uint64_t)a + (uint64_t)b); }
template <class T> MPB_D T wmul(T a, T b) { return a * b; }
template <> MPB_D int64_t wmul<int64_t>(int64_t a, int64_t b) { return (int64_t)((uint64_t)a * (uint64_t)b); }

template <class T>
__global__ void k_final_real(const T* __restrict__ p, T* __restrict__ c, int64_t np, int64_t out_size, int op,
                             int64_t axis_len) {
  for (int64_t o = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; o < out_size; o += (int64_t)gridDim.x * blockDim.x) {
    const T* q = p + o * np;
    T acc = q[0];
    for (int64_t t = 1; t < np; ++t) {
      const T v = q[t];
      if (op == MPB_R_SUM || op == MPB_R_MEAN) acc = wadd<T>(acc, v);
      else if (op == MPB_R_PROD) acc = wmul<T>(acc, v);
      else if (op == MPB_R_MAX) { if (v > acc) acc = v; }
      else { if (v < acc) acc = v; }
    }
    if (op == MPB_R_MEAN) acc = acc / (T)axis_len;
    c[o] = acc;
  }
}

template <class C>
__global__ void k_final_cplx(const C* __restrict__ p, C* __restrict__ c, int64_t np, int64_t out_size, int op,
                             int64_t axis_len) {
  for (int64_t o = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; o < out_size; o += (int64_t)gridDim.x * blockDim.x) {
    const C* q = p + o * np;
    c128 acc = cvt<c128>(q[0]);
    for (int64_t t = 1; t < np; ++t) acc = op == MPB_R_PROD ? cmul(acc, cvt<c128>(q[t])) : cadd(acc, cvt<c128>(q[t]));
    if (op == MPB_R_MEAN) acc = c128{acc.re / (double)axis_len, acc.im / (double)axis_len};
    c[o] = cvt<C>(acc);
  }
}

template <class T>
void final_v2(int op, const T* p, T* c, size_t np, size_t out_size, size_t axis_len, cudaStream_t s) {
  PeekGuard g;
  if (out_size == 0 || np == 0) return;
  k_final_real<T><<<grid_of((int64_t)out_size), 256, 0, s>>>(p, c, (int64_t)np, (int64_t)out_size, op,
                                                             (int64_t)axis_len);
  launch_check("musapy final stage");
}

template <class C>
void final_cplx_v2(int op, const C* p, C* c, size_t np, size_t out_size, size_t axis_len, cudaStream_t s) {
  PeekGuard g;
  if (out_size == 0 || np == 0) return;
  k_final_cplx<C><<<grid_of((int64_t)out_size), 256, 0, s>>>(p, c, (int64_t)np, (int64_t)out_size, op,
                                                             (int64_t)axis_len);
  launch_check("musapy final stage");
}

// Cumsum v3 with musapy's caller-sized scratch (op_builder.rs:3301-3319).
void cumsum_v3(int dt, size_t esz, const void* a, void* c, void* tmp, int ndim, const size_t* in_shape,
               const ptrdiff_t* in_strides, int axis, size_t axis_len, size_t out_size, cudaStream_t s) {
  PeekGuard g;
  Dims d;
  if (!load(ndim, in_shape, in_strides, nullptr, d)) return;
  const size_t bpr = (axis_len + 255) / 256;
  const size_t rows = axis_len ? out_size / axis_len : 0;
  size_t elems = 0;
  if (bpr > 1) elems = bpr > 256 ? rows * (bpr + (bpr + 255) / 256) : rows * bpr;
  ScanReq r{};
  r.ndim = d.nd;
  r.shape = d.shape;
  r.strides = d.sa;
  r.a = a;
  r.in_dt = dt;
  r.axis = axis;
  r.out = c;
  r.out_dt = dt;
  r.scratch = tmp;
  r.scratch_bytes = tmp ? elems * esz : 0;
  scan_run(r, s);
}

// ------------------------------------------------------------- creation
template <class T>
__global__ void k_arange(T* __restrict__ out, T start, T step, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    if constexpr (std::is_same<T, float>::value) out[i] = __fadd_rn(start, __fmul_rn((float)i, step));
    else if constexpr (std::is_same<T, double>::value) out[i] = __dadd_rn(start, __dmul_rn((double)i, step));
    else out[i] = (T)((uint64_t)start + (uint64_t)i * (uint64_t)step);
  }
}
template <class T>
__global__ void k_eye(T* __restrict__ out, int64_t n, int64_t m, int k) {
  const int64_t total = n * m;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / m, col = i % m;
    out[i] = (col - row == (int64_t)k) ? (T)1 : (T)0;
  }
}
template <class T>
void arange(T* out, T start, T step, size_t n, cudaStream_t s) {
  PeekGuard g;
  if (n == 0) return;
  k_arange<T><<<grid_of((int64_t)n), 256, 0, s>>>(out, start, step, (int64_t)n);
  launch_check("musapy arange");
}
template <class T>
void eye(T* out, size_t n, size_t m, int k, cudaStream_t s) {
  PeekGuard g;
  if (n * m == 0) return;
  k_eye<T><<<grid_of((int64_t)(n * m)), 256, 0, s>>>(out, (int64_t)n, (int64_t)m, k);
  launch_check("musapy eye");
}
template <class T>
void fill(int dt, T* out, double re, size_t n, cudaStream_t s) {
  PeekGuard g;
  EwReq r;
  const int64_t shape = (int64_t)n;
  r.op = MPB_FILL;
  r.ndim = 1;
  r.shape = &shape;
  r.a = nullptr;
  r.a_dt = dt;
  r.a_st = nullptr;
  r.b = nullptr;
  r.b_dt = dt;
  r.b_st = nullptr;
  r.out = out;
  r.out_dt = dt;
  r.compute_dt = dt;
  r.p0 = re;
  r.p1 = 0.0;
  ew_run(r, s);
}

}  // namespace ref
}  // namespace mpb

using namespace mpb;
using namespace mpb::ref;

extern "C" {

// ------------------------------------------------------------ binary
#define REF_BINARY(OP, OPC, SUF, T, DT)                                                                      \
  void musapy_##OP##_##SUF##_v2(const T* a, const T* b, T* c, int32_t ndim, const size_t* shape,           \
                                 const ptrdiff_t* as, const ptrdiff_t* bs, cudaStream_t s) {                \
    ew(OPC, DT, DT, DT, DT, a, b, c, ndim, shape, as, bs, 0.0, 0.0, s);                                    \
  }
#define REF_BINARY_REAL(OP, OPC) REF_BINARY(OP, OPC, f32, float, MPB_F32) REF_BINARY(OP, OPC, f64, double, MPB_F64)
#define REF_BINARY_CPLX(OP, OPC) REF_BINARY(OP, OPC, c64, c64, MPB_C64) REF_BINARY(OP, OPC, c128, c128, MPB_C128)
REF_BINARY_REAL(add, MPB_ADD)
REF_BINARY_REAL(sub, MPB_SUB)
REF_BINARY_REAL(mul, MPB_MUL)
REF_BINARY_REAL(div, MPB_DIV)
REF_BINARY_REAL(pow, MPB_POW)
REF_BINARY_CPLX(add, MPB_ADD)
REF_BINARY_CPLX(sub, MPB_SUB)
REF_BINARY_CPLX(mul, MPB_MUL)
REF_BINARY_CPLX(div, MPB_DIV)

// ------------------------------------------------------------- unary
#define REF_UNARY(OP, OPC, SUF, TI, TO, DI, DO)                                                              \
  void musapy_##OP##_##SUF##_v2(const TI* a, TO* c, int32_t ndim, const size_t* shape, const ptrdiff_t* as, \
                                 cudaStream_t s) {                                                         \
    ew(OPC, DI, DI, DO, DI, a, nullptr, c, ndim, shape, as, nullptr, 0.0, 0.0, s);                         \
  }
#define REF_UNARY_REAL(OP, OPC) \
  REF_UNARY(OP, OPC, f32, float, float, MPB_F32, MPB_F32) REF_UNARY(OP, OPC, f64, double, double, MPB_F64, MPB_F64)
REF_UNARY_REAL(sin, MPB_SIN)
REF_UNARY_REAL(cos, MPB_COS)
REF_UNARY_REAL(exp, MPB_EXP)
REF_UNARY_REAL(log, MPB_LOG)
REF_UNARY_REAL(abs, MPB_ABS)
REF_UNARY_REAL(sign, MPB_SIGN)
REF_UNARY_REAL(neg, MPB_NEG)
REF_UNARY(neg, MPB_NEG, c64, c64, c64, MPB_C64, MPB_C64)
REF_UNARY(neg, MPB_NEG, c128, c128, c128, MPB_C128, MPB_C128)
REF_UNARY(abs, MPB_ABS, c64, c64, float, MPB_C64, MPB_F32)
REF_UNARY(abs, MPB_ABS, c128, c128, double, MPB_C128, MPB_F64)

void musapy_clamp_f32_v2(const float* a, float* c, float lo, float hi, int32_t ndim, const size_t* shape,
                         const ptrdiff_t* as, cudaStream_t s) {
  ew(MPB_CLAMP, MPB_F32, MPB_F32, MPB_F32, MPB_F32, a, nullptr, c, ndim, shape, as, nullptr, lo, hi, s);
}
void musapy_clamp_f64_v2(const double* a, double* c, double lo, double hi, int32_t ndim, const size_t* shape,
                         const ptrdiff_t* as, cudaStream_t s) {
  ew(MPB_CLAMP, MPB_F64, MPB_F64, MPB_F64, MPB_F64, a, nullptr, c, ndim, shape, as, nullptr, lo, hi, s);
}

// -------------------------------------------------------------- casts
#define REF_CAST(SS, DS, TS, TD, DTS, DTD)                                                                  \
  void musapy_cast_##SS##_##DS##_v2(const TS* a, TD* c, int32_t ndim, const size_t* shape,                 \
                                     const ptrdiff_t* as, cudaStream_t s) {                               \
    ew(MPB_CAST, DTS, DTS, DTD, DTD, a, nullptr, c, ndim, shape, as, nullptr, 0.0, 0.0, s);                \
  }
#define REF_CAST_FROM_INTS(DS, TD, DTD)                                                                         \
  REF_CAST(i8, DS, int8_t, TD, MPB_I8, DTD) REF_CAST(i16, DS, int16_t, TD, MPB_I16, DTD)                       \
  REF_CAST(i32, DS, int32_t, TD, MPB_I32, DTD) REF_CAST(u8, DS, uint8_t, TD, MPB_U8, DTD)                       \
  REF_CAST(u16, DS, uint16_t, TD, MPB_U16, DTD) REF_CAST(u32, DS, uint32_t, TD, MPB_U32, DTD)                   \
  REF_CAST(u64, DS, uint64_t, TD, MPB_U64, DTD)
REF_CAST_FROM_INTS(f32, float, MPB_F32)
REF_CAST(i64, f32, int64_t, float, MPB_I64, MPB_F32)
REF_CAST(f64, f32, double, float, MPB_F64, MPB_F32)
REF_CAST_FROM_INTS(f64, double, MPB_F64)
REF_CAST(i64, f64, int64_t, double, MPB_I64, MPB_F64)
REF_CAST(f32, f64, float, double, MPB_F32, MPB_F64)
REF_CAST_FROM_INTS(i64, int64_t, MPB_I64)
REF_CAST(f32, i64, float, int64_t, MPB_F32, MPB_I64)
REF_CAST(f64, i64, double, int64_t, MPB_F64, MPB_I64)
REF_CAST(f32, c64, float, c64, MPB_F32, MPB_C64)
REF_CAST(f32, c128, float, c128, MPB_F32, MPB_C128)
REF_CAST(f64, c64, double, c64, MPB_F64, MPB_C64)
REF_CAST(f64, c128, double, c128, MPB_F64, MPB_C128)
REF_CAST(c64, c128, c64, c128, MPB_C64, MPB_C128)

// -------------------------------------------------------- comparisons
#define REF_CMP(OP, OPC, SUF, T, DT)                                                                          \
  void musapy_##OP##_##SUF##_v2(const T* a, const T* b, uint8_t* c, int32_t ndim, const size_t* shape,       \
                                 const ptrdiff_t* as, const ptrdiff_t* bs, cudaStream_t s) {                \
    ew(OPC, DT, DT, MPB_BOOL, DT, a, b, c, ndim, shape, as, bs, 0.0, 0.0, s);                              \
  }
#define REF_CMP_REAL(OP, OPC) REF_CMP(OP, OPC, f32, float, MPB_F32) REF_CMP(OP, OPC, f64, double, MPB_F64)
REF_CMP_REAL(eq, MPB_EQ)
REF_CMP_REAL(ne, MPB_NE)
REF_CMP_REAL(lt, MPB_LT)
REF_CMP_REAL(gt, MPB_GT)
REF_CMP_REAL(le, MPB_LE)
REF_CMP_REAL(ge, MPB_GE)
REF_CMP(eq, MPB_EQ, c64, c64, MPB_C64)
REF_CMP(eq, MPB_EQ, c128, c128, MPB_C128)
REF_CMP(ne, MPB_NE, c64, c64, MPB_C64)
REF_CMP(ne, MPB_NE, c128, c128, MPB_C128)

// --------------------------------------------- reductions, one launch
#define REF_RED(OP, OPC, SUF, T, DT, TO, DTO)                                                                 \
  void musapy_##OP##_##SUF##_v2(const T* a, TO* c, int32_t ndim, const size_t* in_shape,                      \
                                 const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, \
                                 cudaStream_t s) {                                                         \
    (void)axis_len;                                                                                        \
    (void)out_size;                                                                                        \
    reduce_v2(OPC, DT, DTO, a, c, ndim, in_shape, in_strides, axis, s);                                    \
  }                                                                                                        \
  void musapy_##OP##_small_axis_##SUF##_v2(const T* a, TO* c, int32_t ndim, const size_t* in_shape,           \
                                            const ptrdiff_t* in_strides, int32_t axis, size_t axis_len,       \
                                            size_t out_size, int32_t group_size, cudaStream_t s) {         \
    (void)axis_len;                                                                                        \
    (void)out_size;                                                                                        \
    (void)group_size;                                                                                      \
    reduce_v2(OPC, DT, DTO, a, c, ndim, in_shape, in_strides, axis, s);                                    \
  }
#define REF_RED3(OP, OPC)                                                                                    \
  REF_RED(OP, OPC, i64, int64_t, MPB_I64, int64_t, MPB_I64) REF_RED(OP, OPC, f32, float, MPB_F32, float, MPB_F32) \
  REF_RED(OP, OPC, f64, double, MPB_F64, double, MPB_F64)
REF_RED3(sum, MPB_R_SUM)
REF_RED3(prod, MPB_R_PROD)
REF_RED3(max, MPB_R_MAX)
REF_RED3(min, MPB_R_MIN)
REF_RED(mean, MPB_R_MEAN, f32, float, MPB_F32, float, MPB_F32)
REF_RED(mean, MPB_R_MEAN, f64, double, MPB_F64, double, MPB_F64)
REF_RED(sum, MPB_R_SUM, c64, c64, MPB_C64, c64, MPB_C64)
REF_RED(sum, MPB_R_SUM, c128, c128, MPB_C128, c128, MPB_C128)
REF_RED(prod, MPB_R_PROD, c64, c64, MPB_C64, c64, MPB_C64)
REF_RED(prod, MPB_R_PROD, c128, c128, MPB_C128, c128, MPB_C128)
REF_RED(mean, MPB_R_MEAN, c64, c64, MPB_C64, c64, MPB_C64)
REF_RED(mean, MPB_R_MEAN, c128, c128, MPB_C128, c128, MPB_C128)

#define REF_ARG(OP, OPC, SUF, T, DT)                                                                          \
  void musapy_##OP##_##SUF##_v2(const T* a, int64_t* c, int32_t ndim, const size_t* in_shape,                \
                                 const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, \
                                 cudaStream_t s) {                                                         \
    (void)axis_len;                                                                                        \
    (void)out_size;                                                                                        \
    reduce_v2(OPC, DT, MPB_I64, a, c, ndim, in_shape, in_strides, axis, s);                                \
  }
#define REF_ARG3(OP, OPC) \
  REF_ARG(OP, OPC, i64, int64_t, MPB_I64) REF_ARG(OP, OPC, f32, float, MPB_F32) REF_ARG(OP, OPC, f64, double, MPB_F64)
REF_ARG3(argmax, MPB_R_ARGMAX)
REF_ARG3(argmin, MPB_R_ARGMIN)

// ----------------------------------------------- partial / final stages
#define REF_PARTIAL(OP, OPC, SUF, T, DT, ZERO, ONE)                                                           \
  void musapy_##OP##_partial_##SUF##_v2(const T* a, T* partials, int32_t ndim, const size_t* in_shape,        \
                                         const ptrdiff_t* in_strides, int32_t axis, size_t axis_len,          \
                                         size_t out_size, size_t tiles_per_output, cudaStream_t s) {       \
    (void)axis_len;                                                                                        \
    partial_v2<T>(OPC, DT, a, partials, ndim, in_shape, in_strides, axis, out_size, tiles_per_output, ZERO,  \
                  ONE, s);                                                                                 \
  }
#define REF_FINAL(OP, OPC, SUF, T)                                                                            \
  void musapy_##OP##_final_##SUF##_v2(const T* partials, T* c, size_t num_partials, size_t out_size,          \
                                       cudaStream_t s) {                                                   \
    final_v2<T>(OPC, partials, c, num_partials, out_size, 1, s);                                           \
  }
#define REF_STAGES(OP, OPC)                                                                                  \
  REF_PARTIAL(OP, OPC, i64, int64_t, MPB_I64, (int64_t)0, (int64_t)1)                                        \
  REF_PARTIAL(OP, OPC, f32, float, MPB_F32, 0.0f, 1.0f) REF_PARTIAL(OP, OPC, f64, double, MPB_F64, 0.0, 1.0)   \
  REF_FINAL(OP, OPC, i64, int64_t) REF_FINAL(OP, OPC, f32, float) REF_FINAL(OP, OPC, f64, double)
REF_STAGES(sum, MPB_R_SUM)
REF_STAGES(prod, MPB_R_PROD)
REF_STAGES(max, MPB_R_MAX)
REF_STAGES(min, MPB_R_MIN)
REF_PARTIAL(mean, MPB_R_MEAN, f32, float, MPB_F32, 0.0f, 1.0f)
REF_PARTIAL(mean, MPB_R_MEAN, f64, double, MPB_F64, 0.0, 1.0)
void musapy_mean_final_f32_v2(const float* p, float* c, size_t np, size_t out_size, size_t axis_len, cudaStream_t s) {
  final_v2<float>(MPB_R_MEAN, p, c, np, out_size, axis_len, s);
}
void musapy_mean_final_f64_v2(const double* p, double* c, size_t np, size_t out_size, size_t axis_len,
                              cudaStream_t s) {
  final_v2<double>(MPB_R_MEAN, p, c, np, out_size, axis_len, s);
}

#define REF_CPLX_STAGES(OP, OPC, SUF, C, DT, ZERO, ONE)                                                       \
  REF_PARTIAL(OP, OPC, SUF, C, DT, ZERO, ONE)                                                                \
  void musapy_##OP##_final_##SUF##_v2(const C* partials, C* c, size_t num_partials, size_t out_size,          \
                                       size_t axis_len, cudaStream_t s) {                                  \
    final_cplx_v2<C>(OPC, partials, c, num_partials, out_size, axis_len, s);                               \
  }
REF_CPLX_STAGES(sum, MPB_R_SUM, c64, c64, MPB_C64, (c64{0.0f, 0.0f}), (c64{1.0f, 0.0f}))
REF_CPLX_STAGES(sum, MPB_R_SUM, c128, c128, MPB_C128, (c128{0.0, 0.0}), (c128{1.0, 0.0}))
REF_CPLX_STAGES(prod, MPB_R_PROD, c64, c64, MPB_C64, (c64{0.0f, 0.0f}), (c64{1.0f, 0.0f}))
REF_CPLX_STAGES(prod, MPB_R_PROD, c128, c128, MPB_C128, (c128{0.0, 0.0}), (c128{1.0, 0.0}))
REF_CPLX_STAGES(mean, MPB_R_MEAN, c64, c64, MPB_C64, (c64{0.0f, 0.0f}), (c64{1.0f, 0.0f}))
REF_CPLX_STAGES(mean, MPB_R_MEAN, c128, c128, MPB_C128, (c128{0.0, 0.0}), (c128{1.0, 0.0}))

#define REF_ARG_STAGES(OP, ISMAX, SUF, T, DT)                                                                 \
  void musapy_##OP##_partial_##SUF##_v2(const T* a, T* pv, int64_t* pi, int32_t ndim, const size_t* in_shape,  \
                                         const ptrdiff_t* in_strides, int32_t axis, size_t axis_len,          \
                                         size_t out_size, size_t tiles_per_output, cudaStream_t s) {       \
    (void)axis_len;                                                                                        \
    arg_partial_v2<T>(ISMAX, DT, a, pv, pi, ndim, in_shape, in_strides, axis, out_size, tiles_per_output, s); \
  }                                                                                                        \
  void musapy_##OP##_final_##SUF##_v2(const T* pv, const int64_t* pi, int64_t* c, size_t num_partials,        \
                                       size_t out_size, cudaStream_t s) {                                  \
    arg_final_v2<T>(ISMAX, pv, pi, c, num_partials, out_size, s);                                          \
  }                                                                                                        \
  void musapy_##OP##_mid_##SUF##_v2(const T* pv, const int64_t* pi, T* ov, int64_t* oi, size_t out_size,      \
                                     size_t tiles_per_output, size_t axis_len, cudaStream_t s) {           \
    (void)axis_len;                                                                                        \
    arg_mid_v2<T>(ISMAX, pv, pi, ov, oi, out_size, tiles_per_output, s);                                   \
  }
REF_ARG_STAGES(argmax, true, i64, int64_t, MPB_I64)
REF_ARG_STAGES(argmax, true, f32, float, MPB_F32)
REF_ARG_STAGES(argmax, true, f64, double, MPB_F64)
REF_ARG_STAGES(argmin, false, i64, int64_t, MPB_I64)
REF_ARG_STAGES(argmin, false, f32, float, MPB_F32)
REF_ARG_STAGES(argmin, false, f64, double, MPB_F64)

// ------------------------------------------------------------- cumsum
#define REF_CUMSUM(SUF, T, DT)                                                                                \
  void musapy_cumsum_##SUF##_v3(const T* a, T* c, T* tmp, int32_t ndim, const size_t* in_shape,              \
                                 const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, \
                                 cudaStream_t s) {                                                         \
    cumsum_v3(DT, sizeof(T), a, c, tmp, ndim, in_shape, in_strides, axis, axis_len, out_size, s);          \
  }
REF_CUMSUM(i64, int64_t, MPB_I64)
REF_CUMSUM(f32, float, MPB_F32)
REF_CUMSUM(f64, double, MPB_F64)

// ----------------------------------------------------------- creation
#define REF_FILL(SUF, T, DT) \
  void musapy_fill_##SUF(T* out, T value, size_t n, cudaStream_t s) { fill<T>(DT, out, (double)value, n, s); }
REF_FILL(f32, float, MPB_F32)
REF_FILL(f64, double, MPB_F64)
REF_FILL(i64, int64_t, MPB_I64)
REF_FILL(i32, int32_t, MPB_I32)
REF_FILL(i16, int16_t, MPB_I16)
REF_FILL(i8, int8_t, MPB_I8)
REF_FILL(u64, uint64_t, MPB_U64)
REF_FILL(u32, uint32_t, MPB_U32)
REF_FILL(u16, uint16_t, MPB_U16)
REF_FILL(u8, uint8_t, MPB_U8)
#define REF_ARANGE(SUF, T) \
  void musapy_arange_##SUF(T* out, T start, T step, size_t n, cudaStream_t s) { arange<T>(out, start, step, n, s); }
REF_ARANGE(f32, float)
REF_ARANGE(f64, double)
REF_ARANGE(i64, int64_t)
REF_ARANGE(i32, int32_t)
// linspace: step = (stop - start) / (n - 1) in T, then start + i*step (init.mu wrapper semantics)
void musapy_linspace_f32(float* out, float start, float stop, size_t n, cudaStream_t s) {
  const float step = n > 1 ? (stop - start) / (float)(n - 1) : 0.0f;
  arange<float>(out, start, step, n, s);
}
void musapy_linspace_f64(double* out, double start, double stop, size_t n, cudaStream_t s) {
  const double step = n > 1 ? (stop - start) / (double)(n - 1) : 0.0;
  arange<double>(out, start, step, n, s);
}
#define REF_EYE(SUF, T) \
  void musapy_eye_##SUF(T* out, size_t n, size_t m, int32_t k, cudaStream_t s) { eye<T>(out, n, m, k, s); }
REF_EYE(f32, float)
REF_EYE(f64, double)
REF_EYE(i64, int64_t)
REF_EYE(i32, int32_t)

// --------------------------------------------------------------- copy
#define REF_COPY(SUF, T, DT)                                                                                  \
  void musapy_copy_##SUF(const T* input, T* output, int32_t ndim, const size_t* shape,                        \
                         const ptrdiff_t* in_strides, cudaStream_t s) {                                    \
    ew(MPB_CAST, DT, DT, DT, DT, input, nullptr, output, ndim, shape, in_strides, nullptr, 0.0, 0.0, s);     \
  }                                                                                                        \
  void musapy_copy_transpose2d_##SUF(const T* src, T* dst, size_t rows, size_t cols, cudaStream_t s) {     \
    const size_t shape[2] = {rows, cols};                                                                  \
    const ptrdiff_t st[2] = {1, (ptrdiff_t)rows};                                                          \
    ew(MPB_CAST, DT, DT, DT, DT, src, nullptr, dst, 2, shape, st, nullptr, 0.0, 0.0, s);                   \
  }
REF_COPY(f32, float, MPB_F32)
REF_COPY(f64, double, MPB_F64)
REF_COPY(i32, int32_t, MPB_I32)
REF_COPY(i64, int64_t, MPB_I64)

}  // extern "C"
