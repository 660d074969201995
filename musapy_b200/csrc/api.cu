// Extended C-ABI of libmusapy_b200: status-returning entry points with a
// dtype tag per operand (fused promotion casts), host-side helpers that
// restate musapy's promotion and broadcast rules, and plan inspection hooks
// used by the CPU test-suite. Declarations live in include/musapy_b200.h.
#include <stdarg.h>
#include <stdio.h>
#include <string.h>
#include "internal.h"
#include "plan.h"
#include "reduce.h"

namespace mpb {

static thread_local char g_err[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_check(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return MPB_OK;
  return fail(MPB_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

static unsigned long long g_launches = 0;
static thread_local bool g_preserve_last_error = false;

void set_preserve_last_error(bool on) { g_preserve_last_error = on; }

int launch_check(const char* what) {
  __atomic_add_fetch(&g_launches, 1ull, __ATOMIC_RELAXED);
  return cuda_check(g_preserve_last_error ? cudaPeekAtLastError() : cudaGetLastError(), what);
}

int launch_check_pdl(cudaError_t e, const char* what) {
  const int rc = launch_check(what);
  if (rc) return rc;
  return cuda_check(e, what);
}

int sm_count() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    cudaGetLastError();
    return 148;  // B200; used only when planning without a device
  }
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = 148;
    }
    cache[dev] = n;
  }
  return cache[dev];
}

// ------------------------------------------------------------ promotion
// Restatement of rust/musapy-core/src/dtype.rs:206-338 (jax_promote and
// promote with the GPU narrow-first rule).
namespace {
int category(int d) {
  if (d == MPB_BOOL) return 0;
  if (d >= MPB_I8 && d <= MPB_I64) return 1;
  if (d >= MPB_U8 && d <= MPB_U64) return 2;
  if (d == MPB_F16 || d == MPB_F32 || d == MPB_F64 || d == MPB_BF16) return 3;
  return 4;
}
int width(int d) {
  switch (d) {
    case MPB_BOOL: case MPB_I8: case MPB_U8: return 8;
    case MPB_I16: case MPB_U16: case MPB_F16: case MPB_BF16: return 16;
    case MPB_I32: case MPB_U32: case MPB_F32: case MPB_C64: return 32;
    default: return 64;
  }
}
int int_of(int w) { return w == 8 ? MPB_I8 : w == 16 ? MPB_I16 : w == 32 ? MPB_I32 : MPB_I64; }
int float_of(int w) { return w == 16 ? MPB_F16 : w == 32 ? MPB_F32 : MPB_F64; }
int complex_of(int w) { return w <= 32 ? MPB_C64 : MPB_C128; }

int jax_promote(int a, int b) {
  if (a == b) return a;
  if (a == MPB_BOOL) return b;
  if (b == MPB_BOOL) return a;
  const int ca = category(a), cb = category(b), pa = width(a), pb = width(b);
  if (ca == cb) {
    if (ca == 3 && pa == pb) return MPB_F32;  // f16 + bf16
    return pa >= pb ? a : b;
  }
  if ((ca == 1 && cb == 2) || (ca == 2 && cb == 1)) {
    const int iw = ca == 1 ? pa : pb, uw = ca == 1 ? pb : pa;
    const int t = iw > uw ? iw : (uw * 2 > 64 ? 64 : uw * 2);
    return int_of(t);
  }
  if ((ca == 1 || ca == 2) && cb == 3) return b == MPB_BF16 ? MPB_BF16 : float_of(pb);
  if ((cb == 1 || cb == 2) && ca == 3) return a == MPB_BF16 ? MPB_BF16 : float_of(pa);
  if ((ca == 1 || ca == 2) && cb == 4) { int t = pa > pb ? pa : pb; return complex_of(t > 32 ? t : 32); }
  if ((cb == 1 || cb == 2) && ca == 4) { int t = pb > pa ? pb : pa; return complex_of(t > 32 ? t : 32); }
  if (ca == 3 && cb == 4) return complex_of(pa > pb ? pa : pb);
  if (ca == 4 && cb == 3) return complex_of(pa > pb ? pa : pb);
  return -1;
}
}  // namespace

}  // namespace mpb

using namespace mpb;

extern "C" {

const char* mpb_last_error(void) { return g_err; }
// Number of kernels this library has launched in the process so far.
unsigned long long mpb_launch_count(void) { return __atomic_load_n(&g_launches, __ATOMIC_RELAXED); }
int mpb_version(void) { return 1; }
int mpb_num_sms(void) { return sm_count(); }

int mpb_promote(int a, int b, int all_gpu) {
  if (a < 0 || a >= MPB_NUM_DTYPES || b < 0 || b >= MPB_NUM_DTYPES) return -1;
  if (a == b) return a;
  const int jax = jax_promote(a, b);
  if (!all_gpu || jax < 0) return jax;
  const int ca = category(a), cb = category(b), pa = width(a), pb = width(b);
  if (ca != cb) return jax;
  if (ca == 3 && pa == pb && ((a == MPB_F16 && b == MPB_BF16) || (a == MPB_BF16 && b == MPB_F16))) return jax;
  return pa <= pb ? a : b;
}

// NumPy broadcast of two shapes (rust/musapy-ops/src/broadcast.rs:24-58).
// Returns the output ndim, or -1 when the shapes are incompatible.
int mpb_broadcast_shape(int na, const int64_t* sa, int nb, const int64_t* sb, int64_t* out) {
  const int n = na > nb ? na : nb;
  if (n > MPB_MAX_DIMS) return -1;
  for (int i = 0; i < n; ++i) out[i] = 1;
  const int64_t* shapes[2] = {sa, sb};
  const int nds[2] = {na, nb};
  for (int s = 0; s < 2; ++s) {
    const int off = n - nds[s];
    for (int i = 0; i < nds[s]; ++i) {
      const int64_t d = shapes[s][i];
      int64_t& r = out[off + i];
      if (r == 1) r = d;
      else if (d != 1 && d != r) {
        fail(MPB_ERR_SHAPE, "broadcast: incompatible dim %d (%lld vs %lld)", off + i, (long long)r, (long long)d);
        return -1;
      }
    }
  }
  return n;
}

// Operand strides against a broadcast target (broadcast.rs:71-92): kept
// where the extent matches, 0 on broadcast dims and on missing leading dims.
void mpb_broadcast_strides(int nd, const int64_t* shape, const int64_t* strides, int nt, const int64_t* target,
                           int64_t* out) {
  for (int i = 0; i < nt; ++i) out[i] = 0;
  const int off = nt - nd;
  for (int i = 0; i < nd; ++i) {
    const int o = off + i;
    if (o < 0 || o >= nt) continue;
    if (shape[i] == target[o]) out[o] = strides[i];
  }
}

// Collapse `ndim` dims for `nops` operands (strides packed [nops][ndim]).
// Writes the collapsed shape and strides ([nops][result]) and returns the
// collapsed ndim.
int mpb_collapse(int ndim, const int64_t* shape, int nops, const int64_t* strides, int64_t* out_shape,
                 int64_t* out_strides) {
  if (ndim < 0 || ndim > MPB_MAX_DIMS || nops < 1 || nops > 3) return -1;
  const int64_t* sts[3] = {strides, strides + ndim, strides + 2 * ndim};
  Geometry g = collapse(ndim, shape, nops, sts);
  for (int i = 0; i < g.ndim; ++i) {
    out_shape[i] = g.shape[i];
    for (int o = 0; o < nops; ++o) out_strides[o * g.ndim + i] = g.st[o][i];
  }
  return g.ndim;
}

// Kind of kernel the reduction planner picks (RedKind), for host tests.
int mpb_reduce_plan_at(int op, int ndim, const int64_t* shape, const int64_t* strides, const void* a, int in_dtype,
                       uint64_t axes_mask, int64_t* M, int64_t* L, int64_t* splits, int* outputs_per_thread) {
  RedReq r{};
  r.op = op;
  r.ndim = ndim;
  r.shape = shape;
  r.strides = strides;
  r.a = a;
  r.in_dt = in_dtype;
  r.axes_mask = axes_mask;
  r.allow_split = 1;
  RedPlan pl;
  const int rc = red_plan(r, pl);
  if (rc) return -rc;
  if (M) *M = pl.M;
  if (L) *L = pl.L;
  if (splits) *splits = pl.splits;
  if (outputs_per_thread) *outputs_per_thread = pl.colv;
  return pl.kind;
}

int mpb_reduce_plan(int ndim, const int64_t* shape, const int64_t* strides, int in_dtype, uint64_t axes_mask,
                    int64_t* M, int64_t* L, int64_t* splits) {
  return mpb_reduce_plan_at(MPB_R_SUM, ndim, shape, strides, nullptr, in_dtype, axes_mask, M, L, splits, nullptr);
}

int mpb_elementwise(int op, int ndim, const int64_t* shape, const void* a, int a_dtype, const int64_t* a_strides,
                    const void* b, int b_dtype, const int64_t* b_strides, void* out, int out_dtype,
                    int compute_dtype, double p0, double p1, cudaStream_t stream) {
  EwReq r;
  r.op = op;
  r.ndim = ndim;
  r.shape = shape;
  r.a = a;
  r.a_dt = a_dtype;
  r.a_st = a_strides;
  r.b = b;
  r.b_dt = b_dtype;
  r.b_st = b_strides;
  r.out = out;
  r.out_dt = out_dtype;
  r.compute_dt = compute_dtype;
  r.p0 = p0;
  r.p1 = p1;
  return ew_run(r, stream);
}

size_t mpb_reduce_scratch_bytes(int op, int ndim, const int64_t* shape, const int64_t* strides, const void* a,
                                int in_dtype, uint64_t axes_mask, int compute_dtype) {
  RedReq r{};
  r.op = op;
  r.ndim = ndim;
  r.shape = shape;
  r.strides = strides;
  r.a = a;
  r.in_dt = in_dtype;
  r.axes_mask = axes_mask;
  r.compute_dt = compute_dtype;
  r.allow_split = 1;
  return red_scratch_bytes(r);
}

int mpb_reduce(int op, int ndim, const int64_t* shape, const int64_t* strides, const void* a, int in_dtype,
               uint64_t axes_mask, void* out, int out_dtype, int compute_dtype, int nan_first_rule, void* scratch,
               size_t scratch_bytes, cudaStream_t stream) {
  RedReq r{};
  r.op = op;
  r.ndim = ndim;
  r.shape = shape;
  r.strides = strides;
  r.a = a;
  r.in_dt = in_dtype;
  r.axes_mask = axes_mask;
  r.out = out;
  r.out_dt = out_dtype;
  r.compute_dt = compute_dtype;
  r.nan_first_rule = nan_first_rule;
  r.scratch = scratch;
  r.scratch_bytes = scratch_bytes;
  r.allow_split = 1;
  r.out_stride = 1;
  return red_run(r, stream);
}

size_t mpb_cumsum_scratch_bytes(int ndim, const int64_t* shape, const int64_t* strides, const void* a,
                                int in_dtype, int axis, void* out, int out_dtype) {
  ScanReq r{};
  r.ndim = ndim;
  r.shape = shape;
  r.strides = strides;
  r.a = a;
  r.in_dt = in_dtype;
  r.axis = axis;
  r.out = out;
  r.out_dt = out_dtype;
  return scan_scratch_bytes(r);
}

int mpb_cumsum(int ndim, const int64_t* shape, const int64_t* strides, const void* a, int in_dtype, int axis,
               void* out, int out_dtype, void* scratch, size_t scratch_bytes, cudaStream_t stream) {
  ScanReq r{};
  r.ndim = ndim;
  r.shape = shape;
  r.strides = strides;
  r.a = a;
  r.in_dt = in_dtype;
  r.axis = axis;
  r.out = out;
  r.out_dt = out_dtype;
  r.scratch = scratch;
  r.scratch_bytes = scratch_bytes;
  return scan_run(r, stream);
}

// Reads the status word a look-back scan left in its scratch (synchronising
// `stream`): MPB_OK, or MPB_ERR_TIMEOUT when a bounded wait gave up.
int mpb_cumsum_status(const void* scratch, cudaStream_t stream) {
  if (!scratch) return MPB_OK;
  int word = 0;
  int rc = cuda_check(cudaMemcpyAsync(&word, static_cast<const char*>(scratch) + 4, sizeof(int),
                                      cudaMemcpyDeviceToHost, stream),
                      "cumsum status read");
  if (rc) return rc;
  rc = cuda_check(cudaStreamSynchronize(stream), "cumsum status sync");
  if (rc) return rc;
  if (word) return fail(MPB_ERR_TIMEOUT, "cumsum: a bounded look-back wait expired (status 0x%x)", word);
  return MPB_OK;
}

}  // extern "C"
