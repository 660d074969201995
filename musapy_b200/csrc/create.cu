// Creation kernels: arange, linspace, eye (rust/musapy-ops/src/creation.rs:
// 446-521, kernels/init.mu:17-135) as HBM-bound writers.
//
// Values follow the reference CPU path (cpu_fill_ptr, creation.rs:324-400):
// element i is start + i*step evaluated in f64 (a multiply and an add, each
// rounded, never fused) and converted once with Rust `as` semantics, so f32
// and integer outputs match the CPU bit for bit. The reference GPU kernels
// compute in the element type instead; that form stays available through the
// musapy_arange_* / musapy_linspace_* symbols for C callers.
//
// Every generator writes 16-byte packs (st.global.cs) from a grid-stride loop
// over a grid capped at 64 blocks per SM; eye is a fill of zeros followed by a
// kernel that writes only the diagonal.
#include "common.cuh"
#include "internal.h"
#include "musapy_b200.h"

namespace mpb {
namespace {

constexpr int kGenThreads = 256;

template <class T>
struct ArangeGen {
  double start, step;
  MPB_D T operator()(int64_t i) const { return Cvt<T>::from(__dadd_rn(start, __dmul_rn((double)i, step))); }
};
template <class T>
struct ZeroGen {
  MPB_D T operator()(int64_t) const { return Cvt<T>::from(0.0); }
};

template <class T, class G>
__global__ void __launch_bounds__(kGenThreads) k_generate(T* __restrict__ out, int64_t n, G gen, int vec) {
  constexpr int N = sizeof(T) >= 16 ? 1 : 16 / (int)sizeof(T);
  const int64_t gtid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t gstride = (int64_t)gridDim.x * blockDim.x;
  int64_t done = 0;
  if (vec) {
    const int64_t npk = n / N;
    for (int64_t p = gtid; p < npk; p += gstride) {
      uint4 w;
      T* v = reinterpret_cast<T*>(&w);
#pragma unroll
      for (int j = 0; j < N; ++j) v[j] = gen(p * N + j);
      st_stream16(out + p * N, w);
    }
    done = npk * N;
  }
  for (int64_t i = done + gtid; i < n; i += gstride) out[i] = gen(i);
}

// out[r * cols + r + k] = 1 for every row r whose diagonal column lies inside.
template <class T>
__global__ void k_eye_diag(T* __restrict__ out, int64_t r0, int64_t count, int64_t cols, int64_t k) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t < count) {
    const int64_t r = r0 + t;
    out[r * cols + r + k] = Cvt<T>::from(1.0);
  }
}

int grid_of(int64_t items) {
  int64_t b = (items + kGenThreads - 1) / kGenThreads;
  const int64_t cap = (int64_t)sm_count() * 64;
  if (b > cap) b = cap;
  return (int)(b < 1 ? 1 : b);
}

template <class T, class G>
int launch_gen(void* out, int64_t n, const G& g, cudaStream_t s) {
  if (n <= 0) return MPB_OK;
  constexpr int N = sizeof(T) >= 16 ? 1 : 16 / (int)sizeof(T);
  const int vec = (((uintptr_t)out & 15) == 0) ? 1 : 0;
  k_generate<T, G><<<grid_of(vec ? (n + N - 1) / N : n), kGenThreads, 0, s>>>(static_cast<T*>(out), n, g, vec);
  return launch_check("create");
}

template <class T>
int arange_typed(void* out, int64_t n, double start, double step, cudaStream_t s) {
  return launch_gen<T>(out, n, ArangeGen<T>{start, step}, s);
}

int arange_any(void* out, int dt, int64_t n, double start, double step, cudaStream_t s) {
  switch (dt) {
    case MPB_BOOL: return arange_typed<boolean>(out, n, start, step, s);
    case MPB_I8: return arange_typed<int8_t>(out, n, start, step, s);
    case MPB_I16: return arange_typed<int16_t>(out, n, start, step, s);
    case MPB_I32: return arange_typed<int32_t>(out, n, start, step, s);
    case MPB_I64: return arange_typed<int64_t>(out, n, start, step, s);
    case MPB_U8: return arange_typed<uint8_t>(out, n, start, step, s);
    case MPB_U16: return arange_typed<uint16_t>(out, n, start, step, s);
    case MPB_U32: return arange_typed<uint32_t>(out, n, start, step, s);
    case MPB_U64: return arange_typed<uint64_t>(out, n, start, step, s);
    case MPB_F16: return arange_typed<__half>(out, n, start, step, s);
    case MPB_F32: return arange_typed<float>(out, n, start, step, s);
    case MPB_F64: return arange_typed<double>(out, n, start, step, s);
    case MPB_BF16: return arange_typed<__nv_bfloat16>(out, n, start, step, s);
    case MPB_C64: return arange_typed<c64>(out, n, start, step, s);
    case MPB_C128: return arange_typed<c128>(out, n, start, step, s);
    default: return fail(MPB_ERR_DTYPE, "creation: dtype %d not supported", dt);
  }
}

template <class T>
int eye_typed(void* out, int64_t rows, int64_t cols, int64_t k, cudaStream_t s) {
  const int64_t n = rows * cols;
  int rc = launch_gen<T>(out, n, ZeroGen<T>{}, s);
  if (rc != MPB_OK) return rc;
  // rows r with 0 <= r < rows and 0 <= r + k < cols
  const int64_t r0 = k < 0 ? -k : 0;
  int64_t r1 = cols - k;
  if (r1 > rows) r1 = rows;
  if (r1 <= r0) return MPB_OK;
  const int64_t count = r1 - r0;
  k_eye_diag<T><<<(unsigned)((count + 255) / 256), 256, 0, s>>>(static_cast<T*>(out), r0, count, cols, k);
  return launch_check("eye");
}

}  // namespace
}  // namespace mpb

using namespace mpb;

extern "C" {

int mpb_arange(void* out, int dtype, int64_t n, double start, double step, mpb_stream_t stream) {
  if (n < 0) return fail(MPB_ERR_SHAPE, "arange: negative length %lld", (long long)n);
  if (n > 0 && out == nullptr) return fail(MPB_ERR_INVALID, "arange: null output");
  return arange_any(out, dtype, n, start, step, (cudaStream_t)stream);
}

int mpb_linspace(void* out, int dtype, int64_t n, double start, double stop, mpb_stream_t stream) {
  if (n < 0) return fail(MPB_ERR_SHAPE, "linspace: negative length %lld", (long long)n);
  if (n > 0 && out == nullptr) return fail(MPB_ERR_INVALID, "linspace: null output");
  // creation.rs:350-377: step = (stop - start) / (n - 1) in f64; n == 1 gives [start]
  const double step = n > 1 ? (stop - start) / (double)(n - 1) : 0.0;
  return arange_any(out, dtype, n, start, step, (cudaStream_t)stream);
}

int mpb_eye(void* out, int dtype, int64_t rows, int64_t cols, int64_t k, mpb_stream_t stream) {
  if (rows < 0 || cols < 0) return fail(MPB_ERR_SHAPE, "eye: negative shape (%lld, %lld)", (long long)rows, (long long)cols);
  if (rows * cols > 0 && out == nullptr) return fail(MPB_ERR_INVALID, "eye: null output");
  if (rows * cols == 0) return MPB_OK;
  cudaStream_t s = (cudaStream_t)stream;
  switch (dtype) {
    case MPB_BOOL: return eye_typed<boolean>(out, rows, cols, k, s);
    case MPB_I8: return eye_typed<int8_t>(out, rows, cols, k, s);
    case MPB_I16: return eye_typed<int16_t>(out, rows, cols, k, s);
    case MPB_I32: return eye_typed<int32_t>(out, rows, cols, k, s);
    case MPB_I64: return eye_typed<int64_t>(out, rows, cols, k, s);
    case MPB_U8: return eye_typed<uint8_t>(out, rows, cols, k, s);
    case MPB_U16: return eye_typed<uint16_t>(out, rows, cols, k, s);
    case MPB_U32: return eye_typed<uint32_t>(out, rows, cols, k, s);
    case MPB_U64: return eye_typed<uint64_t>(out, rows, cols, k, s);
    case MPB_F16: return eye_typed<__half>(out, rows, cols, k, s);
    case MPB_F32: return eye_typed<float>(out, rows, cols, k, s);
    case MPB_F64: return eye_typed<double>(out, rows, cols, k, s);
    case MPB_BF16: return eye_typed<__nv_bfloat16>(out, rows, cols, k, s);
    case MPB_C64: return eye_typed<c64>(out, rows, cols, k, s);
    case MPB_C128: return eye_typed<c128>(out, rows, cols, k, s);
    default: return fail(MPB_ERR_DTYPE, "eye: dtype %d not supported", dtype);
  }
}

}  // extern "C"
