// Device-side building blocks shared by every kernel of the engine:
// storage types per dtype, conversions with musapy's cast semantics,
// invariant-divisor fast division, and 16-byte vector memory access.
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <utility>
#include "mpb_types.h"

#define MPB_HD __host__ __device__ __forceinline__
#define MPB_D __device__ __forceinline__

// Programmatic dependent launch. The streaming elementwise and reduction
// kernels are launched with launch_pdl, which lets the GPU start launching
// the next kernel of the stream while this one finishes, and each such
// kernel begins with pdl_enter: it lets its own dependents launch once all
// of its CTAs have started, then waits until the kernel before it in the
// stream has completed and its writes are visible. No global memory is
// touched before that wait, so stream order holds exactly as without it;
// what is saved is the launch latency between back-to-back kernels. After a
// kernel launched the ordinary way the wait returns at once.
MPB_D void pdl_enter() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

template <class... KArgs, class... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
#ifdef MPB_NO_PDL
  cfg.numAttrs = 0;
#else
  cfg.numAttrs = 1;
#endif
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

namespace mpb {

// ---------------------------------------------------------------------------
// Complex storage: interleaved {re, im}, the muComplex / muDoubleComplex
// layout bound at rust/musapy-ops/src/kernels.rs:12.
// ---------------------------------------------------------------------------
struct __align__(8) c64 {
  float re, im;
};
struct __align__(16) c128 {
  double re, im;
};

// Boolean stored as a byte 0/1 but converted with bool semantics.
struct boolean {
  uint8_t v;
};

// dtype tag -> storage type
template <int D> struct Storage;
template <> struct Storage<MPB_BOOL> { using type = boolean; };
template <> struct Storage<MPB_I8> { using type = int8_t; };
template <> struct Storage<MPB_I16> { using type = int16_t; };
template <> struct Storage<MPB_I32> { using type = int32_t; };
template <> struct Storage<MPB_I64> { using type = int64_t; };
template <> struct Storage<MPB_U8> { using type = uint8_t; };
template <> struct Storage<MPB_U16> { using type = uint16_t; };
template <> struct Storage<MPB_U32> { using type = uint32_t; };
template <> struct Storage<MPB_U64> { using type = uint64_t; };
template <> struct Storage<MPB_F16> { using type = __half; };
template <> struct Storage<MPB_F32> { using type = float; };
template <> struct Storage<MPB_F64> { using type = double; };
template <> struct Storage<MPB_BF16> { using type = __nv_bfloat16; };
template <> struct Storage<MPB_C64> { using type = c64; };
template <> struct Storage<MPB_C128> { using type = c128; };


// ---------------------------------------------------------------------------
// Conversions. Semantics follow Rust `as` (the reference CPU path,
// rust/musapy-ops/src/op_builder.rs:2052-2097): float -> int truncates
// toward zero, saturates, and maps NaN to 0; int -> float rounds to nearest
// even; int -> int wraps. 16-bit floats round to nearest even.
// ---------------------------------------------------------------------------
template <class I>
MPB_D I float_to_int(double x) {
  // Saturating truncation with NaN -> 0 for any integer width.
  constexpr bool is_signed = (I)(-1) < (I)0;
  constexpr int bits = sizeof(I) * 8;
  if (x != x) return (I)0;
  if (is_signed) {
    const double half_range = (double)((uint64_t)1 << (bits - 1));  // 2^(bits-1), exact
    if (x <= -half_range) return (I)((uint64_t)1 << (bits - 1));    // INT_MIN bit pattern
    if (x >= half_range) return (I)(((uint64_t)1 << (bits - 1)) - 1);
    return (I)(int64_t)x;  // in range: truncation toward zero
  } else {
    const double range = (bits == 64) ? 18446744073709551616.0 : (double)((uint64_t)1 << (bits & 63));
    if (x <= 0.0) return (I)0;
    if (x >= range) return (I)(~(uint64_t)0);
    return (I)(uint64_t)x;
  }
}

template <class To> struct Cvt;

template <> struct Cvt<float> {
  MPB_D static float from(float x) { return x; }
  MPB_D static float from(double x) { return __double2float_rn(x); }
  MPB_D static float from(__half x) { return __half2float(x); }
  MPB_D static float from(__nv_bfloat16 x) { return __bfloat162float(x); }
  MPB_D static float from(int8_t x) { return (float)x; }
  MPB_D static float from(int16_t x) { return (float)x; }
  MPB_D static float from(int32_t x) { return __int2float_rn(x); }
  MPB_D static float from(int64_t x) { return __ll2float_rn(x); }
  MPB_D static float from(uint8_t x) { return (float)x; }
  MPB_D static float from(uint16_t x) { return (float)x; }
  MPB_D static float from(uint32_t x) { return __uint2float_rn(x); }
  MPB_D static float from(uint64_t x) { return __ull2float_rn(x); }
  MPB_D static float from(boolean x) { return x.v ? 1.0f : 0.0f; }
  // complex -> real is rejected by the host layer; defined for completeness.
  MPB_D static float from(c64 x) { return x.re; }
  MPB_D static float from(c128 x) { return __double2float_rn(x.re); }
};
template <> struct Cvt<double> {
  MPB_D static double from(float x) { return (double)x; }
  MPB_D static double from(double x) { return x; }
  MPB_D static double from(__half x) { return (double)__half2float(x); }
  MPB_D static double from(__nv_bfloat16 x) { return (double)__bfloat162float(x); }
  MPB_D static double from(int8_t x) { return (double)x; }
  MPB_D static double from(int16_t x) { return (double)x; }
  MPB_D static double from(int32_t x) { return (double)x; }
  MPB_D static double from(int64_t x) { return __ll2double_rn(x); }
  MPB_D static double from(uint8_t x) { return (double)x; }
  MPB_D static double from(uint16_t x) { return (double)x; }
  MPB_D static double from(uint32_t x) { return (double)x; }
  MPB_D static double from(uint64_t x) { return __ull2double_rn(x); }
  MPB_D static double from(boolean x) { return x.v ? 1.0 : 0.0; }
  MPB_D static double from(c64 x) { return (double)x.re; }
  MPB_D static double from(c128 x) { return x.re; }
};
template <> struct Cvt<__half> {
  MPB_D static __half from(float x) { return __float2half_rn(x); }
  MPB_D static __half from(double x) { return __double2half(x); }
  MPB_D static __half from(__half x) { return x; }
  MPB_D static __half from(__nv_bfloat16 x) { return __float2half_rn(__bfloat162float(x)); }
  template <class I> MPB_D static __half from(I x) { return __double2half(Cvt<double>::from(x)); }
};
template <> struct Cvt<__nv_bfloat16> {
  MPB_D static __nv_bfloat16 from(float x) { return __float2bfloat16_rn(x); }
  MPB_D static __nv_bfloat16 from(double x) { return __double2bfloat16(x); }
  MPB_D static __nv_bfloat16 from(__nv_bfloat16 x) { return x; }
  MPB_D static __nv_bfloat16 from(__half x) { return __float2bfloat16_rn(__half2float(x)); }
  template <class I> MPB_D static __nv_bfloat16 from(I x) { return __double2bfloat16(Cvt<double>::from(x)); }
};

// Integer targets.
template <class I> struct CvtInt {
  MPB_D static I from(float x) { return float_to_int<I>((double)x); }
  MPB_D static I from(double x) { return float_to_int<I>(x); }
  MPB_D static I from(__half x) { return float_to_int<I>((double)__half2float(x)); }
  MPB_D static I from(__nv_bfloat16 x) { return float_to_int<I>((double)__bfloat162float(x)); }
  MPB_D static I from(boolean x) { return (I)x.v; }
  // int -> int wraps (two's complement truncation / extension).
  MPB_D static I from(int8_t x) { return (I)x; }
  MPB_D static I from(int16_t x) { return (I)x; }
  MPB_D static I from(int32_t x) { return (I)x; }
  MPB_D static I from(int64_t x) { return (I)x; }
  MPB_D static I from(uint8_t x) { return (I)x; }
  MPB_D static I from(uint16_t x) { return (I)x; }
  MPB_D static I from(uint32_t x) { return (I)x; }
  MPB_D static I from(uint64_t x) { return (I)x; }
  MPB_D static I from(c64 x) { return float_to_int<I>((double)x.re); }
  MPB_D static I from(c128 x) { return float_to_int<I>(x.re); }
};
template <> struct Cvt<int8_t> : CvtInt<int8_t> {};
template <> struct Cvt<int16_t> : CvtInt<int16_t> {};
template <> struct Cvt<int32_t> : CvtInt<int32_t> {};
template <> struct Cvt<int64_t> : CvtInt<int64_t> {};
template <> struct Cvt<uint16_t> : CvtInt<uint16_t> {};
template <> struct Cvt<uint32_t> : CvtInt<uint32_t> {};
template <> struct Cvt<uint64_t> : CvtInt<uint64_t> {};
template <> struct Cvt<uint8_t> : CvtInt<uint8_t> {};

// Bool target: nonzero (NaN included) -> 1.
template <> struct Cvt<boolean> {
  MPB_D static boolean from(float x) { return boolean{(uint8_t)(x != 0.0f)}; }
  MPB_D static boolean from(double x) { return boolean{(uint8_t)(x != 0.0)}; }
  MPB_D static boolean from(__half x) { return boolean{(uint8_t)(__half2float(x) != 0.0f)}; }
  MPB_D static boolean from(__nv_bfloat16 x) { return boolean{(uint8_t)(__bfloat162float(x) != 0.0f)}; }
  MPB_D static boolean from(boolean x) { return x; }
  MPB_D static boolean from(c64 x) { return boolean{(uint8_t)(x.re != 0.0f || x.im != 0.0f)}; }
  MPB_D static boolean from(c128 x) { return boolean{(uint8_t)(x.re != 0.0 || x.im != 0.0)}; }
  template <class I> MPB_D static boolean from(I x) { return boolean{(uint8_t)(x != 0)}; }
};

// Complex targets (real -> complex: re = x, im = 0; c64 <-> c128 per part).
template <> struct Cvt<c64> {
  MPB_D static c64 from(c64 x) { return x; }
  MPB_D static c64 from(c128 x) { return c64{__double2float_rn(x.re), __double2float_rn(x.im)}; }
  template <class R> MPB_D static c64 from(R x) { return c64{Cvt<float>::from(x), 0.0f}; }
};
template <> struct Cvt<c128> {
  MPB_D static c128 from(c128 x) { return x; }
  MPB_D static c128 from(c64 x) { return c128{(double)x.re, (double)x.im}; }
  template <class R> MPB_D static c128 from(R x) { return c128{Cvt<double>::from(x), 0.0}; }
};

template <class To, class From>
MPB_D To cvt(From x) {
  return Cvt<To>::from(x);
}

// ---------------------------------------------------------------------------
// Division by an invariant 32-bit divisor: q = (umulhi(n, m) + n) >> s,
// evaluated in 64 bits so that the sum cannot overflow. Method of
// Granlund & Montgomery, "Division by Invariant Integers using
// Multiplication" (PLDI 1994), round-up variant; exact for every n < 2^32.
// ---------------------------------------------------------------------------
struct FastDiv {
  uint32_t d;
  uint32_t m;
  uint32_t s;
  MPB_HD FastDiv() : d(1), m(0), s(0) {}
  MPB_HD explicit FastDiv(uint32_t div) : d(div), m(0), s(0) {
    if (div > 1) {
      uint32_t l = 0;
      while (((uint64_t)1 << l) < div) ++l;
      m = (uint32_t)((((uint64_t)1 << 32) * (((uint64_t)1 << l) - div)) / div + 1);
      s = l;
    }
  }
  MPB_D uint32_t div(uint32_t n) const {
    if (d == 1) return n;
    uint32_t t = __umulhi(n, m);
    return (uint32_t)(((uint64_t)t + n) >> s);
  }
  MPB_D void divmod(uint32_t n, uint32_t& q, uint32_t& r) const {
    q = div(n);
    r = n - q * d;
  }
};

// ---------------------------------------------------------------------------
// Memory access. `ldg` uses the read-only path; `ld_stream` adds the
// evict-first hint for data read exactly once (inputs larger than L2).
// ---------------------------------------------------------------------------
template <class T>
MPB_D T ldg(const T* p) {
  return *p;
}

MPB_D uint4 ld_stream16(const void* p) {
  uint4 r;
  asm volatile("ld.global.cs.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
MPB_D uint4 ld_nc16(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
MPB_D void st_stream16(void* p, uint4 v) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}

}  // namespace mpb
