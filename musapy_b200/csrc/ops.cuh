// Elementwise operator functors.
//
// Numerics follow the reference CPU path (the parity oracle):
//  * f32/f64 add/sub/mul/div are single IEEE operations
//    (rust/musapy-ops/src/op_builder.rs:1618-1627);
//  * complex64 arithmetic is evaluated in f64 and narrowed once, exactly as
//    cpu_binary_cplx (op_builder.rs:1689-1731) does; every f64 step uses an
//    explicitly rounded intrinsic so no FMA contraction can change a bit;
//  * f32 sin/cos/exp/log are within 1 ulp of the correctly rounded value
//    (mathf.cuh); libm's sinf/expf/... are within 1 ulp too, so the two agree
//    within 2 ulp. sin/cos/exp also take two elements at once (`pair`, packed
//    f32x2 arithmetic) with results identical to the one-element form;
//  * f16/bf16 arithmetic runs in f32 and rounds once (f32 carries >= 2p+2 bits
//    of either format, so +,-,*,/ are correctly rounded);
//  * sign(NaN) = sign(+-0) = +0 and clamp lets NaN through, as the CPU loops do
//    (op_builder.rs:1878-1886, :2035-2043).
#pragma once
#include "common.cuh"
#include "mathf.cuh"

namespace mpb {

// ----------------------------------------------------------------- binary
struct OpAdd {
  MPB_D float operator()(float a, float b) const { return __fadd_rn(a, b); }
  MPB_D double operator()(double a, double b) const { return __dadd_rn(a, b); }
  MPB_D c64 operator()(c64 a, c64 b) const {
    // (double)a + (double)b rounded to f32 equals the f32 sum (innocuous double rounding).
    return c64{__fadd_rn(a.re, b.re), __fadd_rn(a.im, b.im)};
  }
  MPB_D c128 operator()(c128 a, c128 b) const {
    return c128{__dadd_rn(a.re, b.re), __dadd_rn(a.im, b.im)};
  }
};
struct OpSub {
  MPB_D float operator()(float a, float b) const { return __fsub_rn(a, b); }
  MPB_D double operator()(double a, double b) const { return __dsub_rn(a, b); }
  MPB_D c64 operator()(c64 a, c64 b) const {
    return c64{__fsub_rn(a.re, b.re), __fsub_rn(a.im, b.im)};
  }
  MPB_D c128 operator()(c128 a, c128 b) const {
    return c128{__dsub_rn(a.re, b.re), __dsub_rn(a.im, b.im)};
  }
};
struct OpMul {
  MPB_D float operator()(float a, float b) const { return __fmul_rn(a, b); }
  MPB_D double operator()(double a, double b) const { return __dmul_rn(a, b); }
  MPB_D c128 operator()(c128 a, c128 b) const {
    double re = __dsub_rn(__dmul_rn(a.re, b.re), __dmul_rn(a.im, b.im));
    double im = __dadd_rn(__dmul_rn(a.re, b.im), __dmul_rn(a.im, b.re));
    return c128{re, im};
  }
  MPB_D c64 operator()(c64 a, c64 b) const {
    c128 r = (*this)(c128{a.re, a.im}, c128{b.re, b.im});
    return c64{__double2float_rn(r.re), __double2float_rn(r.im)};
  }
};
struct OpDiv {
  MPB_D float operator()(float a, float b) const { return __fdiv_rn(a, b); }
  MPB_D double operator()(double a, double b) const { return __ddiv_rn(a, b); }
  MPB_D c128 operator()(c128 a, c128 b) const {
    double den = __dadd_rn(__dmul_rn(b.re, b.re), __dmul_rn(b.im, b.im));
    double nr = __dadd_rn(__dmul_rn(a.re, b.re), __dmul_rn(a.im, b.im));
    double ni = __dsub_rn(__dmul_rn(a.im, b.re), __dmul_rn(a.re, b.im));
    return c128{__ddiv_rn(nr, den), __ddiv_rn(ni, den)};
  }
  MPB_D c64 operator()(c64 a, c64 b) const {
    c128 r = (*this)(c128{a.re, a.im}, c128{b.re, b.im});
    return c64{__double2float_rn(r.re), __double2float_rn(r.im)};
  }
};
// pow: the f32 instance (used for f32 outputs) goes through f64; the
// 16-bit formats compute in f32 (tag OpPowLow) because one f32 rounding is
// already far below their half-ulp.
struct OpPow {
  static constexpr bool kHeavy = true;
  MPB_D float operator()(float a, float b) const {
    return __double2float_rn(pow((double)a, (double)b));
  }
  MPB_D double operator()(double a, double b) const { return pow(a, b); }
};
// 16-bit pow: 2^(b log2 a) through the SFU (lg2.approx / ex2.approx) when a
// is positive and finite, |b| < 64 and |b log2 a| < 24. The absolute error of
// lg2.approx is about 2^-22, so t = b log2 a is off by at most 2^-16 and 2^t by
// about 1e-5 relative, far under half an f16 ulp (2^-11): one more rounding to
// 16 bits gives the correctly rounded value or a neighbour (checked over all
// 2^32 f16 pairs: within 1 ulp of the correctly rounded value, and within 1 ulp
// of pow evaluated in f32). Everything else (a <= 0, inf, NaN, large |b|,
// results outside the f16 range) goes through powf.
struct OpPowLow {
  static constexpr bool kHeavy = true;
  MPB_D static float lg2_approx(float x) {
    float y;
    asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
  }
  MPB_D static float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
  }
  MPB_D float operator()(float a, float b) const {
    // a subnormal a (possible from bf16) is flushed to 0 by lg2.approx.ftz,
    // which makes t infinite or NaN and sends it to powf
    const float t = b * lg2_approx(a);
    if (a > 0.0f && a < __int_as_float(0x7f800000) && fabsf(b) < 64.0f && fabsf(t) < 24.0f) return ex2_approx(t);
    return powf(a, b);
  }
};

// ------------------------------------------------------------- comparisons
#define MPB_CMP(NAME, EXPR)                                                            \
  struct NAME {                                                                        \
    template <class T> MPB_D boolean operator()(T a, T b) const {                      \
      return boolean{(uint8_t)(EXPR)};                                                 \
    }                                                                                  \
  };
MPB_CMP(OpEq, a == b)
MPB_CMP(OpNe, a != b)
MPB_CMP(OpLt, a < b)
MPB_CMP(OpGt, a > b)
MPB_CMP(OpLe, a <= b)
MPB_CMP(OpGe, a >= b)
#undef MPB_CMP

// Complex equality compares both parts (op_builder.rs:1776-1781).
struct OpEqC {
  MPB_D boolean operator()(c64 a, c64 b) const { return boolean{(uint8_t)(a.re == b.re && a.im == b.im)}; }
  MPB_D boolean operator()(c128 a, c128 b) const { return boolean{(uint8_t)(a.re == b.re && a.im == b.im)}; }
};
struct OpNeC {
  MPB_D boolean operator()(c64 a, c64 b) const { return boolean{(uint8_t)(a.re != b.re || a.im != b.im)}; }
  MPB_D boolean operator()(c128 a, c128 b) const { return boolean{(uint8_t)(a.re != b.re || a.im != b.im)}; }
};

// ------------------------------------------------------------------- unary
// Paired ops also expose their fast path (`pair_fast`, no range branch) and
// its range test (`pair_ok`); out-of-range pairs go through `pair`, whose
// results are the same as the one-element form's.
struct OpSin {
  static constexpr bool kPaired = true;
  MPB_D float operator()(float a) const { return mathf::sinf_(a); }
  MPB_D float2 pair(float2 a) const { return mathf::sincosf2_<0>(a); }
  MPB_D float2 pair_fast(float2 a) const { return mathf::sincosf2_fast<0>(a); }
  MPB_D bool pair_ok(float2 a) const { return mathf::trig_fast_ok(a); }
  MPB_D double operator()(double a) const { return sin(a); }
};
struct OpCos {
  static constexpr bool kPaired = true;
  MPB_D float operator()(float a) const { return mathf::cosf_(a); }
  MPB_D float2 pair(float2 a) const { return mathf::sincosf2_<1>(a); }
  MPB_D float2 pair_fast(float2 a) const { return mathf::sincosf2_fast<1>(a); }
  MPB_D bool pair_ok(float2 a) const { return mathf::trig_fast_ok(a); }
  MPB_D double operator()(double a) const { return cos(a); }
};
struct OpExp {
  static constexpr bool kPaired = true;
  MPB_D float operator()(float a) const { return mathf::expf_(a); }
  MPB_D float2 pair(float2 a) const { return mathf::expf2_(a); }
  MPB_D float2 pair_fast(float2 a) const { return mathf::expf2_fast(a); }
  MPB_D bool pair_ok(float2 a) const { return mathf::exp_fast_ok(a); }
  MPB_D double operator()(double a) const { return exp(a); }
};
struct OpLog {
  static constexpr bool kHeavy = true;
  MPB_D float operator()(float a) const { return mathf::logf_(a); }
  MPB_D double operator()(double a) const { return log(a); }
};
struct OpAbs {
  MPB_D float operator()(float a) const { return fabsf(a); }
  MPB_D double operator()(double a) const { return fabs(a); }
  // |z| = sqrt(re^2 + im^2) in f64, narrowed once (op_builder.rs:1924-1948).
  MPB_D double operator()(c128 a) const {
    return __dsqrt_rn(__dadd_rn(__dmul_rn(a.re, a.re), __dmul_rn(a.im, a.im)));
  }
  MPB_D float operator()(c64 a) const {
    double re = a.re, im = a.im;
    return __double2float_rn(__dsqrt_rn(__dadd_rn(__dmul_rn(re, re), __dmul_rn(im, im))));
  }
};
struct OpSign {
  MPB_D float operator()(float a) const { return a > 0.0f ? 1.0f : (a < 0.0f ? -1.0f : 0.0f); }
  MPB_D double operator()(double a) const { return a > 0.0 ? 1.0 : (a < 0.0 ? -1.0 : 0.0); }
};
struct OpNeg {
  MPB_D float operator()(float a) const { return -a; }
  MPB_D double operator()(double a) const { return -a; }
  MPB_D c64 operator()(c64 a) const { return c64{-a.re, -a.im}; }
  MPB_D c128 operator()(c128 a) const { return c128{-a.re, -a.im}; }
};
template <class T>
struct OpClamp {
  T lo, hi;
  MPB_D T operator()(T v) const { return v < lo ? lo : (v > hi ? hi : v); }
};
struct OpIdentity {
  template <class T> MPB_D T operator()(T a) const { return a; }
};

}  // namespace mpb
