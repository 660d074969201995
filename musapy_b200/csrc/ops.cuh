// Elementwise operator functors.
//
// Numerics follow the reference CPU path (the parity oracle):
//  * f32/f64 add/sub/mul/div are single IEEE operations
//    (rust/musapy-ops/src/op_builder.rs:1618-1627);
//  * complex64 arithmetic is evaluated in f64 and narrowed once, exactly as
//    cpu_binary_cplx (op_builder.rs:1689-1731) does; every f64 step uses an
//    explicitly rounded intrinsic so no FMA contraction can change a bit;
//  * f32 transcendentals are evaluated in f64 and rounded once, which keeps
//    them within 1 ulp of the correctly rounded value (libm's sinf/expf/... are
//    within 1 ulp too, so the two agree within 2 ulp);
//  * f16/bf16 arithmetic runs in f32 and rounds once (f32 carries >= 2p+2 bits
//    of either format, so +,-,*,/ are correctly rounded);
//  * sign(NaN) = sign(+-0) = +0 and clamp lets NaN through, as the CPU loops do
//    (op_builder.rs:1878-1886, :2035-2043).
#pragma once
#include "common.cuh"

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
  MPB_D float operator()(float a, float b) const {
    return __double2float_rn(pow((double)a, (double)b));
  }
  MPB_D double operator()(double a, double b) const { return pow(a, b); }
};
struct OpPowLow {
  MPB_D float operator()(float a, float b) const { return powf(a, b); }
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
struct OpSin {
  MPB_D float operator()(float a) const { return __double2float_rn(sin((double)a)); }
  MPB_D double operator()(double a) const { return sin(a); }
};
struct OpCos {
  MPB_D float operator()(float a) const { return __double2float_rn(cos((double)a)); }
  MPB_D double operator()(double a) const { return cos(a); }
};
struct OpExp {
  MPB_D float operator()(float a) const { return __double2float_rn(exp((double)a)); }
  MPB_D double operator()(double a) const { return exp(a); }
};
struct OpLog {
  MPB_D float operator()(float a) const { return __double2float_rn(log((double)a)); }
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
