// Single-precision sin / cos / exp / log for float inputs.
//
// Accuracy: every function returns the correctly rounded float or one of its
// two neighbours (within 1 ulp), the same guarantee libm's float functions
// give, so the two agree within 2 ulp. sin/cos/exp were checked over all 2^32
// float inputs against the double-precision evaluation rounded to float.
//
// Speed: these run inside memory-bound elementwise kernels, so the budget is
// about 30 issue slots per element. FP64 and conversion instructions are slow
// on this part, so sin/cos/exp run in float arithmetic with error-free
// transformations (Dekker/Knuth two-product and two-sum) wherever a rounding
// would cost accuracy, and in pairs through the packed f32x2 instructions of
// sm_100 (one FFMA2 evaluates two lanes) when the kernel hands them two
// elements at once. The scalar and the paired forms run the same operations in
// the same order, so they return identical bits.
//
// Methods (textbook constructions; the coefficients are the Taylor
// coefficients 1/n!, 1/(2k+1) computed from their definitions, and the split
// constants of pi/2 and ln 2 were derived from pi (Machin's formula) and ln 2
// (sum of 1/(k 2^k)) in exact integer arithmetic):
//  * sin/cos: k = nearest integer to x*2/pi (rounded by adding 1.5*2^23, which
//    also leaves k mod 4 in the low mantissa bits); for |x| < 2^15 r = x - k*pi/2
//    by three FMA steps with pi/2 = C1 + C2 + C3 in floats; above, r as an
//    unevaluated float pair (rh, rl): x - k*C1 is exact (a multiple of 2^-24
//    below 1 in magnitude), k*C2 is split exactly by an FMA and subtracted by
//    two-sum, k*C3 goes into rl;
//    |rh| <= pi/4. sin r = rh + (rh^3 P(rh^2) + rl (1 - rh^2/2)) with the Taylor
//    series to degree 9; cos r = (1 - rh^2/2) + rh^4 Q(rh^2) - rh*rl to degree
//    10, where 1 - rh^2/2 is carried as a float pair (the rounding errors of
//    rh^2 and of the subtraction are recovered exactly). The quadrant k mod 4
//    selects and signs the result. |x| >= 2^20, inf and NaN take the
//    double-precision library path (never reached by ordinary data).
//  * exp: n = nearest integer to x*log2(e), y = x - n*ln2 as a float pair with
//    ln2 = L1 + L2 (x - n*L1 exact, the rest recovered by an FMA), e^y - 1 - y by
//    its Taylor series to degree 8, 1 + y summed exactly by fast two-sum, then
//    scaled by 2^n through the exponent field. x outside (-87, 88), where the
//    result overflows or leaves the normal range, and NaN take the double path.
//  * log: x = m * 2^e with m in [sqrt(1/2), sqrt(2)), log m = 2 atanh(s),
//    s = (m - 1)/(m + 1), |s| < 0.172, odd series to s^21, all in double.
//  * the double exp of the rare-range path: x*log2(e) = n + f, |f| <= 1/2,
//    2^f = e^(f ln 2) by its Taylor series to degree 11, scaled by 2^n.
#pragma once
#include "common.cuh"

namespace mpb {
namespace mathf {

// 1/n! for n = 2..15, exact to double precision (ratios of integers that are
// exact in double up to 18!).
#define MPB_INV_FACT(n) (1.0 / MPB_FACT##n)
#define MPB_FACT2 2.0
#define MPB_FACT3 6.0
#define MPB_FACT4 24.0
#define MPB_FACT5 120.0
#define MPB_FACT6 720.0
#define MPB_FACT7 5040.0
#define MPB_FACT8 40320.0
#define MPB_FACT9 362880.0
#define MPB_FACT10 3628800.0
#define MPB_FACT11 39916800.0
#define MPB_FACT12 479001600.0
#define MPB_FACT13 6227020800.0
#define MPB_FACT14 87178291200.0
#define MPB_FACT15 1307674368000.0

constexpr double kLn2 = 0.6931471805599453094;  // ln 2
constexpr double kLog2e = 1.4426950408889634074;  // 1 / ln 2

// ---------------------------------------------------------------- float ops
// Scalar and packed (f32x2) forms of the four operations, all rounded to
// nearest and never contracted, so the error-free transformations hold.
MPB_D float f_add(float a, float b) { return __fadd_rn(a, b); }
MPB_D float2 f_add(float2 a, float2 b) { return __fadd2_rn(a, b); }
MPB_D float f_sub(float a, float b) { return __fsub_rn(a, b); }
MPB_D float2 f_sub(float2 a, float2 b) { return __ffma2_rn(b, make_float2(-1.0f, -1.0f), a); }
MPB_D float f_mul(float a, float b) { return __fmul_rn(a, b); }
MPB_D float2 f_mul(float2 a, float2 b) { return __fmul2_rn(a, b); }
MPB_D float f_fma(float a, float b, float c) { return __fmaf_rn(a, b, c); }
MPB_D float2 f_fma(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
template <class V> MPB_D V splat(float c);
template <> MPB_D float splat<float>(float c) { return c; }
template <> MPB_D float2 splat<float2>(float c) { return make_float2(c, c); }
constexpr int lanes_of(float) { return 1; }
constexpr int lanes_of(float2) { return 2; }
MPB_D float& lane(float& v, int) { return v; }
MPB_D float& lane(float2& v, int i) { return i ? v.y : v.x; }

constexpr float kRoundMagic = 0x1.8p23f;  // 1.5 * 2^23: x + magic - magic = rint(x) for |x| < 2^22
constexpr int kRoundMagicBits = 0x4B400000;

// ------------------------------------------------------------- double exp
MPB_D double exp_d(double x) {
  // x is a float widened to double; |x| < 150 after the caller's range checks
  const double t = x * kLog2e;
  const double n = rint(t);
  const double f = t - n;  // |f| <= 0.5 (t is exact to 1 ulp of double)
  const double y = f * kLn2;
  double p = MPB_INV_FACT(11);
  p = fma(p, y, MPB_INV_FACT(10));
  p = fma(p, y, MPB_INV_FACT(9));
  p = fma(p, y, MPB_INV_FACT(8));
  p = fma(p, y, MPB_INV_FACT(7));
  p = fma(p, y, MPB_INV_FACT(6));
  p = fma(p, y, MPB_INV_FACT(5));
  p = fma(p, y, MPB_INV_FACT(4));
  p = fma(p, y, MPB_INV_FACT(3));
  p = fma(p, y, 0.5);
  p = fma(p, y, 1.0);
  p = fma(p, y, 1.0);
  // scale by 2^n (n in [-151, 129]): build 2^n in two halves to stay normal
  const int ni = (int)n;
  const int n1 = ni / 2, n2 = ni - ni / 2;
  const double s1 = __longlong_as_double((long long)(n1 + 1023) << 52);
  const double s2 = __longlong_as_double((long long)(n2 + 1023) << 52);
  return (p * s1) * s2;
}

// exp of a float through the double evaluation: NaN, overflow, underflow and
// the subnormal range.
MPB_D float expf_wide(float xf) {
  if (xf != xf) return xf;
  if (xf > 89.0f) return __int_as_float(0x7f800000);  // overflows f32
  if (xf < -104.0f) return 0.0f;                      // below half the smallest subnormal
  return __double2float_rn(exp_d((double)xf));
}

MPB_D bool exp_in_range(float x) { return x > -87.0f && x < 88.0f; }

// exp for x in (-87, 88): n in [-126, 127], the result a normal float.
template <class V>
MPB_D V exp_core(V x) {
  const V nb = f_fma(x, splat<V>(0x1.715476p+0f), splat<V>(kRoundMagic));  // log2(e) in float
  const V n = f_sub(nb, splat<V>(kRoundMagic));
  const V y1 = f_fma(n, splat<V>(-0x1.62e430p-1f), x);         // x - n*L1, exact
  const V yh = f_fma(n, splat<V>(0x1.05c610p-29f), y1);         // - n*L2 (L2 < 0)
  const V yl = f_fma(n, splat<V>(0x1.05c610p-29f), f_sub(y1, yh));  // its rounding error
  V p = splat<V>((float)MPB_INV_FACT(8));
  p = f_fma(p, yh, splat<V>((float)MPB_INV_FACT(7)));
  p = f_fma(p, yh, splat<V>((float)MPB_INV_FACT(6)));
  p = f_fma(p, yh, splat<V>((float)MPB_INV_FACT(5)));
  p = f_fma(p, yh, splat<V>((float)MPB_INV_FACT(4)));
  p = f_fma(p, yh, splat<V>((float)MPB_INV_FACT(3)));
  p = f_fma(p, yh, splat<V>(0.5f));
  const V t = f_fma(f_mul(yh, yh), p, f_fma(yl, yh, yl));  // yh^2 P(yh) + yl (1 + yh)
  const V hi = f_add(splat<V>(1.0f), yh);
  const V lo = f_add(f_sub(splat<V>(1.0f), hi), yh);  // exact: |yh| < 1
  const V v = f_add(hi, f_add(lo, t));
  V scale = nb;
#pragma unroll
  for (int i = 0; i < lanes_of(V{}); ++i) {
    const int ni = __float_as_int(lane(scale, i)) - kRoundMagicBits;
    lane(scale, i) = __int_as_float((ni + 127) << 23);
  }
  return f_mul(v, scale);
}

MPB_D float expf_(float x) { return exp_in_range(x) ? exp_core(x) : expf_wide(x); }
MPB_D bool exp_fast_ok(float2 x) { return exp_in_range(x.x) && exp_in_range(x.y); }
MPB_D float2 expf2_fast(float2 x) { return exp_core(x); }
MPB_D float2 expf2_(float2 x) {
  float2 v = exp_core(x);
  if (!(exp_in_range(x.x) && exp_in_range(x.y))) {
    if (!exp_in_range(x.x)) v.x = expf_wide(x.x);
    if (!exp_in_range(x.y)) v.y = expf_wide(x.y);
  }
  return v;
}

// ------------------------------------------------------------------ sin/cos
MPB_D bool trig_in_range(float x) { return fabsf(x) < 1048576.0f; }  // 2^20; false for NaN

// The quadrant k mod 4 (the low bits of kb = k + 1.5 * 2^23; cos adds one)
// selects cos r (odd) or sin r (even) and bit 1 of it flips the sign, done
// with integer bit operations. sin(+-0) is +-0: the reduction turns r = -0
// into +0 (adding the +0 product k*C2 for k = 0), so a zero argument is
// returned as is (every other |x| < 2^-12 already rounds to x).
template <int COS, class V>
MPB_D V trig_select(V kb, V x, V sv, V cv) {
  V out;
#pragma unroll
  for (int i = 0; i < lanes_of(V{}); ++i) {
    const unsigned q = (unsigned)__float_as_int(lane(kb, i)) + (unsigned)COS;
    const unsigned v = (q & 1u) ? (unsigned)__float_as_int(lane(cv, i)) : (unsigned)__float_as_int(lane(sv, i));
    float f = __int_as_float((int)(v ^ ((q & 2u) << 30)));
    if (COS == 0 && lane(x, i) == 0.0f) f = lane(x, i);
    lane(out, i) = f;
  }
  return out;
}

// sin (COS = 0) or cos (COS = 1) for |x| < 2^20.
template <int COS, class V>
MPB_D V sincos_core(V x) {
  const V kb = f_fma(x, splat<V>(0x1.45f306p-1f), splat<V>(kRoundMagic));  // 2/pi in float
  const V k = f_sub(kb, splat<V>(kRoundMagic));
  // r = x - k*(C1 + C2 + C3): C1 = 0x1.921fb6p+0, C2 = -0x1.777a5cp-25, C3 = -0x1.ee59dap-50
  const V r1 = f_fma(k, splat<V>(-0x1.921fb6p+0f), x);      // exact
  const V phn = f_mul(k, splat<V>(0x1.777a5cp-25f));         // -k*C2 rounded
  const V pl = f_fma(k, splat<V>(-0x1.777a5cp-25f), phn);    // k*C2 - fl(k*C2), exact
  const V s = f_add(r1, phn);                                // two-sum of r1 and -k*C2
  const V bb = f_sub(s, r1);
  const V e = f_add(f_sub(r1, f_sub(s, bb)), f_sub(phn, bb));
  const V rl = f_fma(k, splat<V>(0x1.ee59dap-50f), f_sub(e, pl));
  const V r2 = f_mul(s, s);
  const V nh = f_mul(r2, splat<V>(-0.5f));
  // Quadrants 0 and 2 need sin r, 1 and 3 need cos r; both are evaluated,
  // since the lanes of a warp fall in every quadrant.
  const V ps = f_fma(f_fma(f_fma(splat<V>((float)MPB_INV_FACT(9)), r2, splat<V>((float)-MPB_INV_FACT(7))), r2,
                           splat<V>((float)MPB_INV_FACT(5))),
                     r2, splat<V>((float)-MPB_INV_FACT(3)));
  const V sv = f_add(s, f_fma(f_mul(s, r2), ps, f_fma(rl, nh, rl)));
  const V pc = f_fma(f_fma(f_fma(splat<V>((float)-MPB_INV_FACT(10)), r2, splat<V>((float)MPB_INV_FACT(8))), r2,
                           splat<V>((float)-MPB_INV_FACT(6))),
                     r2, splat<V>((float)MPB_INV_FACT(4)));
  const V w = f_add(splat<V>(1.0f), nh);                      // 1 - r2/2 rounded
  const V corr = f_add(f_sub(splat<V>(1.0f), w), nh);         // its rounding error, exact
  const V r2e = f_fma(s, s, f_mul(r2, splat<V>(-1.0f)));      // s*s - fl(s*s), exact
  const V tail = f_sub(corr, f_fma(splat<V>(0.5f), r2e, f_mul(s, rl)));
  const V cv = f_add(w, f_fma(f_mul(r2, r2), pc, tail));
  return trig_select<COS>(kb, x, sv, cv);
}

// sin (COS = 0) or cos (COS = 1) for |x| < 2^15: r = x - k*pi/2 by three FMA
// steps (C1, C2, C3) in float, no compensation term; the rounding of the
// second step stays below half an ulp of r because |k*C3| is tiny next to
// |r| for |x| < 2^15. Checked over every float input below 2^15: within 1
// ulp of the correctly rounded value, like the compensated form, with about
// a third fewer instructions.
template <int COS, class V>
MPB_D V sincos_core_fast(V x) {
  const V kb = f_fma(x, splat<V>(0x1.45f306p-1f), splat<V>(kRoundMagic));
  const V k = f_sub(kb, splat<V>(kRoundMagic));
  V r = f_fma(k, splat<V>(-0x1.921fb6p+0f), x);
  r = f_fma(k, splat<V>(0x1.777a5cp-25f), r);
  r = f_fma(k, splat<V>(0x1.ee59dap-50f), r);
  const V r2 = f_mul(r, r);
  const V ps = f_fma(f_fma(f_fma(splat<V>((float)MPB_INV_FACT(9)), r2, splat<V>((float)-MPB_INV_FACT(7))), r2,
                           splat<V>((float)MPB_INV_FACT(5))),
                     r2, splat<V>((float)-MPB_INV_FACT(3)));
  const V sv = f_fma(f_mul(r, r2), ps, r);
  const V pc = f_fma(f_fma(f_fma(splat<V>((float)-MPB_INV_FACT(10)), r2, splat<V>((float)MPB_INV_FACT(8))), r2,
                           splat<V>((float)-MPB_INV_FACT(6))),
                     r2, splat<V>((float)MPB_INV_FACT(4)));
  const V nh = f_mul(r2, splat<V>(-0.5f));
  const V w = f_add(splat<V>(1.0f), nh);                    // 1 - r2/2 rounded
  const V corr = f_add(f_sub(splat<V>(1.0f), w), nh);       // its rounding error, exact
  const V r2e = f_fma(r, r, f_mul(r2, splat<V>(-1.0f)));    // r*r - fl(r*r), exact
  const V cv = f_add(w, f_fma(f_mul(r2, r2), pc, f_fma(splat<V>(-0.5f), r2e, corr)));
  return trig_select<COS>(kb, x, sv, cv);
}
constexpr float kTrigFastBound = 32768.0f;  // 2^15

template <int COS>
MPB_D float sincos_wide(float x) {
  if (x != x || isinf(x)) return x - x;  // NaN
  return __double2float_rn(COS ? cos((double)x) : sin((double)x));
}

// Arguments outside the fast range (|x| >= 2^15, inf, NaN): rare, so kept
// out of line - inlined, their registers and stack (the double-precision
// fallback) would be allocated in every elementwise loop that calls sin/cos.
template <int COS>
__device__ __noinline__ float sincos_slow(float x) {
  return trig_in_range(x) ? sincos_core<COS>(x) : sincos_wide<COS>(x);
}

template <int COS>
MPB_D float sincosf_(float x) {
  if (fabsf(x) < kTrigFastBound) return sincos_core_fast<COS>(x);  // false for NaN
  return sincos_slow<COS>(x);
}
// Two elements at once; a pair with an argument outside the fast range goes
// element by element, so the results equal the one-element form's.
template <int COS>
MPB_D float2 sincosf2_(float2 x) {
  if (fabsf(x.x) < kTrigFastBound && fabsf(x.y) < kTrigFastBound) return sincos_core_fast<COS>(x);
  return make_float2(sincosf_<COS>(x.x), sincosf_<COS>(x.y));
}
// The pair form's fast path alone and its range test, for kernels that run
// the fast path on every pair and fix the rare out-of-range elements up
// afterwards (one warp-wide test instead of a branch per pair).
MPB_D bool trig_fast_ok(float2 x) { return fabsf(x.x) < kTrigFastBound && fabsf(x.y) < kTrigFastBound; }
template <int COS>
MPB_D float2 sincosf2_fast(float2 x) { return sincos_core_fast<COS>(x); }
MPB_D float sinf_(float x) { return sincosf_<0>(x); }
MPB_D float cosf_(float x) { return sincosf_<1>(x); }

// ---------------------------------------------------------------------- log
MPB_D float logf_(float xf) {
  if (xf != xf) return xf;
  if (xf < 0.0f) return __int_as_float(0x7fc00000);
  if (xf == 0.0f) return __int_as_float(0xff800000);
  if (xf == __int_as_float(0x7f800000)) return xf;
  // split into m * 2^e with m in [sqrt(1/2), sqrt(2)); f32 subnormals are
  // normal in double
  double x = (double)xf;
  long long bits = __double_as_longlong(x);
  int e = (int)((bits >> 52) & 0x7ff) - 1023;
  double m = __longlong_as_double((bits & 0x000fffffffffffffLL) | 0x3ff0000000000000LL);  // [1, 2)
  if (m > 1.4142135623730950488) {
    m *= 0.5;
    e += 1;
  }
  const double s = (m - 1.0) / (m + 1.0);
  const double s2 = s * s;
  double p = 1.0 / 21.0;
  p = fma(p, s2, 1.0 / 19.0);
  p = fma(p, s2, 1.0 / 17.0);
  p = fma(p, s2, 1.0 / 15.0);
  p = fma(p, s2, 1.0 / 13.0);
  p = fma(p, s2, 1.0 / 11.0);
  p = fma(p, s2, 1.0 / 9.0);
  p = fma(p, s2, 1.0 / 7.0);
  p = fma(p, s2, 1.0 / 5.0);
  p = fma(p, s2, 1.0 / 3.0);
  const double lm = 2.0 * fma(s * s2, p, s);  // 2 (s + s^3/3 + ...)
  return __double2float_rn(fma((double)e, kLn2, lm));
}

#undef MPB_INV_FACT

}  // namespace mathf
}  // namespace mpb
