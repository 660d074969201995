/*
 * TEST INFRASTRUCTURE ONLY - the parity oracle of musapy_b200.
 *
 * A plain-C restatement of the CPU path of musapy's operator layer
 * (rust/musapy-ops/src/op_builder.rs:1559-3688), which is the reference
 * behaviour the CUDA kernels must reproduce. Nothing in the product links,
 * imports or executes this file; tests/, __graft_entry__.smoke() and the
 * cpu_baseline / reference legs of bench.py use it as the checker.
 *
 * Build: see oracle/Makefile (gcc -O2 -ffp-contract=off -fno-fast-math, so
 * every float operation is evaluated exactly as written, like Rust without
 * FMA contraction). Transcendentals come from glibc's libm, which is what
 * Rust's f32::sin / f64::exp etc. call on Linux.
 *
 * Dtype codes are those of musapy's Dtype enum (rust/musapy-core/src/
 * dtype.rs:25-41): bool=0 i8 i16 i32 i64 u8 u16 u32 u64 f16=9 f32=10 f64=11
 * bf16=12 c64=13 c128=14.
 *
 * Beyond the reference (it rejects them): f16 / bf16 arithmetic is restated
 * as "compute in f64, round once to the 16-bit format (nearest-even)", and
 * integer comparisons compare the promoted integers.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

enum { BOOL = 0, I8, I16, I32, I64, U8, U16, U32, U64, F16, F32, F64, BF16, C64, C128 };
enum { ADD = 0, SUB, MUL, DIV, POW };
enum { EQ = 10, NE, LT, GT, LE, GE };
enum { SIN = 20, COS, EXP, LOG, ABS, SIGN, NEG };
enum { R_SUM = 0, R_PROD, R_MAX, R_MIN, R_MEAN, R_ARGMAX, R_ARGMIN };

typedef struct { float re, im; } c64_t;
typedef struct { double re, im; } c128_t;

static int g_threads = 1;
void or_set_threads(int n) { g_threads = n > 0 ? n : 1; }
int or_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* cpu_offset_nd (op_builder.rs:1581-1590): linear index -> element offset. */
static int64_t offset_nd(uint64_t idx, int ndim, const int64_t* shape, const int64_t* strides) {
  int64_t off = 0;
  for (int i = ndim - 1; i >= 0; --i) {
    uint64_t c = idx % (uint64_t)shape[i];
    idx /= (uint64_t)shape[i];
    off += (int64_t)c * strides[i];
  }
  return off;
}

static uint64_t numel(int ndim, const int64_t* shape) {
  uint64_t n = 1;
  for (int i = 0; i < ndim; ++i) n *= (uint64_t)shape[i];
  return n;
}

/* ------------------------------------------------------------------------ */
/* 16-bit float formats: exact decode, round-to-nearest-even encode.        */
/* ------------------------------------------------------------------------ */
static double f16_to_double(uint16_t h) {
  int s = h >> 15, e = (h >> 10) & 31, m = h & 1023;
  double v;
  if (e == 0) v = ldexp((double)m, -24);
  else if (e == 31) v = m ? NAN : INFINITY;
  else v = ldexp((double)(m | 1024), e - 25);
  return s ? -v : v;
}
static double bf16_to_double(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return (double)f;
}
/* Round x to a binary format with p significand bits and minimum normal
 * exponent emin (value range [2^emin, 2^(emax+1))), nearest-even, and encode
 * with `ebits` exponent bits. The scaled significand is exact in double. */
static uint16_t encode16(double x, int p, int emin, int emax, int ebits) {
  uint16_t sign = signbit(x) ? (uint16_t)(1u << 15) : 0;
  const int mbits = p - 1;
  const uint16_t inf = (uint16_t)(((1u << ebits) - 1) << mbits);
  if (isnan(x)) return (uint16_t)(sign | inf | (1u << (mbits - 1)));
  double a = fabs(x);
  if (isinf(a)) return (uint16_t)(sign | inf);
  if (a == 0.0) return sign;
  int e;
  frexp(a, &e); /* a = f * 2^e, f in [0.5, 1): exponent of a is e-1 */
  int ex = e - 1;
  if (ex < emin) ex = emin; /* subnormal quantum */
  double q = ldexp(a, p - 1 - ex);  /* significand scaled to an integer range */
  double r = nearbyint(q);          /* round-half-even (default mode) */
  /* r may reach 2^p: renormalise */
  if (r >= ldexp(1.0, p)) {
    r = ldexp(r, -1);
    ex += 1;
  }
  if (ex > emax) return (uint16_t)(sign | inf);
  uint32_t sig = (uint32_t)r;
  if (sig < (1u << mbits)) return (uint16_t)(sign | sig); /* subnormal (ex == emin) */
  uint32_t biased = (uint32_t)(ex - emin + 1);
  return (uint16_t)(sign | (biased << mbits) | (sig & ((1u << mbits) - 1)));
}
static uint16_t double_to_f16(double x) { return encode16(x, 11, -14, 15, 5); }
static uint16_t double_to_bf16(double x) { return encode16(x, 8, -126, 127, 8); }
uint16_t or_double_to_f16(double x) { return double_to_f16(x); }
uint16_t or_double_to_bf16(double x) { return double_to_bf16(x); }
double or_f16_to_double(uint16_t h) { return f16_to_double(h); }
double or_bf16_to_double(uint16_t h) { return bf16_to_double(h); }

/* Load any real dtype as double (exact for every dtype but 64-bit ints). */
static double load_real(const void* p, int64_t off, int dt) {
  switch (dt) {
    case BOOL: return ((const uint8_t*)p)[off] ? 1.0 : 0.0;
    case I8: return ((const int8_t*)p)[off];
    case I16: return ((const int16_t*)p)[off];
    case I32: return ((const int32_t*)p)[off];
    case I64: return (double)((const int64_t*)p)[off];
    case U8: return ((const uint8_t*)p)[off];
    case U16: return ((const uint16_t*)p)[off];
    case U32: return ((const uint32_t*)p)[off];
    case U64: return (double)((const uint64_t*)p)[off];
    case F16: return f16_to_double(((const uint16_t*)p)[off]);
    case F32: return ((const float*)p)[off];
    case F64: return ((const double*)p)[off];
    case BF16: return bf16_to_double(((const uint16_t*)p)[off]);
    default: return 0.0;
  }
}

/* ------------------------------------------------------------------------ */
/* Binary arithmetic (cpu_binary_typed / cpu_binary_op, op_builder.rs:      */
/* 1618-1760) and complex (cpu_binary_cplx, :1689-1731: f64, then narrow). */
/* ------------------------------------------------------------------------ */
static float bin_f32(int op, float a, float b) {
  switch (op) {
    case ADD: return a + b;
    case SUB: return a - b;
    case MUL: return a * b;
    case DIV: return a / b;
    default: return powf(a, b);
  }
}
static double bin_f64(int op, double a, double b) {
  switch (op) {
    case ADD: return a + b;
    case SUB: return a - b;
    case MUL: return a * b;
    case DIV: return a / b;
    default: return pow(a, b);
  }
}
static void bin_cplx(int op, double ar, double ai, double br, double bi, double* re, double* im) {
  switch (op) {
    case ADD: *re = ar + br; *im = ai + bi; break;
    case SUB: *re = ar - br; *im = ai - bi; break;
    case MUL: *re = ar * br - ai * bi; *im = ar * bi + ai * br; break;
    default: {
      double den = br * br + bi * bi;
      *re = (ar * br + ai * bi) / den;
      *im = (ai * br - ar * bi) / den;
    }
  }
}

/* Operands are already in the compute dtype `dt` (musapy casts first). */
void or_binary(int op, int dt, const void* a, const void* b, void* c, int ndim, const int64_t* shape,
               const int64_t* as, const int64_t* bs) {
  const uint64_t n = numel(ndim, shape);
#pragma omp parallel for schedule(static) num_threads(g_threads) if (g_threads > 1)
  for (uint64_t i = 0; i < n; ++i) {
    const int64_t oa = offset_nd(i, ndim, shape, as), ob = offset_nd(i, ndim, shape, bs);
    switch (dt) {
      case F32: ((float*)c)[i] = bin_f32(op, ((const float*)a)[oa], ((const float*)b)[ob]); break;
      case F64: ((double*)c)[i] = bin_f64(op, ((const double*)a)[oa], ((const double*)b)[ob]); break;
      case F16:
      case BF16: {
        const double r = bin_f64(op, load_real(a, oa, dt), load_real(b, ob, dt));
        ((uint16_t*)c)[i] = dt == F16 ? double_to_f16(r) : double_to_bf16(r);
        break;
      }
      case C64: {
        const c64_t x = ((const c64_t*)a)[oa], y = ((const c64_t*)b)[ob];
        double re, im;
        bin_cplx(op, x.re, x.im, y.re, y.im, &re, &im);
        ((c64_t*)c)[i].re = (float)re;
        ((c64_t*)c)[i].im = (float)im;
        break;
      }
      case C128: {
        const c128_t x = ((const c128_t*)a)[oa], y = ((const c128_t*)b)[ob];
        double re, im;
        bin_cplx(op, x.re, x.im, y.re, y.im, &re, &im);
        ((c128_t*)c)[i].re = re;
        ((c128_t*)c)[i].im = im;
        break;
      }
      default: break;
    }
  }
}

/* cpu_compare_typed / cpu_compare_cplx (op_builder.rs:1828-1864, :1785-1822). */
void or_compare(int op, int dt, const void* a, const void* b, uint8_t* c, int ndim, const int64_t* shape,
                const int64_t* as, const int64_t* bs) {
  const uint64_t n = numel(ndim, shape);
#pragma omp parallel for schedule(static) num_threads(g_threads) if (g_threads > 1)
  for (uint64_t i = 0; i < n; ++i) {
    const int64_t oa = offset_nd(i, ndim, shape, as), ob = offset_nd(i, ndim, shape, bs);
    int r = 0;
    if (dt == C64 || dt == C128) {
      double ar, ai, br, bi;
      if (dt == C64) {
        ar = ((const c64_t*)a)[oa].re; ai = ((const c64_t*)a)[oa].im;
        br = ((const c64_t*)b)[ob].re; bi = ((const c64_t*)b)[ob].im;
      } else {
        ar = ((const c128_t*)a)[oa].re; ai = ((const c128_t*)a)[oa].im;
        br = ((const c128_t*)b)[ob].re; bi = ((const c128_t*)b)[ob].im;
      }
      r = op == EQ ? (ar == br && ai == bi) : (ar != br || ai != bi);
    } else if (dt == I64 || dt == U64) {
      /* 64-bit integers compare exactly (no double rounding) */
      if (dt == I64) {
        const int64_t x = ((const int64_t*)a)[oa], y = ((const int64_t*)b)[ob];
        r = op == EQ ? x == y : op == NE ? x != y : op == LT ? x < y : op == GT ? x > y : op == LE ? x <= y : x >= y;
      } else {
        const uint64_t x = ((const uint64_t*)a)[oa], y = ((const uint64_t*)b)[ob];
        r = op == EQ ? x == y : op == NE ? x != y : op == LT ? x < y : op == GT ? x > y : op == LE ? x <= y : x >= y;
      }
    } else if (dt == F32) {
      const float x = ((const float*)a)[oa], y = ((const float*)b)[ob];
      r = op == EQ ? x == y : op == NE ? x != y : op == LT ? x < y : op == GT ? x > y : op == LE ? x <= y : x >= y;
    } else {
      const double x = load_real(a, oa, dt), y = load_real(b, ob, dt);
      r = op == EQ ? x == y : op == NE ? x != y : op == LT ? x < y : op == GT ? x > y : op == LE ? x <= y : x >= y;
    }
    c[i] = (uint8_t)r;
  }
}

/* cpu_unary_elementwise (op_builder.rs:1869-1924) + complex neg/abs. */
static float un_f32(int op, float v) {
  switch (op) {
    case SIN: return sinf(v);
    case COS: return cosf(v);
    case EXP: return expf(v);
    case LOG: return logf(v);
    case ABS: return fabsf(v);
    case SIGN: return v > 0.0f ? 1.0f : (v < 0.0f ? -1.0f : 0.0f);
    default: return -v;
  }
}
static double un_f64(int op, double v) {
  switch (op) {
    case SIN: return sin(v);
    case COS: return cos(v);
    case EXP: return exp(v);
    case LOG: return log(v);
    case ABS: return fabs(v);
    case SIGN: return v > 0.0 ? 1.0 : (v < 0.0 ? -1.0 : 0.0);
    default: return -v;
  }
}
void or_unary(int op, int dt, const void* a, void* c, int ndim, const int64_t* shape, const int64_t* as) {
  const uint64_t n = numel(ndim, shape);
#pragma omp parallel for schedule(static) num_threads(g_threads) if (g_threads > 1)
  for (uint64_t i = 0; i < n; ++i) {
    const int64_t oa = offset_nd(i, ndim, shape, as);
    switch (dt) {
      case F32: ((float*)c)[i] = un_f32(op, ((const float*)a)[oa]); break;
      case F64: ((double*)c)[i] = un_f64(op, ((const double*)a)[oa]); break;
      case F16: ((uint16_t*)c)[i] = double_to_f16(un_f64(op, load_real(a, oa, dt))); break;
      case BF16: ((uint16_t*)c)[i] = double_to_bf16(un_f64(op, load_real(a, oa, dt))); break;
      case C64: {
        const c64_t x = ((const c64_t*)a)[oa];
        if (op == NEG) {
          ((c64_t*)c)[i].re = -x.re;
          ((c64_t*)c)[i].im = -x.im;
        } else {
          const double re = x.re, im = x.im;
          ((float*)c)[i] = (float)sqrt(re * re + im * im);
        }
        break;
      }
      case C128: {
        const c128_t x = ((const c128_t*)a)[oa];
        if (op == NEG) {
          ((c128_t*)c)[i].re = -x.re;
          ((c128_t*)c)[i].im = -x.im;
        } else {
          ((double*)c)[i] = sqrt(x.re * x.re + x.im * x.im);
        }
        break;
      }
      default: break;
    }
  }
}

/* cpu_clamp_typed (op_builder.rs:2017-2047): lo/hi narrowed to the dtype. */
void or_clamp(int dt, const void* a, void* c, double lo, double hi, int ndim, const int64_t* shape,
              const int64_t* as) {
  const uint64_t n = numel(ndim, shape);
  const float lof = (float)lo, hif = (float)hi;
  const double lo16 = dt == F16 ? f16_to_double(double_to_f16(lo)) : bf16_to_double(double_to_bf16(lo));
  const double hi16 = dt == F16 ? f16_to_double(double_to_f16(hi)) : bf16_to_double(double_to_bf16(hi));
#pragma omp parallel for schedule(static) num_threads(g_threads) if (g_threads > 1)
  for (uint64_t i = 0; i < n; ++i) {
    const int64_t oa = offset_nd(i, ndim, shape, as);
    if (dt == F32) {
      const float v = ((const float*)a)[oa];
      ((float*)c)[i] = v < lof ? lof : (v > hif ? hif : v);
    } else if (dt == F64) {
      const double v = ((const double*)a)[oa];
      ((double*)c)[i] = v < lo ? lo : (v > hi ? hi : v);
    } else {
      const double v = load_real(a, oa, dt);
      const double r = v < lo16 ? lo16 : (v > hi16 ? hi16 : v);
      ((uint16_t*)c)[i] = dt == F16 ? double_to_f16(r) : double_to_bf16(r);
    }
  }
}

/* Rust `as` float -> integer: truncate, saturate, NaN -> 0. */
static int64_t sat_i(double x, int bits) {
  if (isnan(x)) return 0;
  const double hr = ldexp(1.0, bits - 1);
  if (x <= -hr) return bits == 64 ? INT64_MIN : -(int64_t)hr;
  if (x >= hr) return bits == 64 ? INT64_MAX : (int64_t)hr - 1;
  return (int64_t)x;
}
static uint64_t sat_u(double x, int bits) {
  if (isnan(x) || x <= 0.0) return 0;
  const double r = ldexp(1.0, bits);
  if (x >= r) return bits == 64 ? UINT64_MAX : (uint64_t)r - 1;
  return (uint64_t)x;
}

/* cpu_cast (op_builder.rs:2052-2160): Rust `as` semantics; plus the 16-bit
 * float and bool targets (nearest-even; bool = nonzero). */
void or_cast(int src, int dst, const void* a, void* c, int ndim, const int64_t* shape, const int64_t* as) {
  const uint64_t n = numel(ndim, shape);
#pragma omp parallel for schedule(static) num_threads(g_threads) if (g_threads > 1)
  for (uint64_t i = 0; i < n; ++i) {
    const int64_t oa = offset_nd(i, ndim, shape, as);
    if (src == C64 || src == C128) { /* complex -> complex only */
      double re, im;
      if (src == C64) { re = ((const c64_t*)a)[oa].re; im = ((const c64_t*)a)[oa].im; }
      else { re = ((const c128_t*)a)[oa].re; im = ((const c128_t*)a)[oa].im; }
      if (dst == C128) { ((c128_t*)c)[i].re = re; ((c128_t*)c)[i].im = im; }
      else { ((c64_t*)c)[i].re = (float)re; ((c64_t*)c)[i].im = (float)im; }
      continue;
    }
    /* exact integer paths for 64-bit sources */
    const int src_int = (src >= I8 && src <= U64) || src == BOOL;
    int64_t iv = 0;
    uint64_t uv = 0;
    if (src == I64) { iv = ((const int64_t*)a)[oa]; uv = (uint64_t)iv; }
    else if (src == U64) { uv = ((const uint64_t*)a)[oa]; iv = (int64_t)uv; }
    else if (src_int) { iv = (int64_t)load_real(a, oa, src); uv = (uint64_t)iv; }
    const double dv = src_int ? 0.0 : load_real(a, oa, src);
    switch (dst) {
      case F32:
        if (src == F32) ((float*)c)[i] = ((const float*)a)[oa];
        else if (src == U64) ((float*)c)[i] = (float)uv;
        else if (src_int) ((float*)c)[i] = (float)iv;
        else ((float*)c)[i] = (float)dv;
        break;
      case F64:
        if (src == U64) ((double*)c)[i] = (double)uv;
        else if (src_int) ((double*)c)[i] = (double)iv;
        else ((double*)c)[i] = dv;
        break;
      case F16:
      case BF16: {
        double v;
        if (src == U64) v = (double)uv; else if (src_int) v = (double)iv; else v = dv;
        ((uint16_t*)c)[i] = dst == F16 ? double_to_f16(v) : double_to_bf16(v);
        break;
      }
      case C64:
        ((c64_t*)c)[i].re = src_int ? (float)iv : (float)dv;
        ((c64_t*)c)[i].im = 0.0f;
        break;
      case C128:
        ((c128_t*)c)[i].re = src_int ? (double)iv : dv;
        ((c128_t*)c)[i].im = 0.0;
        break;
      case BOOL: ((uint8_t*)c)[i] = src_int ? (uv != 0) : (dv != 0.0); break;
      case I8: ((int8_t*)c)[i] = src_int ? (int8_t)iv : (int8_t)sat_i(dv, 8); break;
      case I16: ((int16_t*)c)[i] = src_int ? (int16_t)iv : (int16_t)sat_i(dv, 16); break;
      case I32: ((int32_t*)c)[i] = src_int ? (int32_t)iv : (int32_t)sat_i(dv, 32); break;
      case I64: ((int64_t*)c)[i] = src_int ? iv : sat_i(dv, 64); break;
      case U8: ((uint8_t*)c)[i] = src_int ? (uint8_t)uv : (uint8_t)sat_u(dv, 8); break;
      case U16: ((uint16_t*)c)[i] = src_int ? (uint16_t)uv : (uint16_t)sat_u(dv, 16); break;
      case U32: ((uint32_t*)c)[i] = src_int ? (uint32_t)uv : (uint32_t)sat_u(dv, 32); break;
      case U64: ((uint64_t*)c)[i] = src_int ? uv : sat_u(dv, 64); break;
      default: break;
    }
  }
}

/* ------------------------------------------------------------------------ */
/* Reductions (cpu_reduce_typed :3496-3582, cpu_mean_typed :3585-3619,      */
/* cpu_reduce_cplx :3439-3492), one axis; base offset per output as in      */
/* cpu_reduce_offset (:3374-3399). `dt` is the compute dtype.               */
/* ------------------------------------------------------------------------ */
static int64_t reduce_base(uint64_t out_idx, int ndim, const int64_t* shape, const int64_t* strides, int axis) {
  int64_t off = 0;
  uint64_t t = out_idx;
  for (int i = ndim - 1; i >= 0; --i) {
    if (i == axis) continue;
    uint64_t c = t % (uint64_t)shape[i];
    t /= (uint64_t)shape[i];
    off += (int64_t)c * strides[i];
  }
  return off;
}

/* One-output max/min/argmax/argmin over many threads with the sequential
 * loop's exact result: chunk 0 runs the loop from element 0 (a NaN there
 * decides, as x > NaN never holds); every later chunk finds the first
 * occurrence of its largest (smallest) non-NaN element; the chunks are
 * merged in order with the same strict comparison, so an equal value in a
 * later chunk never replaces an earlier one. */
#define OR_EXT_ALL(T, IS_NAN)                                                                  \
  do {                                                                                        \
    const T* x = (const T*)a + base;                                                          \
    T cb[256];                                                                                \
    int64_t ci[256];                                                                          \
    int has[256];                                                                             \
    _Pragma("omp parallel for schedule(static) num_threads(nch)")                             \
    for (int t = 0; t < nch; ++t) {                                                           \
      const int64_t k0 = axis_len * t / nch, k1 = axis_len * (t + 1) / nch;                  \
      T best = x[0];                                                                          \
      int64_t bi = 0;                                                                         \
      int h = (t == 0);                                                                       \
      for (int64_t k = (t == 0 ? 1 : k0); k < k1; ++k) {                                      \
        const T v = x[k * ast];                                                               \
        if (!h) {                                                                             \
          if (!(IS_NAN(v))) { best = v; bi = k; h = 1; }                                      \
        } else if ((want_max && v > best) || (!want_max && v < best)) {                       \
          best = v; bi = k;                                                                   \
        }                                                                                     \
      }                                                                                       \
      cb[t] = best; ci[t] = bi; has[t] = h;                                                   \
    }                                                                                         \
    T best = cb[0];                                                                           \
    int64_t bi = ci[0];                                                                       \
    for (int t = 1; t < nch; ++t)                                                             \
      if (has[t] && ((want_max && cb[t] > best) || (!want_max && cb[t] < best))) {            \
        best = cb[t]; bi = ci[t];                                                             \
      }                                                                                       \
    if (op == R_MAX || op == R_MIN) *(T*)c = best; else *(int64_t*)c = bi;                     \
  } while (0)

#define OR_NAN_F(v) ((v) != (v))
#define OR_NAN_I(v) 0

static int reduce_ext_all_parallel(int op, int dt, const void* a, void* c, int64_t base, int64_t ast,
                                   int64_t axis_len) {
  if (!(op == R_MAX || op == R_MIN || op == R_ARGMAX || op == R_ARGMIN)) return 0;
  if (!(dt == F32 || dt == F64 || dt == I64) || g_threads <= 1 || axis_len < (1 << 16)) return 0;
  const int want_max = (op == R_MAX || op == R_ARGMAX);
  int nch = g_threads < 256 ? g_threads : 256;
  if (dt == F32) OR_EXT_ALL(float, OR_NAN_F);
  else if (dt == F64) OR_EXT_ALL(double, OR_NAN_F);
  else OR_EXT_ALL(int64_t, OR_NAN_I);
  return 1;
}

void or_reduce(int op, int dt, const void* a, void* c, int ndim, const int64_t* shape, const int64_t* strides,
               int axis, int64_t axis_len, int64_t out_size) {
  if (out_size <= 0 || axis_len <= 0) return;
  const int64_t ast = strides[axis];
  if (out_size == 1 &&
      reduce_ext_all_parallel(op, dt, a, c, reduce_base(0, ndim, shape, strides, axis), ast, axis_len))
    return;
#pragma omp parallel for schedule(static) num_threads(g_threads) if (g_threads > 1)
  for (int64_t o = 0; o < out_size; ++o) {
    const int64_t base = reduce_base((uint64_t)o, ndim, shape, strides, axis);
    if (dt == C64 || dt == C128) {
      double re = 0.0, im = 0.0;
      if (op == R_PROD) re = 1.0;
      for (int64_t k = 0; k < axis_len; ++k) {
        const int64_t off = base + k * ast;
        double br, bi;
        if (dt == C64) { br = ((const c64_t*)a)[off].re; bi = ((const c64_t*)a)[off].im; }
        else { br = ((const c128_t*)a)[off].re; bi = ((const c128_t*)a)[off].im; }
        if (op == R_PROD) {
          const double ar = re, ai = im;
          re = ar * br - ai * bi;
          im = ar * bi + ai * br;
        } else {
          re += br;
          im += bi;
        }
      }
      if (op == R_MEAN) { re /= (double)axis_len; im /= (double)axis_len; }
      if (dt == C64) { ((c64_t*)c)[o].re = (float)re; ((c64_t*)c)[o].im = (float)im; }
      else { ((c128_t*)c)[o].re = re; ((c128_t*)c)[o].im = im; }
      continue;
    }
    if (dt == F32) {
      const float* x = (const float*)a;
      if (op == R_SUM || op == R_MEAN) {
        float acc = 0.0f;
        for (int64_t k = 0; k < axis_len; ++k) acc = acc + x[base + k * ast];
        if (op == R_MEAN) {
          float count = 0.0f; /* the count is built by repeated addition in T (:3611-3616) */
          for (int64_t k = 0; k < axis_len; ++k) count = count + 1.0f;
          acc = acc / count;
        }
        ((float*)c)[o] = acc;
      } else if (op == R_PROD) {
        float acc = 1.0f;
        for (int64_t k = 0; k < axis_len; ++k) acc = acc * x[base + k * ast];
        ((float*)c)[o] = acc;
      } else {
        const int want_max = (op == R_MAX || op == R_ARGMAX);
        float best = x[base];
        int64_t bi = 0;
        for (int64_t k = 1; k < axis_len; ++k) {
          const float v = x[base + k * ast];
          if ((want_max && v > best) || (!want_max && v < best)) { best = v; bi = k; }
        }
        if (op == R_MAX || op == R_MIN) ((float*)c)[o] = best; else ((int64_t*)c)[o] = bi;
      }
    } else if (dt == F64) {
      const double* x = (const double*)a;
      if (op == R_SUM || op == R_MEAN) {
        double acc = 0.0;
        for (int64_t k = 0; k < axis_len; ++k) acc = acc + x[base + k * ast];
        if (op == R_MEAN) {
          double count = 0.0;
          for (int64_t k = 0; k < axis_len; ++k) count = count + 1.0;
          acc = acc / count;
        }
        ((double*)c)[o] = acc;
      } else if (op == R_PROD) {
        double acc = 1.0;
        for (int64_t k = 0; k < axis_len; ++k) acc = acc * x[base + k * ast];
        ((double*)c)[o] = acc;
      } else {
        const int want_max = (op == R_MAX || op == R_ARGMAX);
        double best = x[base];
        int64_t bi = 0;
        for (int64_t k = 1; k < axis_len; ++k) {
          const double v = x[base + k * ast];
          if ((want_max && v > best) || (!want_max && v < best)) { best = v; bi = k; }
        }
        if (op == R_MAX || op == R_MIN) ((double*)c)[o] = best; else ((int64_t*)c)[o] = bi;
      }
    } else { /* I64 (wrapping arithmetic, like release-mode Rust) */
      const int64_t* x = (const int64_t*)a;
      if (op == R_SUM) {
        uint64_t acc = 0;
        for (int64_t k = 0; k < axis_len; ++k) acc += (uint64_t)x[base + k * ast];
        ((int64_t*)c)[o] = (int64_t)acc;
      } else if (op == R_PROD) {
        uint64_t acc = 1;
        for (int64_t k = 0; k < axis_len; ++k) acc *= (uint64_t)x[base + k * ast];
        ((int64_t*)c)[o] = (int64_t)acc;
      } else {
        const int want_max = (op == R_MAX || op == R_ARGMAX);
        int64_t best = x[base], bi = 0;
        for (int64_t k = 1; k < axis_len; ++k) {
          const int64_t v = x[base + k * ast];
          if ((want_max && v > best) || (!want_max && v < best)) { best = v; bi = k; }
        }
        if (op == R_MAX || op == R_MIN) ((int64_t*)c)[o] = best; else ((int64_t*)c)[o] = bi;
      }
    }
  }
}

/* cpu_cumsum_typed (op_builder.rs:3640-3688). The reference re-adds each
 * output's whole prefix; a running sum performs the same additions in the
 * same order, so it is bit-identical and O(N). */
void or_cumsum(int dt, const void* a, void* c, int ndim, const int64_t* shape, const int64_t* strides, int axis) {
  const uint64_t n = numel(ndim, shape);
  if (n == 0) return;
  const int64_t L = shape[axis];
  const uint64_t rows = n / (uint64_t)L;
  int64_t inner = 1; /* output (C-contiguous) stride of the axis */
  for (int i = axis + 1; i < ndim; ++i) inner *= shape[i];
  const int64_t ast = strides[axis];
#pragma omp parallel for schedule(static) num_threads(g_threads) if (g_threads > 1)
  for (uint64_t r = 0; r < rows; ++r) {
    /* row r: the C-order index of the first element of this lane */
    const uint64_t hi = r / (uint64_t)inner, lo = r % (uint64_t)inner;
    const uint64_t first = hi * (uint64_t)L * (uint64_t)inner + lo;
    const int64_t base = offset_nd(first, ndim, shape, strides);
    if (dt == F32) {
      float acc = 0.0f;
      for (int64_t k = 0; k < L; ++k) {
        acc = acc + ((const float*)a)[base + k * ast];
        ((float*)c)[first + (uint64_t)k * inner] = acc;
      }
    } else if (dt == F64) {
      double acc = 0.0;
      for (int64_t k = 0; k < L; ++k) {
        acc = acc + ((const double*)a)[base + k * ast];
        ((double*)c)[first + (uint64_t)k * inner] = acc;
      }
    } else {
      uint64_t acc = 0;
      for (int64_t k = 0; k < L; ++k) {
        acc += (uint64_t)((const int64_t*)a)[base + k * ast];
        ((int64_t*)c)[first + (uint64_t)k * inner] = (int64_t)acc;
      }
    }
  }
}
