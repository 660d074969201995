// Reduction kernels and policies (see reduce.cu for the planning side).
// Kernels are templated on the policy only: the output dtype is a runtime
// switch at the single store per output, and the vectorised / split variants
// are runtime flags, which keeps the instantiation count small.
#pragma once
#include <math.h>
#include <stdint.h>
#include <type_traits>
#include "common.cuh"
#include "internal.h"
#include "plan.h"
#include "reduce.h"

namespace mpb {
namespace red {

constexpr int kRedThreads = 256;

// ----------------------------------------------------------- accumulators
template <class V>
struct ArgAcc {
  V v;
  int64_t i;
};

MPB_D float shfl_dn(float x, int o) { return __shfl_down_sync(0xffffffffu, x, o); }
MPB_D double shfl_dn(double x, int o) { return __shfl_down_sync(0xffffffffu, x, o); }
MPB_D uint64_t shfl_dn(uint64_t x, int o) { return __shfl_down_sync(0xffffffffu, (unsigned long long)x, o); }
MPB_D int64_t shfl_dn(int64_t x, int o) { return __shfl_down_sync(0xffffffffu, (long long)x, o); }
MPB_D c128 shfl_dn(c128 x, int o) { return c128{shfl_dn(x.re, o), shfl_dn(x.im, o)}; }
template <class V>
MPB_D ArgAcc<V> shfl_dn(ArgAcc<V> x, int o) {
  return ArgAcc<V>{shfl_dn(x.v, o), shfl_dn(x.i, o)};
}
MPB_D float shfl_x(float x, int o) { return __shfl_xor_sync(0xffffffffu, x, o); }
MPB_D double shfl_x(double x, int o) { return __shfl_xor_sync(0xffffffffu, x, o); }
MPB_D int64_t shfl_x(int64_t x, int o) { return __shfl_xor_sync(0xffffffffu, (long long)x, o); }
MPB_D uint64_t shfl_x(uint64_t x, int o) { return __shfl_xor_sync(0xffffffffu, (unsigned long long)x, o); }

MPB_D float radd(float a, float b) { return a + b; }
MPB_D double radd(double a, double b) { return a + b; }
MPB_D uint64_t radd(uint64_t a, uint64_t b) { return a + b; }  // wraps like i64 in release Rust
MPB_D c128 radd(c128 a, c128 b) { return c128{a.re + b.re, a.im + b.im}; }
MPB_D float rmul(float a, float b) { return a * b; }
MPB_D double rmul(double a, double b) { return a * b; }
MPB_D uint64_t rmul(uint64_t a, uint64_t b) { return a * b; }
// Complex product as the CPU loop writes it (op_builder.rs:3474-3481).
MPB_D c128 rmul(c128 a, c128 b) {
  return c128{__dsub_rn(__dmul_rn(a.re, b.re), __dmul_rn(a.im, b.im)),
              __dadd_rn(__dmul_rn(a.re, b.im), __dmul_rn(a.im, b.re))};
}

template <class Acc> MPB_D Acc zero_of();
template <> MPB_D float zero_of<float>() { return 0.0f; }
template <> MPB_D double zero_of<double>() { return 0.0; }
template <> MPB_D uint64_t zero_of<uint64_t>() { return 0; }
template <> MPB_D c128 zero_of<c128>() { return c128{0.0, 0.0}; }
template <class Acc> MPB_D Acc one_of();
template <> MPB_D float one_of<float>() { return 1.0f; }
template <> MPB_D double one_of<double>() { return 1.0; }
template <> MPB_D uint64_t one_of<uint64_t>() { return 1; }
template <> MPB_D c128 one_of<c128>() { return c128{1.0, 0.0}; }

// Reduction policies: In = storage type read, Acc = accumulator.
template <class TIn, class TAcc>
struct PSum {
  using In = TIn;
  using Acc = TAcc;
  static constexpr bool kArg = false;
  static constexpr bool kExt = false;
  MPB_D static Acc ident() { return zero_of<Acc>(); }
  MPB_D static void fold(Acc& a, const In& x, int64_t) { a = radd(a, cvt<Acc>(x)); }
  MPB_D static void fold_seq(Acc& a, const In& x, int64_t i) { fold(a, x, i); }
  MPB_D static Acc merge(const Acc& l, const Acc& r) { return radd(l, r); }
};
template <class TIn, class TAcc>
struct PProd {
  using In = TIn;
  using Acc = TAcc;
  static constexpr bool kArg = false;
  static constexpr bool kExt = false;
  MPB_D static Acc ident() { return one_of<Acc>(); }
  MPB_D static void fold(Acc& a, const In& x, int64_t) { a = rmul(a, cvt<Acc>(x)); }
  MPB_D static void fold_seq(Acc& a, const In& x, int64_t i) { fold(a, x, i); }
  MPB_D static Acc merge(const Acc& l, const Acc& r) { return rmul(l, r); }
};
template <class V> MPB_D V lowest();
template <class V> MPB_D V highest();
template <> MPB_D float lowest<float>() { return -INFINITY; }
template <> MPB_D float highest<float>() { return INFINITY; }
template <> MPB_D double lowest<double>() { return -INFINITY; }
template <> MPB_D double highest<double>() { return INFINITY; }
template <> MPB_D int64_t lowest<int64_t>() { return INT64_MIN; }
template <> MPB_D int64_t highest<int64_t>() { return INT64_MAX; }

template <class TIn, class V, bool IS_MAX>
struct PArg {
  using In = TIn;
  using Acc = ArgAcc<V>;
  static constexpr bool kArg = true;
  static constexpr bool kExt = false;
  MPB_D static Acc ident() { return Acc{IS_MAX ? lowest<V>() : highest<V>(), INT64_MAX}; }
  MPB_D static bool better(V v, int64_t i, const Acc& a) {
    return IS_MAX ? (v > a.v || (v == a.v && i < a.i)) : (v < a.v || (v == a.v && i < a.i));
  }
  MPB_D static void fold(Acc& a, const In& x, int64_t idx) {
    const V v = cvt<V>(x);
    if (better(v, idx, a)) a = Acc{v, idx};
  }
  // Fold for a traversal in increasing index order: an equal value can only
  // win while nothing has been taken yet, so no index comparison is needed.
  MPB_D static void fold_seq(Acc& a, const In& x, int64_t idx) {
    const V v = cvt<V>(x);
    if (IS_MAX ? (v > a.v || (v == a.v && a.i == INT64_MAX)) : (v < a.v || (v == a.v && a.i == INT64_MAX)))
      a = Acc{v, idx};
  }
  MPB_D static Acc merge(const Acc& l, const Acc& r) { return better(r.v, r.i, l) ? r : l; }
  // strictly better value (ties keep the earlier one)
  MPB_D static bool beats(V m, V b) { return IS_MAX ? (m > b) : (m < b); }
  // NaN-ignoring extreme of two values (fmax/fmin return the non-NaN one).
  MPB_D static V pick(V a, V b) {
    if constexpr (std::is_same<V, int64_t>::value) {
      return IS_MAX ? (a > b ? a : b) : (a < b ? a : b);
    } else if constexpr (std::is_same<V, float>::value) {
      return IS_MAX ? fmaxf(a, b) : fminf(a, b);
    } else {
      return IS_MAX ? fmax(a, b) : fmin(a, b);
    }
  }
  // Can a group whose extreme is m and whose smallest index is `first` change
  // the accumulator? Any element that `better` would take makes this true:
  // a strictly better value implies m is strictly better, and an equal value
  // only wins with an index below a.i, which needs first < a.i.
  MPB_D static bool improves(V m, const Acc& a, int64_t first) {
    return IS_MAX ? (m > a.v || (m == a.v && first < a.i)) : (m < a.v || (m == a.v && first < a.i));
  }
};

// max / min values alone (no index): the CPU loop keeps the first element
// and replaces it only by a strictly greater (smaller) one, so its result is
//  * NaN when the first element is NaN (write_out applies that rule),
//  * otherwise the extremum of the non-NaN elements, which fmax/fmin give in
//    any order, except for the sign of a zero result: equal values never
//    replace the accumulator, so a zero extremum carries the sign of the first
//    zero in index order. Kernels settle that case by a rescan
//    (ext_zero_fix_*), which runs only for outputs whose extremum is zero.
template <class TIn, class V, bool IS_MAX>
struct PExt {
  using In = TIn;
  using Acc = V;
  static constexpr bool kArg = false;
  static constexpr bool kExt = true;
  MPB_D static Acc ident() { return IS_MAX ? lowest<V>() : highest<V>(); }
  MPB_D static V pick(V a, V b) { return PArg<TIn, V, IS_MAX>::pick(a, b); }
  MPB_D static void fold(Acc& a, const In& x, int64_t) { a = pick(a, cvt<V>(x)); }
  MPB_D static void fold_seq(Acc& a, const In& x, int64_t i) { fold(a, x, i); }
  MPB_D static Acc merge(const Acc& l, const Acc& r) { return pick(l, r); }
};

template <class P>
MPB_D typename P::Acc warp_reduce(typename P::Acc a) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    typename P::Acc other = shfl_dn(a, o);
    a = P::merge(a, other);
  }
  return a;
}

template <class P>
MPB_D typename P::Acc block_reduce(typename P::Acc a) {
  __shared__ __align__(16) char raw[32 * sizeof(typename P::Acc)];
  typename P::Acc* sm = reinterpret_cast<typename P::Acc*>(raw);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  a = warp_reduce<P>(a);
  __syncthreads();  // protect `sm` reuse across output iterations
  if (lane == 0) sm[warp] = a;
  __syncthreads();
  const int nw = blockDim.x >> 5;
  if (warp == 0) {
    a = lane < nw ? sm[lane] : P::ident();
    a = warp_reduce<P>(a);
  }
  return a;
}

// ---------------------------------------------------------------- output
// mode: 0 sum/prod value, 1 mean, 2 extremum value, 3 extremum index,
// 4 extremum (value, index) record for cross-shard combining.
struct RedOut {
  int mode;
  int out_dt;
  int nan_rule;     // apply the first-element NaN rule
  int pad;
  int64_t count;    // elements per output (mean divisor)
  int64_t ostride;  // output element stride
};

template <class V> MPB_D bool is_nan_v(V v) { return v != v; }
template <> MPB_D bool is_nan_v<int64_t>(int64_t) { return false; }

MPB_D float mean_div(float s, int64_t n) { return s / (float)n; }
MPB_D double mean_div(double s, int64_t n) { return s / (double)n; }
MPB_D c128 mean_div(c128 s, int64_t n) { return c128{s.re / (double)n, s.im / (double)n}; }
MPB_D uint64_t mean_div(uint64_t s, int64_t) { return s; }  // unused: integer means accumulate in f64

template <class V>
MPB_D void store_dyn(void* out, int64_t i, int dt, const V& v) {
  switch (dt) {
    case MPB_F32: static_cast<float*>(out)[i] = cvt<float>(v); break;
    case MPB_F64: static_cast<double*>(out)[i] = cvt<double>(v); break;
    case MPB_I64: static_cast<int64_t*>(out)[i] = cvt<int64_t>(v); break;
    case MPB_U64: static_cast<uint64_t*>(out)[i] = cvt<uint64_t>(v); break;
    case MPB_F16: static_cast<__half*>(out)[i] = cvt<__half>(v); break;
    case MPB_BF16: static_cast<__nv_bfloat16*>(out)[i] = cvt<__nv_bfloat16>(v); break;
    case MPB_C64: static_cast<c64*>(out)[i] = cvt<c64>(v); break;
    case MPB_C128: static_cast<c128*>(out)[i] = cvt<c128>(v); break;
    default: break;
  }
}

template <class P>
MPB_D void write_out(void* out, int64_t o, typename P::Acc acc, const RedOut& ro, const typename P::In* first) {
  const int64_t i = o * ro.ostride;
  if constexpr (P::kArg) {
    using V = decltype(acc.v);
    bool nan_first = false;
    if constexpr (!std::is_same<V, int64_t>::value) {
      if (ro.nan_rule) nan_first = is_nan_v<V>(cvt<V>(*first));
    }
    if (ro.mode == 4) {
      // shard record {value bits, index}: double bits for float inputs, the
      // raw value for integer inputs; index INT64_MAX when nothing qualified.
      int64_t* rec = static_cast<int64_t*>(out) + 2 * i;
      if constexpr (std::is_same<V, int64_t>::value) {
        rec[0] = acc.v;
      } else {
        rec[0] = __double_as_longlong(nan_first ? (double)NAN : (double)acc.v);
      }
      rec[1] = nan_first ? 0 : acc.i;
    } else if (ro.mode == 3) {
      store_dyn(out, i, ro.out_dt, (int64_t)(nan_first ? 0 : acc.i));
    } else if (nan_first) {
      store_dyn(out, i, ro.out_dt, *first);
    } else {
      store_dyn(out, i, ro.out_dt, acc.v);
    }
  } else if constexpr (P::kExt) {
    if constexpr (!std::is_same<typename P::Acc, int64_t>::value) {
      if (ro.nan_rule && is_nan_v(cvt<typename P::Acc>(*first))) {
        store_dyn(out, i, ro.out_dt, *first);
        return;
      }
    }
    store_dyn(out, i, ro.out_dt, acc);
  } else {
    if (ro.mode == 1)
      store_dyn(out, i, ro.out_dt, mean_div(acc, ro.count));
    else
      store_dyn(out, i, ro.out_dt, acc);
  }
}

// --------------------------------------------------------------- geometry
struct RedDev {
  int K, R;
  int64_t M, L, Li, Lo;
  int64_t ks[kMaxCollapsed], kst[kMaxCollapsed];
  int64_t rs[kMaxCollapsed], rst[kMaxCollapsed], rw[kMaxCollapsed];
};

MPB_D int64_t kept_off(const RedDev& g, int64_t o) {
  if (g.K <= 1) return g.K == 1 ? o * g.kst[0] : 0;  // o < ks[0]: no division
  int64_t off = 0;
  for (int d = g.K - 1; d >= 0; --d) {
    const int64_t c = o % g.ks[d];
    o /= g.ks[d];
    off += c * g.kst[d];
  }
  return off;
}
// Offset and logical flat index of reduced segment s (all reduced dims but
// the innermost).
MPB_D void seg_off(const RedDev& g, int64_t s, int64_t& off, int64_t& lidx) {
  off = 0;
  lidx = 0;
  for (int d = g.R - 2; d >= 0; --d) {
    const int64_t c = s % g.rs[d];
    s /= g.rs[d];
    off += c * g.rst[d];
    lidx += c * g.rw[d];
  }
}
MPB_D void red_off(const RedDev& g, int64_t f, int64_t& off, int64_t& lidx) {
  off = 0;
  lidx = 0;
  for (int d = g.R - 1; d >= 0; --d) {
    const int64_t c = f % g.rs[d];
    f /= g.rs[d];
    off += c * g.rst[d];
    lidx += c * g.rw[d];
  }
}

// ------------------------------------------- zero extremum sign (PExt)
// Smallest logical index among the zero elements of output o's segment,
// scanned by `n` cooperating threads (thread t takes elements t, t+n, ...);
// returns the index and whether that zero is negative.
template <class P>
MPB_D void first_zero_scan(const typename P::In* __restrict__ seg, const RedDev& g, int t, int n, int64_t& best,
                           bool& neg) {
  best = INT64_MAX;
  neg = false;
  for (int64_t f = t; f < g.L; f += n) {
    int64_t off, lidx;
    red_off(g, f, off, lidx);
    const typename P::Acc v = cvt<typename P::Acc>(seg[off]);
    if (v == 0 && lidx < best) {
      best = lidx;
      neg = signbit(v);
    }
  }
}
template <class V> MPB_D V signed_zero(bool neg) { return neg ? -V(0) : V(0); }

// Warp version: all 32 lanes call it with the warp's result in lane 0.
template <class P>
MPB_D typename P::Acc ext_zero_fix_warp(typename P::Acc acc, const typename P::In* __restrict__ seg,
                                        const RedDev& g, int lane) {
  if constexpr (P::kExt && !std::is_same<typename P::Acc, int64_t>::value) {
    acc = __shfl_sync(0xffffffffu, acc, 0);
    if (acc == 0) {
      int64_t best;
      bool neg;
      first_zero_scan<P>(seg, g, lane, 32, best, neg);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const int64_t ob = shfl_dn(best, o);
        const bool on = __shfl_down_sync(0xffffffffu, (int)neg, o) != 0;
        if (ob < best) {
          best = ob;
          neg = on;
        }
      }
      acc = signed_zero<typename P::Acc>(neg);
    }
  }
  return acc;
}
// Single-thread version.
template <class P>
MPB_D typename P::Acc ext_zero_fix_thread(typename P::Acc acc, const typename P::In* __restrict__ seg,
                                          const RedDev& g) {
  if constexpr (P::kExt && !std::is_same<typename P::Acc, int64_t>::value) {
    if (acc == 0) {
      int64_t best;
      bool neg;
      first_zero_scan<P>(seg, g, 0, 1, best, neg);
      acc = signed_zero<typename P::Acc>(neg);
    }
  }
  return acc;
}

// ------------------------------------------------- ROW: warp per output
template <class A> struct AccValue { using type = A; };
template <class V> struct AccValue<ArgAcc<V>> { using type = V; };

template <class P, int VEC>
MPB_D void fold_segment_vec(typename P::Acc& acc, const typename P::In* __restrict__ p, int64_t li, int64_t lbase,
                            int64_t rwi, int lane, int nthreads, int tid) {
  using In = typename P::In;
  using V = typename AccValue<typename P::Acc>::type;
  constexpr int UNR = 4;
  const int64_t step = (int64_t)nthreads * VEC;
  int64_t c = (int64_t)tid * VEC;
  V best{};
  int64_t cbest = -1;  // start of the group that first reached `best` (arg policies)
  for (; c + (UNR - 1) * step < li; c += UNR * step) {
    uint4 w[UNR][(VEC * sizeof(In) + 15) / 16];
#pragma unroll
    for (int u = 0; u < UNR; ++u) {
#pragma unroll
      for (int k = 0; k < (int)((VEC * sizeof(In) + 15) / 16); ++k)
        w[u][k] = ld_stream16(reinterpret_cast<const char*>(p + c + u * step) + 16 * k);
    }
    if constexpr (P::kArg) {
      // Extreme of the UNR*VEC values (one min/max per element); only which
      // group first reached the best value is remembered (selects, no
      // branch), and that group is re-read once at the end of the segment.
      V m = P::pick(cvt<V>(reinterpret_cast<const In*>(w[0])[0]),
                    cvt<V>(reinterpret_cast<const In*>(w[0])[VEC > 1 ? 1 : 0]));
#pragma unroll
      for (int u = 0; u < UNR; ++u) {
        const In* v = reinterpret_cast<const In*>(w[u]);
#pragma unroll
        for (int j = 0; j < VEC; ++j) m = P::pick(m, cvt<V>(v[j]));
      }
      // the first non-NaN group, then strictly better ones (an all-NaN group
      // gives m = NaN, which never wins)
      const bool take = cbest < 0 ? !is_nan_v<V>(m) : P::beats(m, best);
      best = take ? m : best;
      cbest = take ? c : cbest;
    } else {
#pragma unroll
      for (int u = 0; u < UNR; ++u) {
        const In* v = reinterpret_cast<const In*>(w[u]);
#pragma unroll
        for (int j = 0; j < VEC; ++j) P::fold(acc, v[j], lbase + (c + u * step + j) * rwi);
      }
    }
  }
  if constexpr (P::kArg) {
    // Only a lane whose best equals the warp's best can hold the answer of
    // the main loop's groups (a lower best is beaten by an element of the
    // warp-best group); the other lanes skip the re-read, which on long
    // segments is a DRAM access of four scattered 16-byte words per lane.
    // Every caller runs this with the whole warp.
    {
      V wb = best;
      bool wh = cbest >= 0;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const V ob = shfl_x(wb, o);
        const bool oh = __shfl_xor_sync(0xffffffffu, (int)wh, o) != 0;
        const bool t = oh && (!wh || P::beats(ob, wb));
        wb = t ? ob : wb;
        wh = wh || oh;
      }
      if (cbest >= 0 && !(best == wb)) cbest = -1;
    }
    if (cbest >= 0) {
      // first element of the best group equal to the best value (it exists:
      // the group's extreme is one of its elements), merged with the rule
      int64_t idx = 0;
      bool found = false;
#pragma unroll
      for (int u = 0; u < UNR; ++u) {
        uint4 w[(VEC * sizeof(In) + 15) / 16];
#pragma unroll
        for (int k = 0; k < (int)((VEC * sizeof(In) + 15) / 16); ++k)
          w[k] = ld_nc16(reinterpret_cast<const char*>(p + cbest + u * step) + 16 * k);
        const In* v = reinterpret_cast<const In*>(w);
#pragma unroll
        for (int j = 0; j < VEC; ++j) {
          const bool hit = !found && cvt<V>(v[j]) == best;
          idx = hit ? lbase + (cbest + u * step + j) * rwi : idx;
          found = found || hit;
        }
      }
      acc = P::merge(acc, typename P::Acc{best, idx});
    }
  }
  for (; c < li; c += step) {
    uint4 w[(VEC * sizeof(In) + 15) / 16];
#pragma unroll
    for (int k = 0; k < (int)((VEC * sizeof(In) + 15) / 16); ++k)
      w[k] = ld_stream16(reinterpret_cast<const char*>(p + c) + 16 * k);
    const In* v = reinterpret_cast<const In*>(w);
#pragma unroll
    for (int j = 0; j < VEC; ++j) P::fold(acc, v[j], lbase + (c + j) * rwi);
  }
  (void)lane;
}

template <class P>
MPB_D void fold_segment_scalar(typename P::Acc& acc, const typename P::In* __restrict__ p, int64_t li,
                               int64_t lbase, int64_t rwi, int64_t c0, int64_t c1, int nthreads, int tid) {
  constexpr int UNR = 4;
  int64_t c = c0 + tid;
  for (; c + (UNR - 1) * (int64_t)nthreads < c1; c += UNR * (int64_t)nthreads) {
    typename P::In v[UNR];
#pragma unroll
    for (int u = 0; u < UNR; ++u) v[u] = p[c + u * (int64_t)nthreads];
#pragma unroll
    for (int u = 0; u < UNR; ++u) P::fold(acc, v[u], lbase + (c + u * (int64_t)nthreads) * rwi);
  }
  for (; c < c1; c += nthreads) P::fold(acc, p[c], lbase + c * rwi);
  (void)li;
}

template <class P>
__global__ void __launch_bounds__(kRedThreads) k_red_row_warp(const typename P::In* __restrict__ a, void* out,
                                                               RedDev g, RedOut ro, int vec) {
  pdl_enter();
  constexpr int VEC = 16 / sizeof(typename P::In) > 0 ? 16 / sizeof(typename P::In) : 1;
  const int lane = threadIdx.x & 31;
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int64_t rwi = g.rw[g.R - 1];
  for (int64_t o = gw; o < g.M; o += nw) {
    const int64_t base = kept_off(g, o);
    typename P::Acc acc = P::ident();
    for (int64_t s = 0; s < g.Lo; ++s) {
      int64_t so, sl;
      seg_off(g, s, so, sl);
      if (vec)
        fold_segment_vec<P, VEC>(acc, a + base + so, g.Li, sl, rwi, lane, 32, lane);
      else
        fold_segment_scalar<P>(acc, a + base + so, g.Li, sl, rwi, 0, g.Li, 32, lane);
    }
    acc = warp_reduce<P>(acc);
    acc = ext_zero_fix_warp<P>(acc, a + base, g, lane);
    if (lane == 0) write_out<P>(out, o, acc, ro, a + base);
  }
}

// ROW with a CTA per (output, split). When `partial`, CTA (sx, o) reduces
// [sx*chunk, (sx+1)*chunk) of the single reduced dim into scratch[o*S + sx].
// At most 56 registers a thread: a split grid is exactly one wave of 4 CTAs
// per SM, and at 64 registers those 4 CTAs fill the register file, so any
// small kernel running beside it (a sharded reduction's record exchange on
// its side stream) pushed one CTA into a second wave.
template <class P>
__global__ void __maxnreg__(56) k_red_row_block(const typename P::In* __restrict__ a, void* out,
                                                                typename P::Acc* __restrict__ scratch, RedDev g,
                                                                RedOut ro, int64_t chunk, int vec, int partial) {
  pdl_enter();
  constexpr int VEC = 16 / sizeof(typename P::In) > 0 ? 16 / sizeof(typename P::In) : 1;
  const int S = gridDim.x;
  const int sx = blockIdx.x;
  const int64_t rwi = g.rw[g.R - 1];
  for (int64_t o = blockIdx.y; o < g.M; o += gridDim.y) {
    const int64_t base = kept_off(g, o);
    typename P::Acc acc = P::ident();
    if (!partial) {
      for (int64_t s = 0; s < g.Lo; ++s) {
        int64_t so, sl;
        seg_off(g, s, so, sl);
        if (vec)
          fold_segment_vec<P, VEC>(acc, a + base + so, g.Li, sl, rwi, threadIdx.x & 31, blockDim.x, threadIdx.x);
        else
          fold_segment_scalar<P>(acc, a + base + so, g.Li, sl, rwi, 0, g.Li, blockDim.x, threadIdx.x);
      }
    } else {
      const int64_t c0 = (int64_t)sx * chunk;
      int64_t c1 = c0 + chunk;
      if (c1 > g.Li) c1 = g.Li;
      if (c0 < c1) {
        if (vec)
          fold_segment_vec<P, VEC>(acc, a + base + c0, c1 - c0, c0 * rwi, rwi, threadIdx.x & 31, blockDim.x,
                                   threadIdx.x);
        else
          fold_segment_scalar<P>(acc, a + base, g.Li, 0, rwi, c0, c1, blockDim.x, threadIdx.x);
      }
    }
    acc = block_reduce<P>(acc);
    if (!partial && threadIdx.x < 32) acc = ext_zero_fix_warp<P>(acc, a + base, g, threadIdx.x);
    if (threadIdx.x == 0) {
      if (partial)
        scratch[o * S + sx] = acc;
      else
        write_out<P>(out, o, acc, ro, a + base);
    }
  }
}

// COL: one thread per output walks its reduced elements in index order; when
// `partial`, split sx covers [sx*chunk, (sx+1)*chunk) into scratch[sx*M + o].
template <class P>
__global__ void __launch_bounds__(kRedThreads) k_red_col(const typename P::In* __restrict__ a, void* out,
                                                          typename P::Acc* __restrict__ scratch, RedDev g,
                                                          RedOut ro, int64_t chunk, int partial) {
  pdl_enter();
  const int sx = blockIdx.y;
  const int64_t f0 = partial ? (int64_t)sx * chunk : 0;
  int64_t f1 = partial ? f0 + chunk : g.L;
  if (f1 > g.L) f1 = g.L;
  const int64_t gt = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t gs = (int64_t)gridDim.x * blockDim.x;
  for (int64_t o = gt; o < g.M; o += gs) {
    const int64_t base = kept_off(g, o);
    typename P::Acc acc = P::ident();
    if (g.R == 1) {
      // one reduced dim walked in increasing index order
      const int64_t st = g.rst[0], w = g.rw[0];
      constexpr int UNR = 16;
      int64_t f = f0;
      const typename P::In* ap = a + base + f0 * st;
      for (; f + UNR <= f1; f += UNR, ap += UNR * st) {
        typename P::In v[UNR];
#pragma unroll
        for (int u = 0; u < UNR; ++u) v[u] = ap[u * st];
#pragma unroll
        for (int u = 0; u < UNR; ++u) P::fold_seq(acc, v[u], (f + u) * w);
      }
      for (; f < f1; ++f, ap += st) P::fold_seq(acc, *ap, f * w);
    } else {
      int64_t c[kMaxCollapsed];
      int64_t rem = f0, off = 0, lidx = 0;
      for (int d = g.R - 1; d >= 0; --d) {
        c[d] = rem % g.rs[d];
        rem /= g.rs[d];
        off += c[d] * g.rst[d];
        lidx += c[d] * g.rw[d];
      }
      for (int64_t f = f0; f < f1; ++f) {
        P::fold(acc, a[base + off], lidx);
        for (int d = g.R - 1; d >= 0; --d) {
          ++c[d];
          off += g.rst[d];
          lidx += g.rw[d];
          if (c[d] < g.rs[d]) break;
          off -= c[d] * g.rst[d];
          lidx -= c[d] * g.rw[d];
          c[d] = 0;
        }
      }
    }
    if (partial)
      scratch[(int64_t)sx * g.M + o] = acc;
    else
      write_out<P>(out, o, ext_zero_fix_thread<P>(acc, a + base, g), ro, a + base);
  }
}

// COL with V adjacent outputs per thread (one reduced dim; the plan checks
// that every group of V outputs is contiguous and V * sizeof(In)-aligned at
// every reduced step): each step reads the V inputs as one 8- or 16-byte
// load, and each output folds its elements in index order exactly as
// k_red_col does. Fewer, wider loads and V times fewer threads: the argmax
// over axis 1 of (64, 4096, 4096) f32 takes 131,072 threads (2 outputs
// each), one partial wave with 16 MiB of loads in flight - no column split
// and no merge pass.
template <class P, int V>
__global__ void __launch_bounds__(kRedThreads, 4) k_red_col_v(const typename P::In* __restrict__ a, void* out,
                                                               typename P::Acc* __restrict__ scratch, RedDev g,
                                                               RedOut ro, int64_t chunk, int partial) {
  pdl_enter();
  using In = typename P::In;
  using Acc = typename P::Acc;
  constexpr int B = V * (int)sizeof(In);
  static_assert(B == 8 || B == 16, "8- or 16-byte loads");
  using W = typename std::conditional<B == 16, uint4, uint2>::type;
  constexpr int UNR = B == 16 ? 8 : 16;
  const int sx = blockIdx.y;
  const int64_t f0 = partial ? (int64_t)sx * chunk : 0;
  int64_t f1 = partial ? f0 + chunk : g.L;
  if (f1 > g.L) f1 = g.L;
  const int64_t groups = g.M / V;
  const int64_t st = g.rst[0], w = g.rw[0];
  const int64_t gt = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t gs = (int64_t)gridDim.x * blockDim.x;
  for (int64_t q = gt; q < groups; q += gs) {
    const int64_t o = q * V;
    const int64_t base = kept_off(g, o);
    Acc acc[V];
#pragma unroll
    for (int k = 0; k < V; ++k) acc[k] = P::ident();
    const In* ap = a + base + f0 * st;
    int64_t f = f0;
    for (; f + UNR <= f1; f += UNR, ap += UNR * st) {
      W v[UNR];
#pragma unroll
      for (int u = 0; u < UNR; ++u) v[u] = __ldcs(reinterpret_cast<const W*>(ap + u * st));
#pragma unroll
      for (int u = 0; u < UNR; ++u) {
        In e[V];
        memcpy(e, &v[u], B);
#pragma unroll
        for (int k = 0; k < V; ++k) P::fold_seq(acc[k], e[k], (f + u) * w);
      }
    }
    for (; f < f1; ++f, ap += st) {
      const W v = __ldcs(reinterpret_cast<const W*>(ap));
      In e[V];
      memcpy(e, &v, B);
#pragma unroll
      for (int k = 0; k < V; ++k) P::fold_seq(acc[k], e[k], f * w);
    }
#pragma unroll
    for (int k = 0; k < V; ++k) {
      if (partial)
        scratch[(int64_t)sx * g.M + o + k] = acc[k];
      else
        write_out<P>(out, o + k, ext_zero_fix_thread<P>(acc[k], a + base + k, g), ro, a + base + k);
    }
  }
}

constexpr int kCombineBatch = 8;

// Combine S partials per output. layout 0: [M][S] (row splits, a warp per
// output); layout 1: [S][M] (column splits, a thread per output); layout 2:
// [M][S] with a CTA per output (row splits have few outputs: each thread
// merges partials t, t + 256, ... - one round of loads for S <= 256 * k -
// then the block reduces; a warp needed three dependent rounds of loads for
// 592 partials). Every layout merges in a fixed order, so results do not
// depend on scheduling.
template <class P>
__global__ void __launch_bounds__(kRedThreads) k_red_combine(const typename P::In* __restrict__ a, void* out,
                                                              const typename P::Acc* __restrict__ part, RedDev g,
                                                              RedOut ro, int S, int layout) {
  pdl_enter();
  if (layout == 0) {
    const int lane = threadIdx.x & 31;
    const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t o = gw; o < g.M; o += nw) {
      typename P::Acc acc = P::ident();
      // kCombineBatch partials in flight per lane before they are merged, in
      // the same order as one at a time (the loads do not wait on the merges)
      for (int j0 = lane; j0 < S; j0 += 32 * kCombineBatch) {
        typename P::Acc v[kCombineBatch];
#pragma unroll
        for (int u = 0; u < kCombineBatch; ++u) {
          const int j = j0 + 32 * u;
          if (j < S) v[u] = part[o * S + j];
        }
#pragma unroll
        for (int u = 0; u < kCombineBatch; ++u)
          if (j0 + 32 * u < S) acc = P::merge(acc, v[u]);
      }
      acc = warp_reduce<P>(acc);
      const int64_t base = kept_off(g, o);
      acc = ext_zero_fix_warp<P>(acc, a + base, g, lane);
      if (lane == 0) write_out<P>(out, o, acc, ro, a + base);
    }
  } else if (layout == 2) {
    for (int64_t o = blockIdx.x; o < g.M; o += gridDim.x) {
      typename P::Acc acc = P::ident();
      for (int j = threadIdx.x; j < S; j += blockDim.x) acc = P::merge(acc, part[o * S + j]);
      acc = block_reduce<P>(acc);
      const int64_t base = kept_off(g, o);
      if (threadIdx.x < 32) acc = ext_zero_fix_warp<P>(acc, a + base, g, threadIdx.x);
      if (threadIdx.x == 0) write_out<P>(out, o, acc, ro, a + base);
    }
  } else {
    const int64_t gt = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t gs = (int64_t)gridDim.x * blockDim.x;
    for (int64_t o = gt; o < g.M; o += gs) {
      typename P::Acc acc = part[o];
      for (int j0 = 1; j0 < S; j0 += kCombineBatch) {
        typename P::Acc v[kCombineBatch];
#pragma unroll
        for (int u = 0; u < kCombineBatch; ++u)
          if (j0 + u < S) v[u] = part[(int64_t)(j0 + u) * g.M + o];
#pragma unroll
        for (int u = 0; u < kCombineBatch; ++u)
          if (j0 + u < S) acc = P::merge(acc, v[u]);
      }
      const int64_t base = kept_off(g, o);
      write_out<P>(out, o, ext_zero_fix_thread<P>(acc, a + base, g), ro, a + base);
    }
  }
}

// GEN: a warp per output with gathered loads.
template <class P>
__global__ void __launch_bounds__(kRedThreads) k_red_gen(const typename P::In* __restrict__ a, void* out, RedDev g,
                                                          RedOut ro) {
  pdl_enter();
  const int lane = threadIdx.x & 31;
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t o = gw; o < g.M; o += nw) {
    const int64_t base = kept_off(g, o);
    typename P::Acc acc = P::ident();
    for (int64_t f = lane; f < g.L; f += 32) {
      int64_t off, lidx;
      red_off(g, f, off, lidx);
      P::fold(acc, a[base + off], lidx);
    }
    acc = warp_reduce<P>(acc);
    acc = ext_zero_fix_warp<P>(acc, a + base, g, lane);
    if (lane == 0) write_out<P>(out, o, acc, ro, a + base);
  }
}

// ------------------------------------------------------------- launching
inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }
inline int blocks_for(int64_t items, int per_block, int cap_mult) {
  int64_t b = cdiv(items, per_block);
  const int64_t cap = (int64_t)sm_count() * cap_mult;
  if (b > cap) b = cap;
  if (b < 1) b = 1;
  return (int)b;
}

inline RedDev dev_of(const RedPlan& pl) {
  RedDev g;
  g.K = pl.K;
  g.R = pl.R;
  g.M = pl.M;
  g.L = pl.L;
  g.Li = pl.Li;
  g.Lo = pl.Lo;
  for (int d = 0; d < pl.K; ++d) {
    g.ks[d] = pl.ks[d];
    g.kst[d] = pl.kst[d];
  }
  for (int d = 0; d < pl.R; ++d) {
    g.rs[d] = pl.rs[d];
    g.rst[d] = pl.rst[d];
    g.rw[d] = pl.rw[d];
  }
  return g;
}

// k_red_col_v at the plan's vector width (only the widths whose loads are 8
// or 16 bytes of In are instantiated; the plan picks no other).
template <class P>
int launch_col_v(const typename P::In* a, void* out, typename P::Acc* scratch, const RedDev& g, RedOut ro,
                 const RedPlan& pl, int partial, cudaStream_t s) {
  constexpr int SZ = (int)sizeof(typename P::In);
  const int64_t groups = pl.M / pl.colv;
  dim3 grid(partial ? (unsigned)cdiv(groups, kRedThreads) : (unsigned)blocks_for(groups, kRedThreads, 64),
            partial ? (unsigned)pl.splits : 1u);
  const int64_t chunk = partial ? pl.chunk : 0;
  bool launched = false;
  cudaError_t e = cudaSuccess;
  if constexpr (SZ == 2) {
    if (pl.colv == 8) {
      e = launch_pdl(k_red_col_v<P, 8>, grid, dim3(kRedThreads), 0, s, a, out, scratch, g, ro, chunk, partial);
      launched = true;
    } else if (pl.colv == 4) {
      e = launch_pdl(k_red_col_v<P, 4>, grid, dim3(kRedThreads), 0, s, a, out, scratch, g, ro, chunk, partial);
      launched = true;
    }
  } else if constexpr (SZ == 4) {
    if (pl.colv == 4) {
      e = launch_pdl(k_red_col_v<P, 4>, grid, dim3(kRedThreads), 0, s, a, out, scratch, g, ro, chunk, partial);
      launched = true;
    } else if (pl.colv == 2) {
      e = launch_pdl(k_red_col_v<P, 2>, grid, dim3(kRedThreads), 0, s, a, out, scratch, g, ro, chunk, partial);
      launched = true;
    }
  } else if constexpr (SZ == 8) {
    if (pl.colv == 2) {
      e = launch_pdl(k_red_col_v<P, 2>, grid, dim3(kRedThreads), 0, s, a, out, scratch, g, ro, chunk, partial);
      launched = true;
    }
  }
  if (!launched)
    return fail(MPB_ERR_INVALID, "reduce: no column kernel for %d outputs of %d bytes per thread", pl.colv, SZ);
  return launch_check_pdl(e, partial ? "reduce_col_v_split" : "reduce_col_v");
}

template <class P>
int launch_policy(const RedReq& r, const RedPlan& pl, RedOut ro, cudaStream_t s) {
  using In = typename P::In;
  using Acc = typename P::Acc;
  const In* a = static_cast<const In*>(r.a);
  void* out = r.out;
  RedDev g = dev_of(pl);
  const size_t need = (pl.kind == RK_ROW_SPLIT || pl.kind == RK_COL_SPLIT)
                          ? (size_t)pl.M * (size_t)pl.splits * sizeof(Acc)
                          : 0;
  if (need > r.scratch_bytes || (need && !r.scratch))
    return fail(MPB_ERR_SCRATCH, "reduce: scratch of %zu bytes needed, %zu given", need, r.scratch_bytes);
  Acc* scratch = static_cast<Acc*>(r.scratch);
  const int vec = pl.vectorized ? 1 : 0;
  switch (pl.kind) {
    case RK_ROW_WARP:
      return launch_check_pdl(launch_pdl(k_red_row_warp<P>, dim3(blocks_for(pl.M * 32, kRedThreads, 32)),
                                         dim3(kRedThreads), 0, s, a, out, g, ro, vec),
                              "reduce_row_warp");
    case RK_ROW_BLOCK: {
      dim3 grid(1, (unsigned)(pl.M < 65535 ? pl.M : 65535));
      return launch_check_pdl(
          launch_pdl(k_red_row_block<P>, grid, dim3(kRedThreads), 0, s, a, out, scratch, g, ro, (int64_t)0, vec, 0),
          "reduce_row_block");
    }
    case RK_ROW_SPLIT: {
      dim3 grid((unsigned)pl.splits, (unsigned)(pl.M < 65535 ? pl.M : 65535));
      int rc = launch_check_pdl(
          launch_pdl(k_red_row_block<P>, grid, dim3(kRedThreads), 0, s, a, out, scratch, g, ro, pl.chunk, vec, 1),
          "reduce_row_split");
      if (rc) return rc;
      return launch_check_pdl(launch_pdl(k_red_combine<P>, dim3((unsigned)(pl.M < 65535 ? pl.M : 65535)),
                                         dim3(kRedThreads), 0, s, a, out, (const Acc*)scratch, g, ro, (int)pl.splits, 2),
                              "reduce_row_combine");
    }
    case RK_COL:
      if (pl.colv > 1) return launch_col_v<P>(a, out, scratch, g, ro, pl, 0, s);
      return launch_check_pdl(launch_pdl(k_red_col<P>, dim3(blocks_for(pl.M, kRedThreads, 64)), dim3(kRedThreads), 0,
                                         s, a, out, scratch, g, ro, (int64_t)0, 0),
                              "reduce_col");
    case RK_COL_SPLIT: {
      int rc;
      if (pl.colv > 1) {
        rc = launch_col_v<P>(a, out, scratch, g, ro, pl, 1, s);
      } else {
        dim3 grid((unsigned)cdiv(pl.M, kRedThreads), (unsigned)pl.splits);
        rc = launch_check_pdl(
            launch_pdl(k_red_col<P>, grid, dim3(kRedThreads), 0, s, a, out, scratch, g, ro, pl.chunk, 1),
            "reduce_col_split");
      }
      if (rc) return rc;
      return launch_check_pdl(launch_pdl(k_red_combine<P>, dim3(blocks_for(pl.M, kRedThreads, 64)),
                                         dim3(kRedThreads), 0, s, a, out, (const Acc*)scratch, g, ro, (int)pl.splits, 1),
                              "reduce_col_combine");
    }
    default:
      return launch_check_pdl(launch_pdl(k_red_gen<P>, dim3(blocks_for(pl.M * 32, kRedThreads, 32)),
                                         dim3(kRedThreads), 0, s, a, out, g, ro),
                              "reduce_gen");
  }
}

int run_sum(const RedReq& r, const RedPlan& pl, RedOut ro, cudaStream_t s);
int run_prod(const RedReq& r, const RedPlan& pl, RedOut ro, cudaStream_t s);
int run_arg(const RedReq& r, const RedPlan& pl, RedOut ro, bool is_max, cudaStream_t s);
int run_ext(const RedReq& r, const RedPlan& pl, RedOut ro, bool is_max, cudaStream_t s);

}  // namespace red
}  // namespace mpb
