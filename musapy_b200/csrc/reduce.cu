// Reduction engine: sum / prod / max / min / mean / argmax / argmin over any
// set of axes of any strided view, for sm_100a.
//
// Replaces the naive / small-axis / partial+mid+final kernel ladder of
// kernels/reduction.mu (:81-161, :504-555, :848-1336) and the host path
// choice in rust/musapy-ops/src/op_builder.rs:2513-3101. The host splits the
// dims into kept and reduced sets, collapses each, and picks:
//   ROW   innermost reduced dim is unit-stride: a warp (or a CTA, or several
//         CTAs with a second combine pass) per output, 16-byte vector loads;
//   COL   innermost kept dim is unit-stride: one thread per output walks the
//         reduced elements in index order, so a warp reads contiguous runs;
//         for a single axis this is the CPU path's exact summation order;
//   GEN   anything else: a warp per output with gathered loads.
//
// max/min/argmax/argmin follow the reference CPU rule (op_builder.rs:
// 3543-3578): strict comparisons with the first occurrence kept, and a NaN is
// only ever the answer when it is the first element. Every kernel tracks
// (value, index), breaks ties on the lower index, never lets a NaN win, and
// applies the first-element NaN rule when the output is written, so results
// are bit-identical to the sequential loop whatever the traversal order.
#include <math.h>
#include <stdint.h>
#include "common.cuh"
#include "internal.h"
#include "plan.h"
#include "reduce.h"
#include "reduce_kernels.cuh"

namespace mpb {

using red::cdiv;


// Build the kept/reduced split. Reduced dims are ordered by decreasing
// |stride| (the smallest innermost) and carry their logical C-order weight,
// so any traversal still reports the reference's flat index.
// Full and few-row reductions split each row into this many chunks per SM
// (one wave of the split kernel at 4 CTAs per SM).
#ifndef MPB_RED_SPLIT_PER_SM
#define MPB_RED_SPLIT_PER_SM 4
#endif

int red_plan(const RedReq& r, RedPlan& pl) {
  if (r.ndim < 0 || r.ndim > MPB_MAX_DIMS) return fail(MPB_ERR_INVALID, "reduce: ndim %d out of range", r.ndim);
  pl = RedPlan();
  const int esz = dtype_size(r.in_dt);
  int64_t kshape[MPB_MAX_DIMS], kst[MPB_MAX_DIMS];
  int64_t rshape[MPB_MAX_DIMS], rst[MPB_MAX_DIMS], rw[MPB_MAX_DIMS];
  int K = 0, R = 0;
  pl.M = 1;
  pl.L = 1;
  for (int d = 0; d < r.ndim; ++d) {
    const bool red = (r.axes_mask >> d) & 1ull;
    if (red) {
      pl.L *= r.shape[d];
      if (r.shape[d] != 1) {
        rshape[R] = r.shape[d];
        rst[R] = r.strides[d];
        ++R;
      }
    } else {
      pl.M *= r.shape[d];
      if (r.shape[d] != 1) {
        kshape[K] = r.shape[d];
        kst[K] = r.strides[d];
        ++K;
      }
    }
  }
  // logical weights (C order over the reduced dims as listed)
  {
    int64_t w = 1;
    for (int d = R - 1; d >= 0; --d) {
      rw[d] = w;
      w *= rshape[d];
    }
  }
  // order reduced dims by decreasing |stride| (stable insertion sort)
  for (int i = 1; i < R; ++i) {
    int j = i;
    while (j > 0 && llabs(rst[j - 1]) < llabs(rst[j])) {
      int64_t t;
      t = rst[j - 1]; rst[j - 1] = rst[j]; rst[j] = t;
      t = rshape[j - 1]; rshape[j - 1] = rshape[j]; rshape[j] = t;
      t = rw[j - 1]; rw[j - 1] = rw[j]; rw[j] = t;
      --j;
    }
  }
  // collapse kept dims (outer into inner when the strides line up)
  {
    int64_t sh[MPB_MAX_DIMS], st[MPB_MAX_DIMS];
    int n = 0;
    for (int d = 0; d < K; ++d) {
      if (n > 0 && st[n - 1] == kst[d] * kshape[d]) {
        sh[n - 1] *= kshape[d];
        st[n - 1] = kst[d];
      } else {
        sh[n] = kshape[d];
        st[n] = kst[d];
        ++n;
      }
    }
    K = n;
    for (int d = 0; d < K; ++d) {
      kshape[d] = sh[d];
      kst[d] = st[d];
    }
  }
  // collapse reduced dims (stride and logical weight both linear)
  {
    int64_t sh[MPB_MAX_DIMS], st[MPB_MAX_DIMS], ww[MPB_MAX_DIMS];
    int n = 0;
    for (int d = 0; d < R; ++d) {
      if (n > 0 && st[n - 1] == rst[d] * rshape[d] && ww[n - 1] == rw[d] * rshape[d]) {
        sh[n - 1] *= rshape[d];
        st[n - 1] = rst[d];
        ww[n - 1] = rw[d];
      } else {
        sh[n] = rshape[d];
        st[n] = rst[d];
        ww[n] = rw[d];
        ++n;
      }
    }
    R = n;
    for (int d = 0; d < R; ++d) {
      rshape[d] = sh[d];
      rst[d] = st[d];
      rw[d] = ww[d];
    }
  }
  if (K > kMaxCollapsed || R > kMaxCollapsed)
    return fail(MPB_ERR_SHAPE, "reduce: too many dims after collapsing (%d kept, %d reduced)", K, R);
  if (R == 0) {  // reducing only extent-1 dims: one element per output
    rshape[0] = 1;
    rst[0] = 1;
    rw[0] = 1;
    R = 1;
  }
  pl.K = K;
  pl.R = R;
  for (int d = 0; d < K; ++d) {
    pl.ks[d] = kshape[d];
    pl.kst[d] = kst[d];
  }
  for (int d = 0; d < R; ++d) {
    pl.rs[d] = rshape[d];
    pl.rst[d] = rst[d];
    pl.rw[d] = rw[d];
  }
  pl.Li = rshape[R - 1];
  pl.Lo = pl.L / (pl.Li > 0 ? pl.Li : 1);
  if (pl.M == 0 || pl.L == 0) {
    pl.kind = RK_EMPTY;
    return MPB_OK;
  }
  const int sms = sm_count();
  const bool row = rst[R - 1] == 1;
  const bool col = K > 0 && kst[K - 1] == 1;
  // vector width for ROW: 16 bytes of input
  pl.vec = esz > 0 && esz <= 16 ? 16 / esz : 1;
  bool vec_ok = row && (pl.Li % pl.vec == 0) && (((uintptr_t)r.a & 15) == 0);
  for (int d = 0; d < K && vec_ok; ++d)
    if ((kst[d] * esz) % 16 != 0) vec_ok = false;
  for (int d = 0; d < R - 1 && vec_ok; ++d)
    if ((rst[d] * esz) % 16 != 0) vec_ok = false;
  pl.vectorized = vec_ok;
  pl.splits = 1;
  if (row && pl.Li >= 32) {
    if (R == 1 && pl.M < 2 * sms && pl.L >= 65536) {
      pl.kind = RK_ROW_SPLIT;
      int64_t S = cdiv((int64_t)MPB_RED_SPLIT_PER_SM * sms, pl.M);
      int64_t max_s = pl.L / 16384;
      if (r.scratch_cap > 0 && max_s > (int64_t)(r.scratch_cap / (16 * (size_t)pl.M)))
        max_s = (int64_t)(r.scratch_cap / (16 * (size_t)pl.M));
      if (S > max_s) S = max_s;
      if (S < 1) S = 1;
      int64_t chunk = cdiv(pl.L, S);
      chunk = cdiv(chunk, 64) * 64;  // keep split starts 16-byte aligned for every dtype
      S = cdiv(pl.L, chunk);
      pl.splits = S;
      pl.chunk = chunk;
      if (S == 1) pl.kind = RK_ROW_BLOCK;
    } else if (pl.L >= 16384 || pl.M < (int64_t)sms * 8) {
      pl.kind = RK_ROW_BLOCK;
    } else {
      pl.kind = RK_ROW_WARP;
    }
  } else if (col || (row && pl.Li < 32)) {
    pl.kind = RK_COL;
    // V adjacent outputs per thread with one 8- or 16-byte load per reduced
    // step: one reduced dim, unit-stride kept inner dim, every V-group of
    // outputs contiguous and aligned at every step. Arg reductions of 2- and
    // 4-byte types take 8-byte loads: their fold (value, index, first-taken
    // test) is longer, and twice the threads hide it better (argmax over
    // axis 1 of (64, 4096, 4096) f32: 0.61 ms with 2 outputs per thread,
    // 0.72 ms with 4); the other reductions take 16-byte loads (sum over
    // axis 0: 0.624 ms with 4 per thread, 0.627 ms with 2).
    const bool arg = r.op == MPB_R_ARGMAX || r.op == MPB_R_ARGMIN || r.op == MPB_R_ARGMAX_REC ||
                     r.op == MPB_R_ARGMIN_REC;
    const int max_load = arg && esz <= 4 ? 8 : 16;
    if (R == 1 && col && esz >= 2 && esz <= 8) {
      for (int v = max_load / esz; v >= 2 && v * esz >= 8; v >>= 1) {
        bool ok = kshape[K - 1] % v == 0 && rst[0] % v == 0 && ((uintptr_t)r.a % (uintptr_t)(v * esz)) == 0;
        for (int d = 0; d < K - 1 && ok; ++d)
          if (kst[d] % v != 0) ok = false;
        if (ok) {
          pl.colv = v;
          break;
        }
      }
    }
    // Thread per output: a block of 256 outputs walks its whole chunk of the
    // reduced dim, so a block's time is proportional to the chunk length and
    // the pass takes ceil(w) "waves" of w = blocks * S / capacity. Splitting
    // the reduced dim into S chunks trades that wave quantisation (a grid of
    // 1.15 waves runs at 58%) against the combine pass, which moves 32 bytes
    // per (output, split). S minimises
    //   data_bytes * ceil(w) / w + 32 * M * S
    // with capacity = 6 blocks per SM (the column kernels use <= 40 registers)
    // and chunks of at least 64 elements.
    //
    // With V outputs per thread (k_red_col_v, 4 blocks per SM) a grid that
    // fits in one wave runs at full bandwidth as long as its loads in flight
    // (128 bytes per thread) cover the memory latency, so such a grid with
    // at least kColInflight bytes in flight is not split. Measured on the
    // argmax over axis 1 of (P, 4096, 4096) f32, unsplit: 16 MiB in flight
    // (P = 64) 1.09 of the copy peak, 8 MiB (P = 32) 0.83.
    const int64_t blocks = cdiv(cdiv(pl.M, pl.colv), 256);
    const double cap = (pl.colv > 1 ? 4.0 : 6.0) * sms;
    const double data = (double)pl.M * (double)pl.L * (double)esz;
    int64_t s_max = pl.L / 64;
    if (s_max > 4096) s_max = 4096;
    if (r.scratch_cap > 0 && s_max > (int64_t)(r.scratch_cap / (16 * (size_t)pl.M)))
      s_max = (int64_t)(r.scratch_cap / (16 * (size_t)pl.M));
    constexpr double kColInflight = 16.0 * 1024 * 1024;
    if (pl.colv > 1 && (double)blocks <= cap && (double)(pl.M / pl.colv) * 128.0 >= kColInflight) s_max = 1;
    int64_t best_s = 1;
    double best_cost = 0.0;
    for (int64_t S = 1; S <= (s_max > 1 ? s_max : 1); ++S) {
      const double w = (double)(blocks * S) / cap;
      const double cost = data * ceil(w) / w + (S > 1 ? 32.0 * (double)pl.M * (double)S : 0.0);
      if (S == 1 || cost < best_cost) {
        best_cost = cost;
        best_s = S;
      }
    }
    if (best_s > 1) {
      pl.kind = RK_COL_SPLIT;
      pl.chunk = cdiv(pl.L, best_s);
      pl.splits = cdiv(pl.L, pl.chunk);
    }
  } else {
    pl.kind = RK_GEN;
  }
  if (!r.allow_split) {
    if (pl.kind == RK_ROW_SPLIT) pl.kind = RK_ROW_BLOCK;
    if (pl.kind == RK_COL_SPLIT) pl.kind = RK_COL;
    pl.splits = 1;
  }
  return MPB_OK;
}

size_t red_scratch_bytes(const RedReq& r) {
  RedPlan pl;
  if (red_plan(r, pl) != MPB_OK) return 0;
  if (pl.kind != RK_ROW_SPLIT && pl.kind != RK_COL_SPLIT) return 0;
  // the largest accumulator is ArgAcc<double> / c128: 16 bytes
  return (size_t)pl.M * (size_t)pl.splits * 16;
}

int red_run(const RedReq& r, cudaStream_t s) {
  RedPlan pl;
  int rc = red_plan(r, pl);
  if (rc) return rc;
  if (pl.kind == RK_EMPTY) return MPB_OK;  // the host layer fills empty reductions
  if (!r.a || !r.out) return fail(MPB_ERR_INVALID, "reduce: null pointer");
  red::RedOut ro;
  ro.count = pl.L;
  ro.nan_rule = r.nan_first_rule;
  ro.out_dt = r.out_dt;
  ro.pad = 0;
  ro.ostride = r.out_stride > 1 ? r.out_stride : 1;
  switch (r.op) {
    case MPB_R_SUM: ro.mode = 0; return red::run_sum(r, pl, ro, s);
    case MPB_R_MEAN: ro.mode = 1; return red::run_sum(r, pl, ro, s);
    case MPB_R_PROD: ro.mode = 0; return red::run_prod(r, pl, ro, s);
    case MPB_R_MAX: ro.mode = 2; return red::run_ext(r, pl, ro, true, s);
    case MPB_R_MIN: ro.mode = 2; return red::run_ext(r, pl, ro, false, s);
    case MPB_R_ARGMAX: ro.mode = 3; return red::run_arg(r, pl, ro, true, s);
    case MPB_R_ARGMIN: ro.mode = 3; return red::run_arg(r, pl, ro, false, s);
    case MPB_R_ARGMAX_REC: ro.mode = 4; return red::run_arg(r, pl, ro, true, s);
    case MPB_R_ARGMIN_REC: ro.mode = 4; return red::run_arg(r, pl, ro, false, s);
    default: return fail(MPB_ERR_INVALID, "reduce: unknown op %d", r.op);
  }
}

}  // namespace mpb
