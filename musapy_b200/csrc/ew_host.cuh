// Host-side planning and launch templates of the elementwise engine, shared
// by the per-family translation units (ew_arith.cu, ew_cmp.cu, ew_unary.cu,
// ew_cast.cu) so each compiles its own instantiations in parallel.
#pragma once
#include <stdarg.h>
#include <stdio.h>
#include "elementwise.cuh"
#include "internal.h"
#include "tiled_tma.cuh"

namespace mpb {
namespace ew {

template <class Op>
struct Swapped {
  Op op;
  template <class T>
  MPB_D auto operator()(T x, T y) const {
    return op(y, x);
  }
};

inline bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }
inline bool aligned_to(const void* p, int bytes) { return ((uintptr_t)p % (uintptr_t)bytes) == 0; }
inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }
// Streaming kernels loop over their work with a grid of up to 64 blocks per
// SM: on the 16 GB broadcast add of the benchmark, 64 per SM ran 4% faster
// than 16 (2.57 vs 2.68 ms) through finer load balance at the end.
constexpr int kStreamBlocksPerSm = 64;
inline int grid_for(int64_t work_items, int per_block) {
  int64_t blocks = cdiv(work_items, per_block);
  const int64_t cap = (int64_t)sm_count() * kStreamBlocksPerSm;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return (int)blocks;
}

struct Plan {
  Geometry g;
  int kind = EW_ND;
  int a_bc = 0, b_bc = 0;
  int tiled_op = 0, tiled_p = 0;
};

template <class TA, class TB, class TO, int NIN, bool ALLOW_TILED>
Plan make_plan(const EwReq& r) {
  using TBv = typename std::conditional<NIN == 2, TB, TA>::type;
  constexpr int N = ew_pack<TA, TBv, TO>();
  Plan pl;
  int64_t out_st[MPB_MAX_DIMS];
  int64_t acc = 1;
  for (int i = r.ndim - 1; i >= 0; --i) {
    out_st[i] = acc;
    acc *= r.shape[i];
  }
  const int64_t* sts[3] = {r.a_st, NIN == 2 ? r.b_st : out_st, out_st};
  pl.g = collapse(r.ndim, r.shape, NIN + 1, sts);
  const Geometry& g = pl.g;
  const int k = g.ndim;
  const int oo = NIN;  // output operand index
  const int64_t sa_in = g.st[0][k - 1];
  const int64_t sb_in = NIN == 2 ? g.st[1][k - 1] : 0;
  const bool a_unit_or_bc = (sa_in == 0 || sa_in == 1);
  const bool b_unit_or_bc = NIN == 1 || (sb_in == 0 || sb_in == 1);
  pl.a_bc = (sa_in == 0);
  pl.b_bc = NIN == 2 && (sb_in == 0);
  // input packs are N elements: whole 16-byte words, or one narrower word
  const int a_align = N * (int)sizeof(TA) < 16 ? N * (int)sizeof(TA) : 16;
  const int b_align = N * (int)sizeof(TBv) < 16 ? N * (int)sizeof(TBv) : 16;
  if (k == 1) {
    if (a_unit_or_bc && b_unit_or_bc && aligned16(r.out) && (pl.a_bc || aligned_to(r.a, a_align)) &&
        (NIN == 1 || pl.b_bc || aligned_to(r.b, b_align))) {
      pl.kind = EW_CONTIG;
      return pl;
    }
    pl.kind = EW_ND;
    return pl;
  }
  // EW_ROWS: every input unit-stride or broadcast along the inner dim, with
  // pack-aligned row starts for the unit-stride ones.
  if (g.shape[k - 1] % N == 0 && a_unit_or_bc && b_unit_or_bc && aligned16(r.out)) {
    bool ok = true;
    for (int x = 0; x < NIN && ok; ++x) {
      const void* base = x == 0 ? r.a : r.b;
      const int esz = x == 0 ? (int)sizeof(TA) : (int)sizeof(TBv);
      const int align = x == 0 ? a_align : b_align;
      if (g.st[x][k - 1] == 1) {
        if (!aligned_to(base, align)) ok = false;
        for (int d = 0; d < k - 1 && ok; ++d)
          if (((g.st[x][d] * esz) % align) != 0) ok = false;
      }
    }
    (void)oo;
    if (ok && (g.numel / N) > 0) {
      pl.kind = EW_ROWS;
      return pl;
    }
  }
  // EW_TILED: an input with unit stride on an outer dim and a non-unit,
  // non-broadcast inner stride (a transposed view).
  for (int x = 0; x < NIN && ALLOW_TILED; ++x) {
    const int64_t in_st = g.st[x][k - 1];
    if (in_st == 0 || in_st == 1 || g.shape[k - 1] < 8) continue;
    for (int p = k - 2; p >= 0; --p) {
      if (g.st[x][p] == 1 && g.shape[p] >= 8 && cdiv(g.shape[p], 32) <= 65535) {
        pl.kind = EW_TILED;
        pl.tiled_op = x;
        pl.tiled_p = p;
        return pl;
      }
    }
  }
  pl.kind = EW_ND;
  return pl;
}

inline NdArgs nd_args(const Geometry& g, int nin) {
  NdArgs a;
  a.ndim = g.ndim;
  a.pad = 0;
  for (int d = 0; d < g.ndim; ++d) {
    a.shape[d] = g.shape[d];
    a.fd[d] = FastDiv((uint32_t)(g.shape[d] < 0xffffffffLL ? g.shape[d] : 1));
    a.sa[d] = g.st[0][d];
    a.sb[d] = nin == 2 ? g.st[1][d] : 0;
  }
  return a;
}

inline TiledArgs tiled_args(const Geometry& g, int nin, int tx_op, int p) {
  TiledArgs t;
  const int k = g.ndim, q = k - 1;
  const int other = nin == 2 ? 1 - tx_op : -1;
  const int oo = nin;
  t.ndim = k;
  t.p = p;
  t.dp = g.shape[p];
  t.dq = g.shape[q];
  t.nb = 0;
  t.nbatch = 1;
  for (int d = 0; d < k; ++d) {
    if (d == p || d == q) continue;
    t.bshape[t.nb] = g.shape[d];
    t.bsa[t.nb] = g.st[tx_op][d];
    t.bsb[t.nb] = other >= 0 ? g.st[other][d] : 0;
    t.bso[t.nb] = g.st[oo][d];
    t.nbatch *= g.shape[d];
    ++t.nb;
  }
  t.sa_q = g.st[tx_op][q];
  t.sb_p = other >= 0 ? g.st[other][p] : 0;
  t.sb_q = other >= 0 ? g.st[other][q] : 0;
  t.so_p = g.st[oo][p];
  return t;
}

// Grid for a kernel whose blocks loop over `items` work items: exactly the
// blocks that fit on the GPU at once (256 threads each), so no block starts
// its share after the others have finished theirs.
int blocks_per_sm_cached(const void* kernel, int threads);  // elementwise.cu

template <class K>
unsigned resident_grid(K kernel, int64_t items) {
  const int per_sm = blocks_per_sm_cached(reinterpret_cast<const void*>(kernel), 256);
  int64_t blocks = (int64_t)sm_count() * per_sm;
  if (blocks > items) blocks = items;
  return (unsigned)(blocks < 1 ? 1 : blocks);
}

// TMA form with the second operand as the transposed one.
template <class Op, class TC, class TA, class TB, class TO, int NIN>
int run_tiled_tma_swapped(const Op& op, const TA* a, const TB* b, TO* out, const TiledArgs& t, cudaStream_t s) {
  if constexpr (NIN == 2) {
    return run_tiled_tma<Swapped<Op>, TC, TB, TA, TO, 2>(Swapped<Op>{op}, b, a, out, t, s);
  } else {
    return -1;
  }
}

// Tile counts for an edge of `edge` elements.
inline void tiled_count(TiledArgs& t, int edge) {
  t.ntp = cdiv(t.dp, edge);
  t.ntq = cdiv(t.dq, edge);
  t.ntiles = t.ntp * t.ntq * t.nbatch;
  t.fd_ntq = FastDiv((uint32_t)(t.ntq < 0xffffffffLL ? t.ntq : 1));
  t.fd_ntp = FastDiv((uint32_t)(t.ntp < 0xffffffffLL ? t.ntp : 1));
}

template <class Op, class TC, class TA, class TB, class TO, int NIN, bool ALLOW_TILED = false>
int run_typed(const Op& op, const EwReq& r, cudaStream_t s) {
  using TBv = typename std::conditional<NIN == 2, TB, TA>::type;
  constexpr int N = ew_pack<TA, TBv, TO>();
  Plan pl = make_plan<TA, TB, TO, NIN, ALLOW_TILED>(r);
  const Geometry& g = pl.g;
  if (g.numel == 0) return MPB_OK;
  if (g.ndim > kMaxCollapsed) return fail(MPB_ERR_SHAPE, "elementwise: %d dims remain after collapsing (max %d)", g.ndim, kMaxCollapsed);
  const TA* a = static_cast<const TA*>(r.a);
  const TB* b = static_cast<const TB*>(r.b);
  TO* out = static_cast<TO*>(r.out);
  switch (pl.kind) {
    case EW_CONTIG: {
      const int64_t nvec = g.numel / N;
      const cudaError_t e = launch_pdl(k_ew_contig<Op, TC, TA, TB, TO, NIN>, dim3(grid_for(nvec, kEwThreads * 4)),
                                       dim3(kEwThreads), 0, s, op, a, b, out, g.numel, pl.a_bc, pl.b_bc);
      return launch_check_pdl(e, "ew_contig");
    }
    case EW_ROWS: {
      NdArgs na = nd_args(g, NIN);
      const int64_t spr = g.shape[g.ndim - 1] / N;
      const int64_t rows = g.numel / g.shape[g.ndim - 1];
      const int64_t cpr = cdiv(spr, kRowChunk);
      const int64_t nitems = rows * cpr;
      int64_t blocks = nitems;
      const int64_t cap = (int64_t)sm_count() * kStreamBlocksPerSm;
      if (blocks > cap) blocks = cap;
      const cudaError_t e = launch_pdl(k_ew_rows<Op, TC, TA, TB, TO, NIN>, dim3((unsigned)(blocks < 1 ? 1 : blocks)),
                                       dim3(kEwThreads), 0, s, op, a, b, out, na, nitems, cpr,
                                       FastDiv((uint32_t)(cpr < 0xffffffffLL ? cpr : 1)), pl.a_bc, pl.b_bc);
      return launch_check_pdl(e, "ew_rows");
    }
    case EW_TILED: {
      if constexpr (ALLOW_TILED) {
        TiledArgs t = tiled_args(g, NIN, pl.tiled_op, pl.tiled_p);
        {
          const int rc = pl.tiled_op == 0 ? run_tiled_tma<Op, TC, TA, TB, TO, NIN>(op, a, b, out, t, s)
                                          : run_tiled_tma_swapped<Op, TC, TA, TB, TO, NIN>(op, a, b, out, t, s);
          if (rc >= 0) return rc;
        }
        tiled_count(t, tiled_edge<TC>());
        if (pl.tiled_op == 0) {
          auto k = k_ew_tiled<Op, TC, TA, TB, TO, NIN>;
          k<<<resident_grid(k, t.ntiles), 256, 0, s>>>(op, a, b, out, t);
        } else {
          if constexpr (NIN == 2) {
            auto k = k_ew_tiled<Swapped<Op>, TC, TB, TA, TO, 2>;
            k<<<resident_grid(k, t.ntiles), 256, 0, s>>>(Swapped<Op>{op}, b, a, out, t);
          }
        }
        return launch_check("ew_tiled");
      }
      return fail(MPB_ERR_INVALID, "elementwise: tiled plan without tiled instantiation");
    }
    default: {
      NdArgs na = nd_args(g, NIN);
      if (g.numel < 0xffffffffLL) {
        k_ew_nd<Op, TC, TA, TB, TO, NIN, uint32_t><<<grid_for(g.numel, kEwThreads * kNdEpt), kEwThreads, 0, s>>>(
            op, a, b, out, na, (uint32_t)g.numel);
      } else {
        k_ew_nd<Op, TC, TA, TB, TO, NIN, uint64_t><<<grid_for(g.numel, kEwThreads * kNdEpt), kEwThreads, 0, s>>>(
            op, a, b, out, na, (uint64_t)g.numel);
      }
      return launch_check("ew_nd");
    }
  }
}

template <class Op, class TC, class TO, int NIN>
int run_generic(const Op& op, const EwReq& r, cudaStream_t s) {
  int64_t out_st[MPB_MAX_DIMS];
  int64_t acc = 1;
  for (int i = r.ndim - 1; i >= 0; --i) {
    out_st[i] = acc;
    acc *= r.shape[i];
  }
  const int64_t* sts[3] = {r.a_st, NIN == 2 ? r.b_st : out_st, out_st};
  Geometry g = collapse(r.ndim, r.shape, NIN + 1, sts);
  if (g.numel == 0) return MPB_OK;
  if (g.ndim > kMaxCollapsed) return fail(MPB_ERR_SHAPE, "elementwise: %d dims remain after collapsing (max %d)", g.ndim, kMaxCollapsed);
  NdArgs na = nd_args(g, NIN);
  const char* a = static_cast<const char*>(r.a);
  const char* b = static_cast<const char*>(r.b);
  TO* out = static_cast<TO*>(r.out);
  if (g.numel < 0xffffffffLL) {
    k_ew_generic<Op, TC, TO, NIN, uint32_t><<<grid_for(g.numel, kEwThreads * kNdEpt), kEwThreads, 0, s>>>(
        op, a, r.a_dt, b, r.b_dt, out, na, (uint32_t)g.numel);
  } else {
    k_ew_generic<Op, TC, TO, NIN, uint64_t><<<grid_for(g.numel, kEwThreads * kNdEpt), kEwThreads, 0, s>>>(
        op, a, r.a_dt, b, r.b_dt, out, na, (uint64_t)g.numel);
  }
  return launch_check("ew_generic");
}

}  // namespace ew
}  // namespace mpb
