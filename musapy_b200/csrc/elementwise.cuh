// Elementwise kernel family (binary arithmetic, comparison, unary math,
// clamp, cast / strided copy) for sm_100a.
//
// Replaces the nd / flat / vec4 / scalar-broadcast variants of
// kernels/elementwise.mu:35-573. Instead of one thread per element with a
// 64-bit div/mod per dim per operand (offset_nd, common.h:42-51), the host
// collapses dims and classifies the call:
//   EW_CONTIG  1-D streams: 16-byte vector loads/stores, 4 packs in flight
//              per thread, grid-stride over a grid sized to the SM count;
//   EW_ROWS    [outer..., inner] with every operand unit-stride or broadcast
//              along `inner`: the same vector packs, work items of one row
//              chunk so the row index math runs once per 1024 packs;
//   EW_TILED   an input whose unit stride lies on an outer dim (a transposed
//              view): 32x32 tiles staged through shared memory so that both
//              the read and the write are coalesced, cast fused on the way in;
//   EW_ND      anything else: warp-strided element order (every warp access
//              is one contiguous run when the layout allows) with magic-number
//              division per dim.
// Type promotion casts are fused into the loads: the kernel reads each input
// in its own dtype and converts in registers, so no temporary is written.
#pragma once
#include <type_traits>
#include "common.cuh"
#include "ops.cuh"
#include "plan.h"

namespace mpb {

constexpr int kEwThreads = 256;

// A pack of 16-byte words viewed as N elements of T.
template <class T, int N>
struct VPack {
  static constexpr int kWords = (N * (int)sizeof(T)) / 16;
  static_assert((N * (int)sizeof(T)) % 16 == 0, "pack must be whole 16-byte words");
  uint4 w[kWords];
  MPB_D T& operator[](int i) { return reinterpret_cast<T*>(w)[i]; }
  MPB_D const T& operator[](int i) const { return reinterpret_cast<const T*>(w)[i]; }
};
template <class T, int N, bool STREAM>
MPB_D void vload(VPack<T, N>& d, const T* p) {
#pragma unroll
  for (int i = 0; i < VPack<T, N>::kWords; ++i) {
    const char* q = reinterpret_cast<const char*>(p) + 16 * i;
    d.w[i] = STREAM ? ld_stream16(q) : ld_nc16(q);
  }
}
template <class T, int N>
MPB_D void vstore(T* p, const VPack<T, N>& s) {
#pragma unroll
  for (int i = 0; i < VPack<T, N>::kWords; ++i) st_stream16(reinterpret_cast<char*>(p) + 16 * i, s.w[i]);
}

// Unused second operand of unary ops.
struct NoArg {};

template <class Op, class TC, class TO, int NIN>
struct Apply {
  template <class TA, class TB>
  MPB_D static TO run(const Op& op, const TA& a, const TB& b) {
    if constexpr (NIN == 2) {
      return cvt<TO>(op(cvt<TC>(a), cvt<TC>(b)));
    } else {
      return cvt<TO>(op(cvt<TC>(a)));
    }
  }
};

template <class A, class B, class C>
constexpr int min_size3() {
  int m = (int)sizeof(A);
  if ((int)sizeof(B) < m) m = (int)sizeof(B);
  if ((int)sizeof(C) < m) m = (int)sizeof(C);
  return m;
}

// ------------------------------------------------------------- EW_CONTIG
template <class Op, class TC, class TA, class TB, class TO, int NIN>
__global__ void __launch_bounds__(kEwThreads) k_ew_contig(Op op, const TA* __restrict__ a,
                                                          const TB* __restrict__ b, TO* __restrict__ out,
                                                          int64_t n, int a_bc, int b_bc) {
  using TBv = typename std::conditional<NIN == 2, TB, TA>::type;
  constexpr int N = 16 / min_size3<TA, TBv, TO>();
  constexpr int UNR = 4;
  const int64_t nvec = n / N;
  const int64_t gtid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t gstride = (int64_t)gridDim.x * blockDim.x;
  const TA a0 = a_bc ? a[0] : TA{};
  TBv b0{};
  if constexpr (NIN == 2) {
    if (b_bc) b0 = b[0];
  }
  for (int64_t v = gtid; v < nvec; v += gstride * UNR) {
    VPack<TA, N> pa[UNR];
    VPack<TBv, N> pb[UNR];
#pragma unroll
    for (int u = 0; u < UNR; ++u) {
      const int64_t vi = v + u * gstride;
      if (vi < nvec) {
        if (!a_bc) vload<TA, N, true>(pa[u], a + vi * N);
        if constexpr (NIN == 2) {
          if (!b_bc) vload<TBv, N, true>(pb[u], reinterpret_cast<const TBv*>(b) + vi * N);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < UNR; ++u) {
      const int64_t vi = v + u * gstride;
      if (vi < nvec) {
        VPack<TO, N> po;
#pragma unroll
        for (int j = 0; j < N; ++j) {
          const TA av = a_bc ? a0 : pa[u][j];
          TBv bv{};
          if constexpr (NIN == 2) bv = b_bc ? b0 : pb[u][j];
          po[j] = Apply<Op, TC, TO, NIN>::run(op, av, bv);
        }
        vstore<TO, N>(out + vi * N, po);
      }
    }
  }
  const int64_t t = nvec * N + gtid;
  if (t < n) {
    const TA av = a_bc ? a0 : a[t];
    TBv bv{};
    if constexpr (NIN == 2) bv = b_bc ? b0 : b[t];
    out[t] = Apply<Op, TC, TO, NIN>::run(op, av, bv);
  }
}

// Geometry passed by value to the strided kernels.
struct NdArgs {
  int ndim;
  int pad;
  int64_t shape[kMaxCollapsed];
  FastDiv fd[kMaxCollapsed];
  int64_t sa[kMaxCollapsed];
  int64_t sb[kMaxCollapsed];
};

// --------------------------------------------------------------- EW_ROWS
// Rows of `inner` elements (inner % N == 0); operand inner stride is 0 or 1
// (a_bc/b_bc flag the broadcast ones); row r starts at sum(coord_d * s[d])
// over the outer dims, every unit-stride row start 16-byte aligned
// (host-checked). Work items are (row, chunk of kRowChunk packs): the row and
// its offsets are computed once per item, then each thread moves kRowUnr
// lane-strided packs (coalesced 16-byte accesses) with all loads in flight
// before the first store.
constexpr int kRowUnr = 4;
constexpr int kRowChunk = kEwThreads * kRowUnr;  // packs per work item

template <class Op, class TC, class TA, class TB, class TO, int NIN>
__global__ void __launch_bounds__(kEwThreads) k_ew_rows(Op op, const TA* __restrict__ a,
                                                        const TB* __restrict__ b, TO* __restrict__ out,
                                                        NdArgs g, int64_t nitems, int64_t cpr, FastDiv cpr_div,
                                                        int a_bc, int b_bc) {
  using TBv = typename std::conditional<NIN == 2, TB, TA>::type;
  constexpr int N = 16 / min_size3<TA, TBv, TO>();
  const int64_t inner = g.shape[g.ndim - 1];
  const int64_t spr = inner / N;  // packs per row
  for (int64_t item = blockIdx.x; item < nitems; item += gridDim.x) {
    int64_t row, chunk;
    if (nitems < 0xffffffffLL) {
      uint32_t q, r;
      cpr_div.divmod((uint32_t)item, q, r);
      row = q;
      chunk = r;
    } else {
      row = item / cpr;
      chunk = item - row * cpr;
    }
    int64_t oa = 0, ob = 0, rr = row;
    for (int d = g.ndim - 2; d > 0; --d) {
      const int64_t c = rr % g.shape[d];
      rr /= g.shape[d];
      oa += c * g.sa[d];
      ob += c * g.sb[d];
    }
    oa += rr * g.sa[0];
    ob += rr * g.sb[0];
    const TA* ar = a + oa;
    const TBv* br = reinterpret_cast<const TBv*>(b) + ob;
    TO* orow = out + row * inner;
    const int64_t p0 = chunk * kRowChunk + threadIdx.x;
    VPack<TA, N> pa[kRowUnr];
    VPack<TBv, N> pb[kRowUnr];
    TA as = TA{};
    TBv bs = TBv{};
    if (a_bc) as = ar[0];
    if constexpr (NIN == 2) {
      if (b_bc) bs = br[0];
    }
#pragma unroll
    for (int u = 0; u < kRowUnr; ++u) {
      const int64_t p = p0 + u * kEwThreads;
      if (p < spr) {
        if (!a_bc) vload<TA, N, true>(pa[u], ar + p * N);
        if constexpr (NIN == 2) {
          if (!b_bc) vload<TBv, N, false>(pb[u], br + p * N);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kRowUnr; ++u) {
      const int64_t p = p0 + u * kEwThreads;
      if (p < spr) {
        VPack<TO, N> po;
#pragma unroll
        for (int j = 0; j < N; ++j) {
          const TA av = a_bc ? as : pa[u][j];
          TBv bv{};
          if constexpr (NIN == 2) bv = b_bc ? bs : pb[u][j];
          po[j] = Apply<Op, TC, TO, NIN>::run(op, av, bv);
        }
        vstore<TO, N>(orow + p * N, po);
      }
    }
  }
}

// -------------------------------------------------------------- EW_TILED
// Input `a` has unit stride on dim p (an outer dim); the output is
// contiguous along q = ndim-1. A 32x32 tile of `a` is read along p,
// converted to TC and staged in shared memory, then written along q.
struct TiledArgs {
  int ndim;
  int p;
  int64_t dp, dq;
  int64_t nbatch;
  int nb;                        // number of batch dims
  int64_t bshape[kMaxCollapsed];
  int64_t bsa[kMaxCollapsed], bsb[kMaxCollapsed], bso[kMaxCollapsed];
  int64_t sa_q, sb_p, sb_q, so_p;
};

template <class Op, class TC, class TA, class TB, class TO, int NIN>
__global__ void __launch_bounds__(256) k_ew_tiled(Op op, const TA* __restrict__ a, const TB* __restrict__ b,
                                                  TO* __restrict__ out, TiledArgs t) {
  using TBv = typename std::conditional<NIN == 2, TB, TA>::type;
  __shared__ __align__(16) char tile_raw[32 * 33 * sizeof(TC)];
  TC(*tile)[33] = reinterpret_cast<TC(*)[33]>(tile_raw);
  const int tx = threadIdx.x & 31;
  const int ty = threadIdx.x >> 5;  // 0..7
  const int64_t q0 = (int64_t)blockIdx.x * 32;
  const int64_t p0 = (int64_t)blockIdx.y * 32;
  for (int64_t bi = blockIdx.z; bi < t.nbatch; bi += gridDim.z) {
    int64_t oa = 0, ob = 0, oo = 0;
    int64_t r = bi;
    for (int d = t.nb - 1; d >= 0; --d) {
      const int64_t c = r % t.bshape[d];
      r /= t.bshape[d];
      oa += c * t.bsa[d];
      ob += c * t.bsb[d];
      oo += c * t.bso[d];
    }
    // load a[p0+tx, q0+ty+8i] (coalesced along p)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t pp = p0 + tx, qq = q0 + ty + 8 * i;
      if (pp < t.dp && qq < t.dq) tile[ty + 8 * i][tx] = cvt<TC>(a[oa + pp + qq * t.sa_q]);
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t pp = p0 + ty + 8 * i, qq = q0 + tx;
      if (pp < t.dp && qq < t.dq) {
        const TC av = tile[tx][ty + 8 * i];
        if constexpr (NIN == 2) {
          const TBv bv = reinterpret_cast<const TBv*>(b)[ob + pp * t.sb_p + qq * t.sb_q];
          out[oo + pp * t.so_p + qq] = cvt<TO>(op(av, cvt<TC>(bv)));
        } else {
          out[oo + pp * t.so_p + qq] = cvt<TO>(op(av));
        }
      }
    }
    __syncthreads();
  }
}

// ----------------------------------------------------------------- EW_ND
constexpr int kNdEpt = 8;  // elements per thread per trip

template <class IdxT>
MPB_D void nd_offsets(const NdArgs& g, IdxT e, int64_t& oa, int64_t& ob) {
  oa = 0;
  ob = 0;
  for (int d = g.ndim - 1; d > 0; --d) {
    IdxT q, c;
    if constexpr (sizeof(IdxT) == 4) {
      uint32_t qq, cc;
      g.fd[d].divmod((uint32_t)e, qq, cc);
      q = qq;
      c = cc;
    } else {
      q = e / (IdxT)g.shape[d];
      c = e - q * (IdxT)g.shape[d];
    }
    oa += (int64_t)c * g.sa[d];
    ob += (int64_t)c * g.sb[d];
    e = q;
  }
  oa += (int64_t)e * g.sa[0];
  ob += (int64_t)e * g.sb[0];
}

template <class Op, class TC, class TA, class TB, class TO, int NIN, class IdxT>
__global__ void __launch_bounds__(kEwThreads) k_ew_nd(Op op, const TA* __restrict__ a, const TB* __restrict__ b,
                                                      TO* __restrict__ out, NdArgs g, IdxT n) {
  using TBv = typename std::conditional<NIN == 2, TB, TA>::type;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const IdxT per_block = (IdxT)kEwThreads * kNdEpt;
  for (IdxT base = (IdxT)blockIdx.x * per_block; base < n; base += (IdxT)gridDim.x * per_block) {
    const IdxT e0 = base + (IdxT)warp * (32 * kNdEpt) + lane;
    TA va[kNdEpt];
    TBv vb[kNdEpt];
#pragma unroll
    for (int j = 0; j < kNdEpt; ++j) {
      const IdxT e = e0 + (IdxT)j * 32;
      if (e < n) {
        int64_t oa, ob;
        nd_offsets<IdxT>(g, e, oa, ob);
        va[j] = a[oa];
        if constexpr (NIN == 2) vb[j] = reinterpret_cast<const TBv*>(b)[ob];
      }
    }
#pragma unroll
    for (int j = 0; j < kNdEpt; ++j) {
      const IdxT e = e0 + (IdxT)j * 32;
      if (e < n) out[e] = Apply<Op, TC, TO, NIN>::run(op, va[j], vb[j]);
    }
  }
}

// ------------------------------------------------------- generic (runtime dtypes)
// Loads convert from any storage dtype to TC; used for promotion pairs with
// no dedicated instantiation. Same access pattern as EW_ND.
template <class TC>
MPB_D TC load_as(const char* base, int64_t off, int dt) {
  switch (dt) {
    case MPB_BOOL: return cvt<TC>(reinterpret_cast<const boolean*>(base)[off]);
    case MPB_I8: return cvt<TC>(reinterpret_cast<const int8_t*>(base)[off]);
    case MPB_I16: return cvt<TC>(reinterpret_cast<const int16_t*>(base)[off]);
    case MPB_I32: return cvt<TC>(reinterpret_cast<const int32_t*>(base)[off]);
    case MPB_I64: return cvt<TC>(reinterpret_cast<const int64_t*>(base)[off]);
    case MPB_U8: return cvt<TC>(reinterpret_cast<const uint8_t*>(base)[off]);
    case MPB_U16: return cvt<TC>(reinterpret_cast<const uint16_t*>(base)[off]);
    case MPB_U32: return cvt<TC>(reinterpret_cast<const uint32_t*>(base)[off]);
    case MPB_U64: return cvt<TC>(reinterpret_cast<const uint64_t*>(base)[off]);
    case MPB_F16: return cvt<TC>(reinterpret_cast<const __half*>(base)[off]);
    case MPB_F32: return cvt<TC>(reinterpret_cast<const float*>(base)[off]);
    case MPB_F64: return cvt<TC>(reinterpret_cast<const double*>(base)[off]);
    case MPB_BF16: return cvt<TC>(reinterpret_cast<const __nv_bfloat16*>(base)[off]);
    case MPB_C64: return cvt<TC>(reinterpret_cast<const c64*>(base)[off]);
    default: return cvt<TC>(reinterpret_cast<const c128*>(base)[off]);
  }
}

template <class Op, class TC, class TO, int NIN, class IdxT>
__global__ void __launch_bounds__(kEwThreads) k_ew_generic(Op op, const char* __restrict__ a, int a_dt,
                                                           const char* __restrict__ b, int b_dt,
                                                           TO* __restrict__ out, NdArgs g, IdxT n) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const IdxT per_block = (IdxT)kEwThreads * kNdEpt;
  for (IdxT base = (IdxT)blockIdx.x * per_block; base < n; base += (IdxT)gridDim.x * per_block) {
    const IdxT e0 = base + (IdxT)warp * (32 * kNdEpt) + lane;
    TC va[kNdEpt], vb[kNdEpt];
#pragma unroll
    for (int j = 0; j < kNdEpt; ++j) {
      const IdxT e = e0 + (IdxT)j * 32;
      if (e < n) {
        int64_t oa, ob;
        nd_offsets<IdxT>(g, e, oa, ob);
        va[j] = load_as<TC>(a, oa, a_dt);
        if constexpr (NIN == 2) vb[j] = load_as<TC>(b, ob, b_dt);
      }
    }
#pragma unroll
    for (int j = 0; j < kNdEpt; ++j) {
      const IdxT e = e0 + (IdxT)j * 32;
      if (e < n) {
        if constexpr (NIN == 2) {
          out[e] = cvt<TO>(op(va[j], vb[j]));
        } else {
          out[e] = cvt<TO>(op(va[j]));
        }
      }
    }
  }
}

}  // namespace mpb
