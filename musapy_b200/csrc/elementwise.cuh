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

// A pack of N elements of T moved by vector accesses: 16-byte words, or one
// narrower word (8/4/2/1 bytes) for an input narrower than the output.
template <int BYTES> struct PackWord { using type = uint4; };
template <> struct PackWord<8> { using type = uint2; };
template <> struct PackWord<4> { using type = unsigned int; };
template <> struct PackWord<2> { using type = unsigned short; };
template <> struct PackWord<1> { using type = unsigned char; };

template <class T, int N>
struct VPack {
  static constexpr int kBytes = N * (int)sizeof(T);
  static constexpr int kWordBytes = kBytes >= 16 ? 16 : kBytes;
  static constexpr int kWords = kBytes / kWordBytes;
  static_assert(kBytes % kWordBytes == 0, "pack must be whole words");
  using W = typename PackWord<kWordBytes>::type;
  W w[kWords];
  MPB_D T& operator[](int i) { return reinterpret_cast<T*>(w)[i]; }
  MPB_D const T& operator[](int i) const { return reinterpret_cast<const T*>(w)[i]; }
};
template <class T, int N, bool STREAM>
MPB_D void vload(VPack<T, N>& d, const T* p) {
  using P = VPack<T, N>;
#pragma unroll
  for (int i = 0; i < P::kWords; ++i) {
    const char* q = reinterpret_cast<const char*>(p) + P::kWordBytes * i;
    if constexpr (P::kWordBytes == 16) {
      d.w[i] = STREAM ? ld_stream16(q) : ld_nc16(q);
    } else {
      const typename P::W* qw = reinterpret_cast<const typename P::W*>(q);
      d.w[i] = STREAM ? __ldcs(qw) : __ldg(qw);
    }
  }
}
// Output packs are always whole 16-byte words (ew_pack below).
template <class T, int N>
MPB_D void vstore(T* p, const VPack<T, N>& s) {
  static_assert(VPack<T, N>::kWordBytes == 16, "output packs are 16-byte words");
#pragma unroll
  for (int i = 0; i < VPack<T, N>::kWords; ++i) st_stream16(reinterpret_cast<char*>(p) + 16 * i, s.w[i]);
}

// Elements per pack: one 16-byte word of output. Every thread's store is then
// one 16-byte access, and a warp's stores cover whole 32-byte sectors; an input
// wider than the output takes several words per pack, a narrower one a
// narrower word (writing two words 32 bytes apart per thread instead left half
// sectors to be merged in L2 and cost about a quarter of the bandwidth).
template <class TA, class TB, class TO>
constexpr int ew_pack() {
  return 16 / (int)sizeof(TO) > 0 ? 16 / (int)sizeof(TO) : 1;
}

// Unused second operand of unary ops.
struct NoArg {};

template <class Op, class = void>
struct IsPaired : std::false_type {};
template <class Op>
struct IsPaired<Op, std::void_t<decltype(Op::kPaired)>> : std::bool_constant<Op::kPaired> {};
// Paired ops whose fast path can run on every pair, with a range test for a
// fix-up afterwards (pair_fast / pair_ok).
template <class Op, class = void>
struct HasFastPair : std::false_type {};
template <class Op>
struct HasFastPair<Op, std::void_t<decltype(std::declval<const Op&>().pair_ok(float2{}))>> : std::true_type {};
// Ops with much arithmetic per element (transcendentals, pow).
template <class Op, class = void>
struct IsHeavy : IsPaired<Op> {};
template <class Op>
struct IsHeavy<Op, std::void_t<decltype(Op::kHeavy)>> : std::bool_constant<Op::kHeavy> {};

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
  // Unary float ops with a two-element form (packed f32x2 arithmetic).
  static constexpr bool kPair = NIN == 1 && IsPaired<Op>::value && std::is_same<TC, float>::value;
  template <class TA>
  MPB_D static void run2(const Op& op, const TA& a0, const TA& a1, TO& o0, TO& o1) {
    const float2 r = op.pair(make_float2(cvt<float>(a0), cvt<float>(a1)));
    o0 = cvt<TO>(r.x);
    o1 = cvt<TO>(r.y);
  }
};

// Applies the op to one pack: pairs for ops that have a two-element form.
template <class Op, class TC, class TO, int NIN, class TA, class TBv, int N>
MPB_D void apply_pack(const Op& op, const VPack<TA, N>& pa, const VPack<TBv, N>& pb, bool a_bc, bool b_bc,
                      const TA& as, const TBv& bs, VPack<TO, N>& po) {
  using AP = Apply<Op, TC, TO, NIN>;
  if constexpr (AP::kPair && N % 2 == 0) {
#pragma unroll
    for (int j = 0; j < N; j += 2) {
      AP::run2(op, a_bc ? as : pa[j], a_bc ? as : pa[j + 1], po[j], po[j + 1]);
    }
  } else {
#pragma unroll
    for (int j = 0; j < N; ++j) {
      const TA av = a_bc ? as : pa[j];
      TBv bv{};
      if constexpr (NIN == 2) bv = b_bc ? bs : pb[j];
      po[j] = AP::run(op, av, bv);
    }
  }
}

// ------------------------------------------------------------- EW_CONTIG
// The loop is instantiated without broadcast operands (the common case, no
// per-element selects) and with them, and with 32-bit indices when the
// length allows (64-bit index arithmetic costs several instructions per
// pack). The lanes of a warp run the loop's trips together (the warp's first
// lane decides), so a warp-wide vote inside a trip is safe: unary ops with a
// fast paired path run it on every pair and fix the rare out-of-range
// elements up after one vote, instead of a branch per pair.
template <bool BC, class Op, class TC, class TA, class TB, class TO, int NIN, class IdxT>
MPB_D void contig_loop(const Op& op, const TA* __restrict__ a, const TB* __restrict__ b, TO* __restrict__ out,
                       IdxT n, int a_bc_in, int b_bc_in) {
  using TBv = typename std::conditional<NIN == 2, TB, TA>::type;
  using AP = Apply<Op, TC, TO, NIN>;
  constexpr int N = ew_pack<TA, TBv, TO>();
  constexpr int UNR = 4;
#ifndef MPB_EW_NO_VOTE
  constexpr bool kVote = AP::kPair && HasFastPair<Op>::value && N % 2 == 0 && !BC;
#else
  constexpr bool kVote = false;
#endif
  const bool a_bc = BC && a_bc_in;
  const bool b_bc = BC && b_bc_in;
  const IdxT nvec = n / N;
  const IdxT lane = threadIdx.x & 31;
  const IdxT gtid = (IdxT)blockIdx.x * blockDim.x + threadIdx.x;
  const IdxT gstride = (IdxT)gridDim.x * blockDim.x;
  const TA a0 = a_bc ? a[0] : TA{};
  TBv b0{};
  if constexpr (NIN == 2) {
    if (b_bc) b0 = b[0];
  }
  if constexpr (kVote) {
    // Arithmetic-heavy ops: the next trip's packs are loaded before this
    // trip's are computed, so the loads stay in flight through the compute
    // (otherwise a warp has no loads outstanding while it computes).
    VPack<TA, N> pa[UNR], pn[UNR];
    auto load_trip = [&](IdxT v, VPack<TA, N>(&dst)[UNR]) {
#pragma unroll
      for (int u = 0; u < UNR; ++u) {
        const IdxT vi = v + u * gstride;
        if (vi < nvec) vload<TA, N, true>(dst[u], a + vi * N);
      }
    };
#ifndef MPB_EW_NO_PREFETCH
    load_trip(gtid, pn);
#endif
    for (IdxT v = gtid; v - lane < nvec; v += gstride * UNR) {
#ifndef MPB_EW_NO_PREFETCH
#pragma unroll
      for (int u = 0; u < UNR; ++u) pa[u] = pn[u];
      if (v + gstride * UNR - lane < nvec) load_trip(v + gstride * UNR, pn);
#else
      load_trip(v, pa);
#endif
      bool ok = true;
#pragma unroll
      for (int u = 0; u < UNR; ++u) {
        const IdxT vi = v + u * gstride;
        if (vi < nvec) {
          VPack<TO, N> po;
#pragma unroll
          for (int j = 0; j < N; j += 2) {
            const float2 x = make_float2(cvt<float>(pa[u][j]), cvt<float>(pa[u][j + 1]));
            const float2 r = op.pair_fast(x);
            ok = ok && op.pair_ok(x);
            po[j] = cvt<TO>(r.x);
            po[j + 1] = cvt<TO>(r.y);
          }
          vstore<TO, N>(out + vi * N, po);
        }
      }
      if (!__all_sync(0xffffffffu, ok)) {
        // rare: an argument outside the fast range; its pair is redone by
        // the full form and rewritten by this same thread
#pragma unroll
        for (int u = 0; u < UNR; ++u) {
          const IdxT vi = v + u * gstride;
          if (vi < nvec) {
#pragma unroll
            for (int j = 0; j < N; j += 2) {
              const float2 x = make_float2(cvt<float>(pa[u][j]), cvt<float>(pa[u][j + 1]));
              if (!op.pair_ok(x)) {
                const float2 r = op.pair(x);
                out[vi * N + j] = cvt<TO>(r.x);
                out[vi * N + j + 1] = cvt<TO>(r.y);
              }
            }
          }
        }
      }
    }
  } else {
    for (IdxT v = gtid; v - lane < nvec; v += gstride * UNR) {
      VPack<TA, N> pa[UNR];
      VPack<TBv, N> pb[UNR];
#pragma unroll
      for (int u = 0; u < UNR; ++u) {
        const IdxT vi = v + u * gstride;
        if (vi < nvec) {
          if (!a_bc) vload<TA, N, true>(pa[u], a + vi * N);
          if constexpr (NIN == 2) {
            if (!b_bc) vload<TBv, N, true>(pb[u], reinterpret_cast<const TBv*>(b) + vi * N);
          }
        }
      }
#pragma unroll
      for (int u = 0; u < UNR; ++u) {
        const IdxT vi = v + u * gstride;
        if (vi < nvec) {
          VPack<TO, N> po;
          apply_pack<Op, TC, TO, NIN>(op, pa[u], pb[u], a_bc, b_bc, a0, b0, po);
          vstore<TO, N>(out + vi * N, po);
        }
      }
    }
  }
  const IdxT t = nvec * N + gtid;
  if (t < n) {
    const TA av = a_bc ? a0 : a[t];
    TBv bv{};
    if constexpr (NIN == 2) bv = b_bc ? b0 : b[t];
    out[t] = Apply<Op, TC, TO, NIN>::run(op, av, bv);
  }
}

// Blocks per SM the register allocation must allow (4 caps a thread at 64
// registers). Left to itself the compiler unrolls the grid-stride loop into
// 90-120 registers, 2 blocks per SM: fine for plain arithmetic (4 blocks cost
// ~4% on f32 add), but ops with much arithmetic per element need the warps to
// hide its latency (pow f16 +24%, sin +15%, exp +7%), and a narrow input word
// (bf16 -> f32 loads 8 bytes per pack) needs them to keep enough bytes in
// flight (+17%).
// The paired float transcendentals (sin/cos/exp) take a 3-block floor: 85
// registers hold their packed constants and four packs in flight without
// spilling, and three blocks of 256 threads still hide the arithmetic.
template <class Op, class TA, class TB, class TO, int NIN>
constexpr int ew_min_blocks() {
  using TBv = typename std::conditional<NIN == 2, TB, TA>::type;
  constexpr int N = ew_pack<TA, TBv, TO>();
#ifndef MPB_EW_PAIRED_MINB
#define MPB_EW_PAIRED_MINB 3
#endif
  if constexpr (IsPaired<Op>::value && std::is_same<TA, float>::value && std::is_same<TO, float>::value)
    return MPB_EW_PAIRED_MINB;
  return (IsHeavy<Op>::value || VPack<TA, N>::kBytes < 16) ? 4 : 1;
}

template <class Op, class TC, class TA, class TB, class TO, int NIN>
__global__ void __launch_bounds__(kEwThreads, ew_min_blocks<Op, TA, TB, TO, NIN>()) k_ew_contig(Op op, const TA* __restrict__ a,
                                                          const TB* __restrict__ b, TO* __restrict__ out,
                                                          int64_t n, int a_bc, int b_bc) {
  pdl_enter();
  // 32-bit indices while n and every index the loop forms stay below 2^31
  const bool small = n < (int64_t(1) << 31) - (int64_t)gridDim.x * blockDim.x * 64;
  if (a_bc || b_bc) {
    if (small)
      contig_loop<true, Op, TC, TA, TB, TO, NIN, uint32_t>(op, a, b, out, (uint32_t)n, a_bc, b_bc);
    else
      contig_loop<true, Op, TC, TA, TB, TO, NIN, int64_t>(op, a, b, out, n, a_bc, b_bc);
  } else {
    if (small)
      contig_loop<false, Op, TC, TA, TB, TO, NIN, uint32_t>(op, a, b, out, (uint32_t)n, 0, 0);
    else
      contig_loop<false, Op, TC, TA, TB, TO, NIN, int64_t>(op, a, b, out, n, 0, 0);
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
// over the outer dims, every unit-stride row start aligned to its pack
// (host-checked). Work items are (row, chunk of kRowChunk packs): the row and
// its offsets are computed once per item, then each thread moves kRowUnr
// lane-strided packs (coalesced 16-byte accesses) with all loads in flight
// before the first store.
constexpr int kRowUnr = 4;
constexpr int kRowChunk = kEwThreads * kRowUnr;  // packs per work item

template <bool BC, class Op, class TC, class TA, class TB, class TO, int NIN>
MPB_D void rows_loop(const Op& op, const TA* __restrict__ a, const TB* __restrict__ b, TO* __restrict__ out,
                     const NdArgs& g, int64_t nitems, int64_t cpr, FastDiv cpr_div, int a_bc_in, int b_bc_in) {
  using TBv = typename std::conditional<NIN == 2, TB, TA>::type;
  constexpr int N = ew_pack<TA, TBv, TO>();
  const bool a_bc = BC && a_bc_in;
  const bool b_bc = BC && b_bc_in;
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
        apply_pack<Op, TC, TO, NIN>(op, pa[u], pb[u], a_bc, b_bc, as, bs, po);
        vstore<TO, N>(orow + p * N, po);
      }
    }
  }
}

template <class Op, class TC, class TA, class TB, class TO, int NIN>
__global__ void __launch_bounds__(kEwThreads, ew_min_blocks<Op, TA, TB, TO, NIN>()) k_ew_rows(Op op, const TA* __restrict__ a,
                                                        const TB* __restrict__ b, TO* __restrict__ out,
                                                        NdArgs g, int64_t nitems, int64_t cpr, FastDiv cpr_div,
                                                        int a_bc, int b_bc) {
  pdl_enter();
  if (a_bc || b_bc) {
    rows_loop<true, Op, TC, TA, TB, TO, NIN>(op, a, b, out, g, nitems, cpr, cpr_div, a_bc, b_bc);
  } else {
    rows_loop<false, Op, TC, TA, TB, TO, NIN>(op, a, b, out, g, nitems, cpr, cpr_div, 0, 0);
  }
}

// -------------------------------------------------------------- EW_TILED
// Input `a` has unit stride on dim p (an outer dim); the output is
// contiguous along q = ndim-1. Square tiles of T x T elements (T = 64 for
// types up to 8 bytes, 32 for 16-byte ones) are read along p, converted to TC
// and staged in shared memory (row pitch T+1: conflict-free both ways), then
// written along q; each thread moves T*T/256 elements per tile. Blocks loop
// over the tiles (q fastest) and load the next tile into registers while the
// current one is written out, so loads stay in flight through the store phase.
struct TiledArgs {
  int ndim;
  int p;
  int64_t dp, dq;
  int64_t nbatch;
  int nb;                        // number of batch dims
  int64_t bshape[kMaxCollapsed];
  int64_t bsa[kMaxCollapsed], bsb[kMaxCollapsed], bso[kMaxCollapsed];
  int64_t sa_q, sb_p, sb_q, so_p;
  int64_t ntp, ntq, ntiles;      // tiles along p, along q, total
  FastDiv fd_ntq, fd_ntp;        // for tile indices below 2^32
};

template <class TC>
constexpr int tiled_edge() {
  return sizeof(TC) <= 8 ? 64 : 32;
}

// Offsets of tile `ti`: its corner (p0, q0) and the batch offsets of a, b, out.
struct TileAt {
  int64_t p0, q0, oa, ob, oo;
};
MPB_D TileAt tile_at(const TiledArgs& t, int64_t ti, int T) {
  TileAt r;
  int64_t bq, bp, bi;
  if (t.ntiles < 0xffffffffLL) {  // magic-number division (a 64-bit divide is ~100 instructions)
    uint32_t x, q, rem;
    t.fd_ntq.divmod((uint32_t)ti, x, rem);
    bq = rem;
    t.fd_ntp.divmod(x, q, rem);
    bp = rem;
    bi = q;
  } else {
    int64_t x = ti;
    bq = x % t.ntq;
    x /= t.ntq;
    bp = x % t.ntp;
    bi = x / t.ntp;
  }
  r.q0 = bq * T;
  r.p0 = bp * T;
  r.oa = r.ob = r.oo = 0;
  for (int d = t.nb - 1; d >= 0; --d) {
    const int64_t c = bi % t.bshape[d];
    bi /= t.bshape[d];
    r.oa += c * t.bsa[d];
    r.ob += c * t.bsb[d];
    r.oo += c * t.bso[d];
  }
  return r;
}

template <class Op, class TC, class TA, class TB, class TO, int NIN>
__global__ void __launch_bounds__(256) k_ew_tiled(Op op, const TA* __restrict__ a, const TB* __restrict__ b,
                                                  TO* __restrict__ out, TiledArgs t) {
  using TBv = typename std::conditional<NIN == 2, TB, TA>::type;
  constexpr int T = tiled_edge<TC>();
  constexpr int PX = T / 32;          // 32-lane chunks along a tile row
  constexpr int EPT = T * T / 256;    // elements per thread per tile
  __shared__ __align__(16) char tile_raw[T * (T + 1) * sizeof(TC)];
  TC(*tile)[T + 1] = reinterpret_cast<TC(*)[T + 1]>(tile_raw);
  const int tx = threadIdx.x & 31;
  const int ty = threadIdx.x >> 5;  // 0..7
  TA v[EPT];
  // a[p0 + pl, q0 + ql], coalesced along p; interior tiles skip the bounds
  auto load = [&](const TileAt& at) {
    const TA* ab = a + at.oa + at.p0 + tx + (at.q0 + ty) * t.sa_q;
    const int64_t row8 = 8 * t.sa_q;
    if (at.p0 + T <= t.dp && at.q0 + T <= t.dq) {
#pragma unroll
      for (int i = 0; i < EPT; ++i) v[i] = ab[32 * (i % PX) + (i / PX) * row8];
    } else {
#pragma unroll
      for (int i = 0; i < EPT; ++i) {
        const int pl = tx + 32 * (i % PX), ql = ty + 8 * (i / PX);
        if (at.p0 + pl < t.dp && at.q0 + ql < t.dq) v[i] = ab[32 * (i % PX) + (i / PX) * row8];
      }
    }
  };
  int64_t ti = blockIdx.x;
  if (ti >= t.ntiles) return;
  TileAt cur = tile_at(t, ti, T);
  load(cur);
  for (;;) {
#pragma unroll
    for (int i = 0; i < EPT; ++i) {
      const int pl = tx + 32 * (i % PX), ql = ty + 8 * (i / PX);
      if (cur.p0 + pl < t.dp && cur.q0 + ql < t.dq) tile[ql][pl] = cvt<TC>(v[i]);
    }
    __syncthreads();
    // the next tile's loads are in flight while this one is written out
    const int64_t tn = ti + gridDim.x;
    TileAt nxt{};
    if (tn < t.ntiles) {
      nxt = tile_at(t, tn, T);
      load(nxt);
    }
    // out[p0 + pl, q0 + ql], coalesced along q
    {
      TO* ob = out + cur.oo + (cur.p0 + ty) * t.so_p + cur.q0 + tx;
      const TBv* bb = reinterpret_cast<const TBv*>(b) + cur.ob + (cur.p0 + ty) * t.sb_p + (cur.q0 + tx) * t.sb_q;
      const int64_t orow8 = 8 * t.so_p, brow8 = 8 * t.sb_p, bcol32 = 32 * t.sb_q;
      const bool interior = cur.p0 + T <= t.dp && cur.q0 + T <= t.dq;
#pragma unroll
      for (int i = 0; i < EPT; ++i) {
        const int ql = tx + 32 * (i % PX), pl = ty + 8 * (i / PX);
        if (interior || (cur.p0 + pl < t.dp && cur.q0 + ql < t.dq)) {
          const TC av = tile[ql][pl];
          TO r;
          if constexpr (NIN == 2) {
            r = cvt<TO>(op(av, cvt<TC>(bb[(i / PX) * brow8 + (i % PX) * bcol32])));
          } else {
            r = cvt<TO>(op(av));
          }
          ob[(i / PX) * orow8 + 32 * (i % PX)] = r;
        }
      }
    }
    if (tn >= t.ntiles) break;
    __syncthreads();
    ti = tn;
    cur = nxt;
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
