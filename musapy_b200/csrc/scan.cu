// Inclusive prefix sum (cumsum) along one axis, for sm_100a.
//
// Replaces the 3-to-5 launch Blelloch ladder of kernels/reduction.mu:557-820
// and :1723-1776 (block scan -> scan of block sums -> add prefix) and lifts its
// 256^3 length limit (rust/musapy-ops/src/op_builder.rs:3291-3300):
//   ROWS      many rows along a unit-stride axis: one CTA per row walks the row
//             in 4096-element tiles, carrying the running total; loads are
//             warp-striped 16-byte vectors, the scan is thread-sequential over
//             each vector, a warp shuffle scan across lanes and a shared-memory
//             scan across warps;
//   LOOKBACK  few long rows (axis=None included): single pass, tiles taken in
//             order from an atomic ticket, each tile publishes its aggregate
//             and inclusive prefix and looks back over its predecessors
//             (Merrill & Garland, "Single-pass Parallel Prefix Scan with
//             Decoupled Look-back", NVIDIA 2016). Every wait is bounded: on
//             expiry the kernel records MPB_ERR_TIMEOUT in a status word and
//             continues, so it always terminates;
//   COLS      axis with a non-unit stride and unit-stride columns: one thread per
//             column adds along the axis in index order, the same additions in
//             the same order as the CPU loop (op_builder.rs:3640-3688);
//   GEN       anything else: one thread per row, sequential.
#include <stdint.h>
#include <string.h>
#include "async_copy.cuh"
#include "common.cuh"
#include "internal.h"
#include "plan.h"
#include "reduce.h"

namespace mpb {
namespace {

constexpr int kScanThreads = 256;
constexpr int kScanJ = 4;  // vector rows per warp per tile

template <class Acc> MPB_D Acc sadd(Acc a, Acc b) { return a + b; }
MPB_D int64_t sadd(int64_t a, int64_t b) { return (int64_t)((uint64_t)a + (uint64_t)b); }

template <class T> MPB_D T shfl_up(T x, int o);
template <> MPB_D float shfl_up<float>(float x, int o) { return __shfl_up_sync(0xffffffffu, x, o); }
template <> MPB_D double shfl_up<double>(double x, int o) { return __shfl_up_sync(0xffffffffu, x, o); }
template <> MPB_D int64_t shfl_up<int64_t>(int64_t x, int o) { return __shfl_up_sync(0xffffffffu, (long long)x, o); }
template <class T> MPB_D T shfl_x(T x, int o);
template <> MPB_D float shfl_x<float>(float x, int o) { return __shfl_xor_sync(0xffffffffu, x, o); }
template <> MPB_D double shfl_x<double>(double x, int o) { return __shfl_xor_sync(0xffffffffu, x, o); }
template <> MPB_D int64_t shfl_x<int64_t>(int64_t x, int o) { return __shfl_xor_sync(0xffffffffu, (long long)x, o); }
template <class T> MPB_D T shfl_idx(T x, int l);
template <> MPB_D float shfl_idx<float>(float x, int l) { return __shfl_sync(0xffffffffu, x, l); }
template <> MPB_D double shfl_idx<double>(double x, int l) { return __shfl_sync(0xffffffffu, x, l); }
template <> MPB_D int64_t shfl_idx<int64_t>(int64_t x, int l) { return __shfl_sync(0xffffffffu, (long long)x, l); }

// Inclusive warp scan (Kogge-Stone over 32 lanes).
template <class Acc>
MPB_D Acc warp_incl_scan(Acc v, int lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    Acc u = shfl_up<Acc>(v, o);
    if (lane >= o) v = sadd(v, u);
  }
  return v;
}

struct ScanDev {
  int K;
  int64_t M, L;
  int64_t ks[kMaxCollapsed], kin[kMaxCollapsed], kout[kMaxCollapsed];
  int64_t sa, so;  // axis strides of input and output
};

MPB_D void row_offsets(const ScanDev& g, int64_t o, int64_t& oi, int64_t& oo) {
  oi = 0;
  oo = 0;
  for (int d = g.K - 1; d >= 0; --d) {
    const int64_t c = o % g.ks[d];
    o /= g.ks[d];
    oi += c * g.kin[d];
    oo += c * g.kout[d];
  }
}

// One tile of up to kTile elements of a row, scanned in two phases so that
// its values stay in registers in between: tile_scan loads the tile and scans
// it (each thread's vectors sequentially, lanes by a warp shuffle scan, warps
// through shared memory) and returns the tile total (block-uniform);
// tile_store adds `carry` and the warp's prefix and writes the tile.
template <class In, class Acc, int J = kScanJ>
struct Tile {
  static constexpr int VEC = 16 / sizeof(Acc);
  static constexpr int kWarpElems = J * 32 * VEC;
  static constexpr int kTile = (kScanThreads / 32) * kWarpElems;
  Acc v[J][VEC];
  Acc wpre;  // sum of the warps before this one
  bool full;
};

template <class In, class Acc, int J>
MPB_D Acc tile_scan(Tile<In, Acc, J>& T, const In* __restrict__ in, int64_t n, bool vec_ok, Acc* s_warp /* [8] */) {
  using TL = Tile<In, Acc, J>;
  constexpr int VEC = TL::VEC;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t wbase = (int64_t)warp * TL::kWarpElems;
  T.full = vec_ok && (n >= TL::kTile);
#pragma unroll
  for (int j = 0; j < J; ++j) {
    const int64_t e = wbase + (int64_t)j * 32 * VEC + (int64_t)lane * VEC;
    if (T.full) {
      const uint4 w = ld_stream16(in + e);
      const Acc* p = reinterpret_cast<const Acc*>(&w);
#pragma unroll
      for (int k = 0; k < VEC; ++k) T.v[j][k] = p[k];
    } else {
#pragma unroll
      for (int k = 0; k < VEC; ++k) T.v[j][k] = (e + k < n) ? cvt<Acc>(in[e + k]) : Acc(0);
    }
  }
  // thread-sequential over each vector, warp scan over lanes, rows in order
  Acc run = Acc(0);
#pragma unroll
  for (int j = 0; j < J; ++j) {
#pragma unroll
    for (int k = 1; k < VEC; ++k) T.v[j][k] = sadd(T.v[j][k], T.v[j][k - 1]);
    const Acc tot = T.v[j][VEC - 1];
    const Acc incl = warp_incl_scan<Acc>(tot, lane);
    Acc excl = shfl_up<Acc>(incl, 1);
    if (lane == 0) excl = Acc(0);
    const Acc pre = sadd(run, excl);
#pragma unroll
    for (int k = 0; k < VEC; ++k) T.v[j][k] = sadd(T.v[j][k], pre);
    run = sadd(run, shfl_idx<Acc>(incl, 31));
  }
  // cross-warp scan of warp totals
  __syncthreads();
  if (lane == 0) s_warp[warp] = run;
  __syncthreads();
  Acc wpre = Acc(0), total = Acc(0);
  for (int w = 0; w < kScanThreads / 32; ++w) {
    const Acc t = s_warp[w];
    if (w < warp) wpre = sadd(wpre, t);
    total = sadd(total, t);
  }
  T.wpre = wpre;
  return total;
}

template <class In, class Acc, int J>
MPB_D void tile_store(const Tile<In, Acc, J>& T, Acc* __restrict__ out, int64_t n, Acc carry) {
  using TL = Tile<In, Acc, J>;
  constexpr int VEC = TL::VEC;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t wbase = (int64_t)warp * TL::kWarpElems;
  const Acc add = sadd(carry, T.wpre);
#pragma unroll
  for (int j = 0; j < J; ++j) {
    const int64_t e = wbase + (int64_t)j * 32 * VEC + (int64_t)lane * VEC;
    if (T.full) {
      uint4 w;
      Acc* p = reinterpret_cast<Acc*>(&w);
#pragma unroll
      for (int k = 0; k < VEC; ++k) p[k] = sadd(T.v[j][k], add);
      st_stream16(out + e, w);
    } else {
#pragma unroll
      for (int k = 0; k < VEC; ++k)
        if (e + k < n) out[e + k] = sadd(T.v[j][k], add);
    }
  }
}

// ----------------------------------------------------------------- ROWS
template <class In, class Acc>
__global__ void __launch_bounds__(kScanThreads) k_scan_rows(const In* __restrict__ a, Acc* __restrict__ out,
                                                             ScanDev g, int vec_ok) {
  using TL = Tile<In, Acc>;
  __shared__ Acc s_warp[kScanThreads / 32];
  for (int64_t o = blockIdx.x; o < g.M; o += gridDim.x) {
    int64_t oi, oo;
    row_offsets(g, o, oi, oo);
    Acc carry = Acc(0);
    for (int64_t t0 = 0; t0 < g.L; t0 += TL::kTile) {
      TL T;
      const Acc total = tile_scan(T, a + oi + t0, g.L - t0, vec_ok != 0, s_warp);
      tile_store(T, out + oo + t0, g.L - t0, carry);
      carry = sadd(carry, total);
    }
  }
}

// ------------------------------------------------------------- LOOKBACK
// Scratch layout: [u32 ticket][i32 status][pad 8] then one 16-byte
// descriptor per tile: two 8-byte words {flag << 32 | value bits low half,
// flag << 32 | value bits high half}, flag 1 = the tile's aggregate, 2 = its
// inclusive prefix (0 = nothing yet; the scratch is zeroed per call). Each
// word is written and read as one naturally aligned 8-byte access, so a
// reader that sees the same flag in both words holds the value written with
// it: no fence is needed between a value and its flag.
//
// Look-back (Merrill & Garland 2016, a warp-wide window): warp 0 reads the
// descriptors of the kLookWindow tiles before this one in one round of loads
// (kLookPerLane consecutive descriptors per lane), waits (bounded) until each
// has a flag, finds the nearest inclusive prefix and adds it to the
// aggregates in between; with none in the window it adds all of them and
// moves the window back. Tiles take their index from an atomic ticket, so
// every predecessor has started. One descriptor per lane (a 32-tile window,
// one contiguous 512-byte load per round) is the fastest measured: a round
// costs one L2 round trip whatever its width, but wider windows of 64, 128,
// 256 and 512 tiles (2-16 loads per lane) made each round slower under the
// scan's own traffic and the whole scan 4% to 2.1x slower.
constexpr int64_t kSpinLimit = 1 << 22;  // polls per descriptor before giving up
#ifndef MPB_SCAN_LB_J
#define MPB_SCAN_LB_J 8
#endif
#ifndef MPB_SCAN_LB_MINB
#define MPB_SCAN_LB_MINB 3
#endif
constexpr int kLookJ = MPB_SCAN_LB_J;        // vector rows per warp of a look-back tile
constexpr int kLookMinBlocks = MPB_SCAN_LB_MINB;  // CTAs per SM the registers must allow
#ifndef MPB_SCAN_LB_PER_LANE
#define MPB_SCAN_LB_PER_LANE 1
#endif
constexpr int kLookPerLane = MPB_SCAN_LB_PER_LANE;
constexpr int kLookWindow = 32 * kLookPerLane;

template <class Acc>
MPB_D void desc_publish(unsigned long long* d, Acc v, unsigned flag) {
  static_assert(sizeof(Acc) == 4 || sizeof(Acc) == 8, "4- or 8-byte accumulators");
  unsigned long long bits = 0;
  memcpy(&bits, &v, sizeof(Acc));
  const unsigned long long f = (unsigned long long)flag << 32;
  const unsigned long long w0 = f | (bits & 0xffffffffull), w1 = f | (bits >> 32);
  asm volatile("st.relaxed.gpu.global.v2.u64 [%0], {%1, %2};" ::"l"(d), "l"(w0), "l"(w1) : "memory");
}

// One read of descriptor `d`: its flag (0 = nothing yet, or the two words
// disagree because a write landed between them) and value.
template <class Acc>
MPB_D unsigned desc_read(const unsigned long long* d, Acc& v) {
  unsigned long long w0, w1;
  asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(w0), "=l"(w1) : "l"(d) : "memory");
  const unsigned f0 = (unsigned)(w0 >> 32), f1 = (unsigned)(w1 >> 32);
  const unsigned long long bits = (w0 & 0xffffffffull) | ((w1 & 0xffffffffull) << 32);
  memcpy(&v, &bits, sizeof(Acc));
  return f0 == f1 ? f0 : 0u;
}

// Exclusive prefix of tile `tid` (local index `t` in its row), run by warp 0.
// Each round reads the whole window once; it is settled when the nearest
// inclusive prefix in it (or the row start) has only aggregates in front of
// it, and otherwise read again (bounded) - so a tile waits only for the
// predecessors between itself and the nearest inclusive prefix, not for the
// whole window.
template <class Acc>
MPB_D Acc look_back(const unsigned long long* desc, int64_t tid, int64_t t, int* status) {
  const int lane = threadIdx.x & 31;
  Acc excl = Acc(0);
  int64_t back = 0;  // tiles already covered behind this one
  int64_t spins = 0;
  unsigned ns = 32;
  for (;;) {
    Acc v[kLookPerLane];
    unsigned f[kLookPerLane];
    // slot k of this lane: distance back + lane * kLookPerLane + k + 1
#pragma unroll
    for (int k = 0; k < kLookPerLane; ++k) {
      const int64_t dist = back + (int64_t)lane * kLookPerLane + k + 1;
      f[k] = 3;  // before the row start: not a tile
      v[k] = Acc(0);
      if (dist <= t) f[k] = desc_read<Acc>(desc + 2 * (tid - dist), v[k]);
    }
    // nearest inclusive prefix of the window (slot index), and nearest
    // descriptor still without a flag
    int my_inc = 0x7fffffff, my_zero = 0x7fffffff;
#pragma unroll
    for (int k = kLookPerLane - 1; k >= 0; --k) {
      if (f[k] == 2) my_inc = lane * kLookPerLane + k;
      if (f[k] == 0) my_zero = lane * kLookPerLane + k;
    }
    const int inc = __reduce_min_sync(0xffffffffu, my_inc);
    const int zero = __reduce_min_sync(0xffffffffu, my_zero);
    if (zero < inc) {  // a predecessor in front of the nearest prefix has not published yet
      // give up after the spin limit, or at once when another tile already
      // gave up (the status word is non-zero): the result is then wrong and
      // the status word says so, and no further tile waits out its limit
      if (++spins > kSpinLimit || *(volatile int*)status != 0) {
        if (lane == 0) atomicOr(status, 1 << MPB_ERR_TIMEOUT);
        spins = kSpinLimit + 1;
      } else {
        __nanosleep(ns);
        if (ns < 256) ns <<= 1;
        continue;
      }
    }
    Acc part = Acc(0);
#pragma unroll
    for (int k = 0; k < kLookPerLane; ++k)
      if (lane * kLookPerLane + k <= inc && f[k] != 3) part = sadd(part, v[k]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) part = sadd(part, shfl_x<Acc>(part, o));
    excl = sadd(excl, part);
    if (inc != 0x7fffffff || spins > kSpinLimit) return excl;
    back += kLookWindow;
    if (back >= t) return excl;  // cannot happen: the row's tile 0 publishes an inclusive prefix
    ns = 32;
  }
}

template <class In, class Acc>
__global__ void __launch_bounds__(kScanThreads, kLookMinBlocks) k_scan_lookback(const In* __restrict__ a, Acc* __restrict__ out,
                                                                 ScanDev g, int vec_ok, char* __restrict__ scratch,
                                                                 int64_t tiles_per_row) {
  using TL = Tile<In, Acc, kLookJ>;
  __shared__ Acc s_warp[kScanThreads / 32];
  __shared__ uint32_t s_ticket;
  __shared__ Acc s_prefix;
  unsigned* ticket = reinterpret_cast<unsigned*>(scratch);
  int* status = reinterpret_cast<int*>(scratch + 4);
  unsigned long long* desc = reinterpret_cast<unsigned long long*>(scratch + 16);
  const int64_t ntiles = g.M * tiles_per_row;
  if (threadIdx.x == 0) s_ticket = atomicAdd(ticket, 1u);
  __syncthreads();
  const int64_t tid = s_ticket;
  if (tid >= ntiles) return;
  const int64_t row = tid / tiles_per_row;
  const int64_t t = tid - row * tiles_per_row;
  int64_t oi, oo;
  row_offsets(g, row, oi, oo);
  const int64_t t0 = t * TL::kTile;
  const In* in = a + oi + t0;
  Acc* dst = out + oo + t0;
  const int64_t n = g.L - t0;
  // the tile is read once: scanned into registers, its aggregate published,
  // its prefix found by looking back, then the registers written out
  TL T;
  const Acc total = tile_scan(T, in, n, vec_ok != 0, s_warp);
  if (threadIdx.x < 32) {
    if (t == 0) {
      if (threadIdx.x == 0) {
        desc_publish<Acc>(desc + 2 * tid, total, 2u);
        s_prefix = Acc(0);
      }
    } else {
      if (threadIdx.x == 0) desc_publish<Acc>(desc + 2 * tid, total, 1u);
      const Acc excl = look_back<Acc>(desc, tid, t, status);
      if (threadIdx.x == 0) {
        desc_publish<Acc>(desc + 2 * tid, sadd(excl, total), 2u);
        s_prefix = excl;
      }
    }
  }
  __syncthreads();
  tile_store(T, dst, n, s_prefix);
}

// LOOKBACK with the tile in shared memory (contiguous rows of a float or
// int64 type, 16-byte aligned): one bulk copy brings a 32 KiB tile in,
// the scan runs in place row by row, the aggregate is published, warp 0
// looks back, and the threads add the prefix on the way out. The tile's
// values wait out the look-back in shared memory instead of registers, so
// a thread needs few registers and six CTAs fit on an SM: twice the tiles
// in flight of the register tile, which is what a look-back scan's
// bandwidth depends on (each tile waits for the predecessors between it and
// the nearest published prefix).
#ifndef MPB_SCAN_SMEM_TILE
#define MPB_SCAN_SMEM_TILE 32768
#endif
constexpr int kSmemTileBytes = MPB_SCAN_SMEM_TILE;
#ifndef MPB_SCAN_SMEM_MINB
#define MPB_SCAN_SMEM_MINB 6
#endif

template <class Acc>
struct SmemTile {
  static constexpr int VEC = 16 / (int)sizeof(Acc);
  static constexpr int kElems = kSmemTileBytes / (int)sizeof(Acc);
  static constexpr int J = kElems / (kScanThreads * VEC);  // vector rows per warp
  static constexpr int kWarpElems = J * 32 * VEC;
};

template <class Acc>
__global__ void __launch_bounds__(kScanThreads, MPB_SCAN_SMEM_MINB)
    k_scan_lookback_smem(const Acc* __restrict__ a, Acc* __restrict__ out, ScanDev g, char* __restrict__ scratch,
                         int64_t tiles_per_row) {
  using ST = SmemTile<Acc>;
  constexpr int VEC = ST::VEC;
  extern __shared__ __align__(128) char scan_smem[];
  Acc* tile = reinterpret_cast<Acc*>(scan_smem);
  __shared__ Acc s_warp[kScanThreads / 32];
  __shared__ uint32_t s_ticket;
  __shared__ Acc s_prefix;
  __shared__ __align__(8) unsigned long long s_bar;
  unsigned* ticket = reinterpret_cast<unsigned*>(scratch);
  int* status = reinterpret_cast<int*>(scratch + 4);
  unsigned long long* desc = reinterpret_cast<unsigned long long*>(scratch + 16);
  const int64_t ntiles = g.M * tiles_per_row;
  const uint32_t bar = smem_u32(&s_bar);
  if (threadIdx.x == 0) {
    s_ticket = atomicAdd(ticket, 1u);
    mbar_init(bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  const int64_t tid = s_ticket;
  if (tid >= ntiles) return;
  const int64_t row = tid / tiles_per_row;
  const int64_t t = tid - row * tiles_per_row;
  int64_t oi, oo;
  row_offsets(g, row, oi, oo);
  const int64_t t0 = t * ST::kElems;
  const int64_t n = g.L - t0;
  const int cnt = n < ST::kElems ? (int)n : ST::kElems;
  const Acc* in = a + oi + t0;
  Acc* dst = out + oo + t0;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // load: one bulk copy of the tile's whole 16-byte units; the rest (a
  // partial unit at the end of a row, then zeros) by the threads
  const int bulk_elems = cnt / VEC * VEC;
  if (threadIdx.x == 0 && bulk_elems > 0) {
    mbar_expect_tx(bar, (uint32_t)(bulk_elems * sizeof(Acc)));
    bulk_load(smem_u32(tile), in, (uint32_t)(bulk_elems * sizeof(Acc)), bar);
  }
  for (int e = bulk_elems + threadIdx.x; e < ST::kElems; e += kScanThreads) tile[e] = e < cnt ? in[e] : Acc(0);
  if (bulk_elems > 0 && !mbar_wait(bar, 0)) {
    if (threadIdx.x == 0) atomicOr(status, 1 << MPB_ERR_TIMEOUT);
  }
  __syncthreads();
  // scan in place: thread-sequential over each vector, warp scan over lanes,
  // rows in order (the register tile's arithmetic)
  const int wbase = warp * ST::kWarpElems;
  Acc run = Acc(0);
#pragma unroll 2
  for (int j = 0; j < ST::J; ++j) {
    Acc* p = tile + wbase + j * 32 * VEC + lane * VEC;
    uint4 w = *reinterpret_cast<const uint4*>(p);
    Acc* v = reinterpret_cast<Acc*>(&w);
#pragma unroll
    for (int k = 1; k < VEC; ++k) v[k] = sadd(v[k], v[k - 1]);
    const Acc incl = warp_incl_scan<Acc>(v[VEC - 1], lane);
    Acc excl = shfl_up<Acc>(incl, 1);
    if (lane == 0) excl = Acc(0);
    const Acc pre = sadd(run, excl);
#pragma unroll
    for (int k = 0; k < VEC; ++k) v[k] = sadd(v[k], pre);
    *reinterpret_cast<uint4*>(p) = w;
    run = sadd(run, shfl_idx<Acc>(incl, 31));
  }
  if (lane == 0) s_warp[warp] = run;
  __syncthreads();
  Acc wpre = Acc(0), total = Acc(0);
  for (int w = 0; w < kScanThreads / 32; ++w) {
    const Acc tw = s_warp[w];
    if (w < warp) wpre = sadd(wpre, tw);
    total = sadd(total, tw);
  }
  if (threadIdx.x < 32) {
    if (t == 0) {
      if (threadIdx.x == 0) {
        desc_publish<Acc>(desc + 2 * tid, total, 2u);
        s_prefix = Acc(0);
      }
    } else {
      if (threadIdx.x == 0) desc_publish<Acc>(desc + 2 * tid, total, 1u);
      const Acc excl = look_back<Acc>(desc, tid, t, status);
      if (threadIdx.x == 0) {
        desc_publish<Acc>(desc + 2 * tid, sadd(excl, total), 2u);
        s_prefix = excl;
      }
    }
  }
  __syncthreads();
  const Acc add = sadd(s_prefix, wpre);
#pragma unroll 2
  for (int j = 0; j < ST::J; ++j) {
    const int e = wbase + j * 32 * VEC + lane * VEC;
    uint4 w = *reinterpret_cast<const uint4*>(tile + e);
    Acc* v = reinterpret_cast<Acc*>(&w);
#pragma unroll
    for (int k = 0; k < VEC; ++k) v[k] = sadd(v[k], add);
    if (e + VEC <= cnt) {
      st_stream16(dst + e, w);
    } else {
#pragma unroll
      for (int k = 0; k < VEC; ++k)
        if (e + k < cnt) dst[e + k] = v[k];
    }
  }
}

// ----------------------------------------------------------------- COLS
// One thread per column (innermost kept dim unit-stride in and out).
template <class In, class Acc>
__global__ void __launch_bounds__(kScanThreads) k_scan_cols(const In* __restrict__ a, Acc* __restrict__ out,
                                                             ScanDev g) {
  const int64_t gt = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t gs = (int64_t)gridDim.x * blockDim.x;
  for (int64_t o = gt; o < g.M; o += gs) {
    int64_t oi, oo;
    row_offsets(g, o, oi, oo);
    Acc acc = Acc(0);
    constexpr int UNR = 8;
    int64_t k = 0;
    for (; k + UNR <= g.L; k += UNR) {
      Acc v[UNR];
#pragma unroll
      for (int u = 0; u < UNR; ++u) v[u] = cvt<Acc>(a[oi + (k + u) * g.sa]);
#pragma unroll
      for (int u = 0; u < UNR; ++u) {
        acc = sadd(acc, v[u]);
        out[oo + (k + u) * g.so] = acc;
      }
    }
    for (; k < g.L; ++k) {
      acc = sadd(acc, cvt<Acc>(a[oi + k * g.sa]));
      out[oo + k * g.so] = acc;
    }
  }
}

inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

struct ScanPlan {
  ScanDev g;
  int kind;  // 0 rows, 1 lookback, 2 cols/gen (sequential per thread)
  int vec_ok;
  int smem;  // look-back with shared-memory tiles
  int64_t tiles_per_row;
};

template <class In, class Acc>
ScanPlan scan_plan(const ScanReq& r) {
  ScanPlan pl;
  ScanDev& g = pl.g;
  int64_t out_st[MPB_MAX_DIMS];
  int64_t acc = 1;
  for (int i = r.ndim - 1; i >= 0; --i) {
    out_st[i] = acc;
    acc *= r.shape[i];
  }
  g.L = r.shape[r.axis];
  g.sa = r.strides[r.axis];
  g.so = out_st[r.axis];
  g.M = 1;
  int64_t ks[MPB_MAX_DIMS], ki[MPB_MAX_DIMS], ko[MPB_MAX_DIMS];
  int K = 0;
  for (int d = 0; d < r.ndim; ++d) {
    if (d == r.axis) continue;
    g.M *= r.shape[d];
    if (r.shape[d] == 1) continue;
    if (K > 0 && ki[K - 1] == r.strides[d] * r.shape[d] && ko[K - 1] == out_st[d] * r.shape[d]) {
      ks[K - 1] *= r.shape[d];
      ki[K - 1] = r.strides[d];
      ko[K - 1] = out_st[d];
    } else {
      ks[K] = r.shape[d];
      ki[K] = r.strides[d];
      ko[K] = out_st[d];
      ++K;
    }
  }
  g.K = K;
  for (int d = 0; d < K && d < kMaxCollapsed; ++d) {
    g.ks[d] = ks[d];
    g.kin[d] = ki[d];
    g.kout[d] = ko[d];
  }
  const int sms = sm_count();
  pl.tiles_per_row = cdiv(g.L, Tile<In, Acc>::kTile);  // rows kernel's tiles (kind decision)
  if ((g.sa == 1 || g.L == 1) && (g.so == 1 || g.L == 1)) {
    bool vec_ok = std::is_same<In, Acc>::value && (((uintptr_t)r.a & 15) == 0) && (((uintptr_t)r.out & 15) == 0);
    for (int d = 0; d < K && vec_ok; ++d)
      if ((ki[d] * (int64_t)sizeof(In)) % 16 || (ko[d] * (int64_t)sizeof(Acc)) % 16) vec_ok = false;
    pl.vec_ok = vec_ok;
    pl.kind = (g.M >= 2 * sms || pl.tiles_per_row <= 1) ? 0 : 1;
    pl.smem = 0;
#ifndef MPB_SCAN_NO_SMEM
    // shared-memory tiles: input already in the accumulator type, every row
    // start 16-byte aligned (the bulk copy's rule)
    pl.smem = pl.kind == 1 && std::is_same<In, Acc>::value && vec_ok;
#endif
    if (pl.kind == 1)
      pl.tiles_per_row = pl.smem ? cdiv(g.L, (int64_t)SmemTile<Acc>::kElems) : cdiv(g.L, Tile<In, Acc, kLookJ>::kTile);
  } else {
    pl.vec_ok = 0;
    pl.smem = 0;
    pl.kind = 2;
  }
  return pl;
}

template <class Acc>
size_t lookback_bytes(int64_t ntiles) {
  return 16 + (size_t)ntiles * 16;
}

template <class In, class Acc>
int scan_typed(const ScanReq& r, cudaStream_t s, size_t* need_only) {
  ScanPlan pl = scan_plan<In, Acc>(r);
  const ScanDev& g = pl.g;
  if (g.K > kMaxCollapsed) return fail(MPB_ERR_SHAPE, "cumsum: too many dims after collapsing");
  const size_t need = pl.kind == 1 ? lookback_bytes<Acc>(g.M * pl.tiles_per_row) : 0;
  if (need_only) {
    *need_only = need;
    return MPB_OK;
  }
  if (g.M * g.L == 0) return MPB_OK;
  const In* a = static_cast<const In*>(r.a);
  Acc* out = static_cast<Acc*>(r.out);
  const int sms = sm_count();
  switch (pl.kind) {
    case 0: {
      int64_t blocks = g.M < (int64_t)sms * 64 ? g.M : (int64_t)sms * 64;
      k_scan_rows<In, Acc><<<(unsigned)blocks, kScanThreads, 0, s>>>(a, out, g, pl.vec_ok);
      return launch_check("cumsum_rows");
    }
    case 1: {
      if (r.scratch_bytes < need || !r.scratch)
        return fail(MPB_ERR_SCRATCH, "cumsum: scratch of %zu bytes needed, %zu given", need, r.scratch_bytes);
      int rc = cuda_check(cudaMemsetAsync(r.scratch, 0, need, s), "cumsum scratch clear");
      if (rc) return rc;
      const int64_t ntiles = g.M * pl.tiles_per_row;
      if constexpr (std::is_same<In, Acc>::value) {
        if (pl.smem) {
          if (cudaFuncSetAttribute(k_scan_lookback_smem<Acc>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   kSmemTileBytes) != cudaSuccess)
            return cuda_check(cudaGetLastError(), "cumsum_lookback: shared memory size");
          k_scan_lookback_smem<Acc><<<(unsigned)ntiles, kScanThreads, kSmemTileBytes, s>>>(
              a, out, g, static_cast<char*>(r.scratch), pl.tiles_per_row);
          return launch_check("cumsum_lookback_smem");
        }
      }
      k_scan_lookback<In, Acc><<<(unsigned)ntiles, kScanThreads, 0, s>>>(a, out, g, pl.vec_ok,
                                                                       static_cast<char*>(r.scratch),
                                                                       pl.tiles_per_row);
      return launch_check("cumsum_lookback");
    }
    default: {
      int64_t blocks = cdiv(g.M, kScanThreads);
      if (blocks > (int64_t)sms * 64) blocks = (int64_t)sms * 64;
      if (blocks < 1) blocks = 1;
      k_scan_cols<In, Acc><<<(unsigned)blocks, kScanThreads, 0, s>>>(a, out, g);
      return launch_check("cumsum_cols");
    }
  }
}

template <class Acc>
int scan_in(const ScanReq& r, cudaStream_t s, size_t* need) {
  switch (r.in_dt) {
    case MPB_BOOL: return scan_typed<boolean, Acc>(r, s, need);
    case MPB_I8: return scan_typed<int8_t, Acc>(r, s, need);
    case MPB_I16: return scan_typed<int16_t, Acc>(r, s, need);
    case MPB_I32: return scan_typed<int32_t, Acc>(r, s, need);
    case MPB_I64: return scan_typed<int64_t, Acc>(r, s, need);
    case MPB_U8: return scan_typed<uint8_t, Acc>(r, s, need);
    case MPB_U16: return scan_typed<uint16_t, Acc>(r, s, need);
    case MPB_U32: return scan_typed<uint32_t, Acc>(r, s, need);
    case MPB_U64: return scan_typed<uint64_t, Acc>(r, s, need);
    default: return fail(MPB_ERR_DTYPE, "cumsum: input dtype %d not supported", r.in_dt);
  }
}

int scan_dispatch(const ScanReq& r, cudaStream_t s, size_t* need) {
  if (r.ndim < 1 || r.ndim > MPB_MAX_DIMS || r.axis < 0 || r.axis >= r.ndim)
    return fail(MPB_ERR_INVALID, "cumsum: bad ndim/axis (%d, %d)", r.ndim, r.axis);
  switch (r.out_dt) {
    case MPB_F32:
      if (r.in_dt == MPB_F32) return scan_typed<float, float>(r, s, need);
      break;
    case MPB_F64:
      if (r.in_dt == MPB_F64) return scan_typed<double, double>(r, s, need);
      break;
    case MPB_I64: return scan_in<int64_t>(r, s, need);
    default: break;
  }
  return fail(MPB_ERR_DTYPE, "cumsum: input dtype %d -> output dtype %d not supported", r.in_dt, r.out_dt);
}

}  // namespace

size_t scan_scratch_bytes(const ScanReq& r) {
  size_t need = 0;
  if (scan_dispatch(r, nullptr, &need) != MPB_OK) return 0;
  return need;
}

int scan_run(const ScanReq& r, cudaStream_t s) {
  if (!r.a || !r.out) {
    int64_t n = 1;
    for (int i = 0; i < r.ndim; ++i) n *= r.shape[i];
    if (n == 0) return MPB_OK;
    return fail(MPB_ERR_INVALID, "cumsum: null pointer");
  }
  return scan_dispatch(r, s, nullptr);
}

}  // namespace mpb
