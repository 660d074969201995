// EW_TILED through the Tensor Memory Accelerator: elementwise ops whose
// input is a transposed view (unit stride on an outer dim p, stride sa_q on
// the output's inner dim q), the layout of musapy's transpose + op and of
// contiguous() on a transposed view (indexing.mu:217-293 copies such views
// through a padded shared-memory tile, one element per thread).
//
// Each warp runs its own pipeline of tma_stages() tiles: its lane 0 issues a
// 2-D / 3-D TMA load (cp.async.bulk.tensor) of a box of 32 q rows x BOXB
// contiguous bytes along p into a stage, armed on an mbarrier with the box's
// byte count. The warp waits on the stage's barrier, then every lane reads
// an E x E block (E = 16 / sizeof(TA): one 16-byte chunk of E rows) with
// 16-byte shared loads - conflict-free, since the lanes of a shared-memory
// phase read consecutive chunks of one row - transposes it in registers and
// writes E-element runs of the output rows with vector stores. A stage is
// refilled as soon as the warp has read it, so several loads per warp stay
// in flight with no block-wide barrier, and thread work per element is a
// fraction of one shared load and one store.
//
// Used for 2- and 8-byte elements, where it beats the padded-tile kernel
// (k_ew_tiled); the per-size box widths are in run_tiled_tma. Boxes reaching
// past the array are filled with zeros by the TMA unit and the stores of
// those rows are skipped. Waits are bounded: a stage that does not fill
// within 2 s sets the library's tiled-wait flag (read by mpb_ew_wait_status)
// and the warp stops.
#pragma once
#include <cuda.h>
#include <string.h>
#include "async_copy.cuh"
#include "elementwise.cuh"
#include "internal.h"

namespace mpb {
namespace ew {

constexpr int kTmaWarps = 4;  // warps per block, each with its own pipeline
constexpr int kTmaRows = 32;  // q rows per tile
// Per box width (bytes of p per row): tiles in flight per warp and the
// block's shared memory.
constexpr int tma_stages(int boxb) { return boxb <= 128 ? 4 : 3; }
constexpr int tma_smem_bytes(int boxb) { return kTmaWarps * tma_stages(boxb) * (kTmaRows * boxb + 8) + 128; }

struct TmaArgs {
  int64_t dp, dq;            // extents along p (unit stride in the input) and q (inner in the output)
  int64_t ntp, ntq, ntiles;  // tiles along p, along q, total (whole groups, batch outermost)
  int64_t ngp, ngq;          // tile groups along p, along q
  FastDiv fd_ntq, fd_ntp;    // group decode (by ngq, ngp) for tile indices below 2^32
  int sp_log;                // log2 of the tiles along p in a group
  int64_t so_p, bso;         // output strides along p and the batch dim
  int64_t sb_p, sb_q, bsb;   // strides of the other operand (binary ops)
  int batched;               // 3-D tensor map (one batch dim)
  int* err;                  // tiled-wait flag
};

MPB_D void tma_load_tile(uint32_t dst, const CUtensorMap* tm, int batched, int x, int y, int z, uint32_t bar) {
  if (batched) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::
            "r"(dst),
        "l"(tm), "r"(x), "r"(y), "r"(z), "r"(bar)
        : "memory");
  } else {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(dst),
        "l"(tm), "r"(x), "r"(y), "r"(bar)
        : "memory");
  }
}

MPB_D uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}

struct TileIdx {
  int64_t bi, tp, tq;
};
// Tiles are numbered in groups of kTmaWarps forming a (1 << sp_log) x
// (kTmaWarps >> sp_log) block of (p, q) tiles, the groups with q fastest:
// the warps of a block, running together, read adjacent 128-byte segments
// of the same input rows and write adjacent runs of the same output rows.
// Tiles of a group past the array's edge load zeros and store nothing.
MPB_D TileIdx tma_tile(const TmaArgs& t, int64_t ti) {
  TileIdx r;
  const int sub = (int)(ti & (kTmaWarps - 1));
  const int64_t g = ti / kTmaWarps;
  int64_t gp, gq;
  if (t.ntiles < 0xffffffffLL) {
    uint32_t x, q, rem;
    t.fd_ntq.divmod((uint32_t)g, x, rem);
    gq = rem;
    t.fd_ntp.divmod(x, q, rem);
    gp = rem;
    r.bi = q;
  } else {
    gq = g % t.ngq;
    const int64_t x = g / t.ngq;
    gp = x % t.ngp;
    r.bi = x / t.ngp;
  }
  r.tp = (gp << t.sp_log) + (sub & ((1 << t.sp_log) - 1));
  r.tq = gq * (kTmaWarps >> t.sp_log) + (sub >> t.sp_log);
  return r;
}

// E values of TO written as one run (E * sizeof(TO) bytes, aligned to the
// run or to 16 bytes, host-checked).
template <class TO, int E>
MPB_D void store_run(TO* dst, const TO (&v)[E]) {
  constexpr int B = E * (int)sizeof(TO);
  if constexpr (B % 16 == 0) {
#pragma unroll
    for (int w = 0; w < B / 16; ++w) {
      uint4 u;
      memcpy(&u, reinterpret_cast<const char*>(v) + 16 * w, 16);
      reinterpret_cast<uint4*>(dst)[w] = u;
    }
  } else if constexpr (B == 8) {
    uint2 u;
    memcpy(&u, v, 8);
    *reinterpret_cast<uint2*>(dst) = u;
  } else if constexpr (B == 4) {
    uint32_t u;
    memcpy(&u, v, 4);
    *reinterpret_cast<uint32_t*>(dst) = u;
  } else {
#pragma unroll
    for (int k = 0; k < E; ++k) dst[k] = v[k];
  }
}

// BMODE: 0 unary, 1 binary with the other operand constant along p (read
// once per row run; the values of the warp's next tile are loaded while the
// current one is processed, so no tile starts by waiting on them), 2 binary
// with any other strides.
template <class Op, class TC, class TA, class TB, class TO, int NIN, int BMODE, int BOXB>
__global__ void __launch_bounds__(kTmaWarps * 32) k_ew_tiled_tma(const __grid_constant__ CUtensorMap tm, Op op,
                                                                  const TB* __restrict__ b, TO* __restrict__ out,
                                                                  TmaArgs t) {
  constexpr int E = 16 / (int)sizeof(TA);    // elements per 16-byte chunk
  constexpr int PX = BOXB / (int)sizeof(TA);  // p extent of a tile
  constexpr int CH = BOXB / 16;               // chunks per tile row
  constexpr int RB = 32 / CH;                 // row blocks (of E rows) per pass
  constexpr int PASSES = kTmaRows / (RB * E);
  constexpr int STAGES = tma_stages(BOXB);
  using TBv = typename std::conditional<NIN == 2, TB, TA>::type;
  constexpr int TILE = kTmaRows * BOXB;
  constexpr int STAGE = TILE;
  static_assert(CH <= 32 && PASSES >= 1, "tile shape does not fit the lane layout");
  extern __shared__ char tma_smem[];
  const uint32_t base = (smem_u32(tma_smem) + 127u) & ~127u;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t stages = base + (uint32_t)(warp * STAGES * STAGE);
  const uint32_t bars = base + (uint32_t)(kTmaWarps * STAGES * STAGE + warp * STAGES * 8);
  const int64_t gw = (int64_t)blockIdx.x * kTmaWarps + warp;
  const int64_t nw = (int64_t)gridDim.x * kTmaWarps;
  if (gw >= t.ntiles) return;

  auto issue = [&](int64_t ti, int s) {
    const TileIdx x = tma_tile(t, ti);
    const uint32_t bar = bars + 8u * (uint32_t)s;
    const uint32_t dst = stages + (uint32_t)(s * STAGE);
    mbar_expect_tx(bar, TILE);
    tma_load_tile(dst, &tm, t.batched, (int)(x.tp * PX), (int)(x.tq * kTmaRows), (int)x.bi, bar);
  };
  if (lane == 0) {
    for (int s = 0; s < STAGES; ++s) mbar_init(bars + 8u * (uint32_t)s, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    for (int s = 0; s < STAGES; ++s)
      if (gw + s * nw < t.ntiles) issue(gw + s * nw, s);
  }
  __syncwarp();

  // Lane (qb, c) reads chunk c (p in [c*E, c*E + E)) of E rows: the lanes
  // of a shared-memory phase read consecutive chunks of one row, so the
  // 16-byte loads are conflict-free without a swizzle.
  const int c = lane % CH;
  const int qb = lane / CH;
  // BMODE 1: the other operand along q for every pass of a tile; `bq_next`
  // holds the warp's next tile's values, loaded one tile ahead
  constexpr int BQ = NIN == 2 && BMODE == 1 ? PASSES : 1;
  TC bq_all[BQ][E], bq_next[BQ][E];
  auto load_bq = [&](int64_t tile_index, TC (&dstv)[BQ][E]) {
    if constexpr (NIN == 2 && BMODE == 1) {
      const TileIdx y = tma_tile(t, tile_index);
      const TBv* bb = reinterpret_cast<const TBv*>(b) + y.bi * t.bsb;
      const int64_t qy = y.tq * kTmaRows;
#pragma unroll
      for (int pass = 0; pass < PASSES; ++pass) {
        const int64_t q = qy + (pass * RB + qb) * E;
#pragma unroll
        for (int k2 = 0; k2 < E; ++k2) dstv[pass][k2] = q < t.dq ? cvt<TC>(bb[(q + k2) * t.sb_q]) : TC{};
      }
    }
  };
  load_bq(gw, bq_next);
  for (int64_t k = 0;; ++k) {
    const int64_t ti = gw + k * nw;
    if (ti >= t.ntiles) break;
    const int s = (int)(k % STAGES);
    if (!mbar_wait(bars + 8u * (uint32_t)s, (uint32_t)((k / STAGES) & 1))) {
      if (lane == 0) atomicExch(t.err, 1);
      return;
    }
    const TileIdx x = tma_tile(t, ti);
    const uint32_t tile = stages + (uint32_t)(s * STAGE);
    const int64_t p0 = x.tp * PX + c * E, q0 = x.tq * kTmaRows;
    TO* ob = out + x.bi * t.bso;
    if constexpr (NIN == 2 && BMODE == 1) {
      // this tile's values (loaded one tile ago), then the next tile's
#pragma unroll
      for (int pass = 0; pass < PASSES; ++pass)
#pragma unroll
        for (int k2 = 0; k2 < E; ++k2) bq_all[pass][k2] = bq_next[pass][k2];
      if (ti + nw < t.ntiles) load_bq(ti + nw, bq_next);
    }
#pragma unroll
    for (int pass = 0; pass < PASSES; ++pass) {
      const int r0 = (pass * RB + qb) * E;
      const int64_t q = q0 + r0;
      if (q >= t.dq) continue;  // dq % E == 0: the E rows are all in or all out
      uint4 v[E];
#pragma unroll
      for (int k2 = 0; k2 < E; ++k2) {
        const int r = r0 + k2;
        v[k2] = lds128(tile + (uint32_t)(r * BOXB + c * 16));
      }
#pragma unroll
      for (int j = 0; j < E; ++j) {
        const int64_t p = p0 + j;
        if (p < t.dp) {
          TO res[E];
#pragma unroll
          for (int k2 = 0; k2 < E; ++k2) {
            const TC av = cvt<TC>(reinterpret_cast<const TA*>(&v[k2])[j]);
            if constexpr (NIN == 2) {
              TC bv;
              if constexpr (BMODE == 1) {
                bv = bq_all[pass][k2];
              } else {
                bv = cvt<TC>(reinterpret_cast<const TBv*>(b)[x.bi * t.bsb + p * t.sb_p + (q + k2) * t.sb_q]);
              }
              res[k2] = cvt<TO>(op(av, bv));
            } else {
              res[k2] = cvt<TO>(op(av));
            }
          }
          store_run<TO, E>(ob + p * t.so_p + q, res);
        }
      }
    }
    __syncwarp();
    const int64_t tn = ti + STAGES * nw;
    if (lane == 0 && tn < t.ntiles) {
      // the warp's shared reads of this stage are ordered before the
      // asynchronous-proxy write that refills it
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      issue(tn, s);
    }
  }
}

// Host side (elementwise.cu).
int tma_encode(CUtensorMap* m, const void* base, int elem_bytes, int64_t dp, int64_t dq, int64_t nb, int64_t sq_bytes,
               int64_t sb_bytes, int box_p, int box_q);
int* tiled_wait_flag();
bool tiled_tma_enabled();
void count_tma_launch();
int blocks_per_sm_smem(const void* kernel, int threads, int smem);
inline int64_t tma_cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

template <class Op, class TC, class TA, class TB, class TO, int NIN, int BOXB, int SP_LOG>
int launch_tiled_tma(const Op& op, const TA* a, const TB* b, TO* out, const TiledArgs& ta, int* err, cudaStream_t s) {
  constexpr int SZ = (int)sizeof(TA);
  constexpr int PX = BOXB / SZ;
  CUtensorMap tm;
  const int64_t nbatch = ta.nb ? ta.bshape[0] : 1;
  if (tma_encode(&tm, a, SZ, ta.dp, ta.dq, nbatch, ta.sa_q * SZ, ta.nb ? ta.bsa[0] * SZ : 0, PX, kTmaRows) != 0)
    return -1;
  TmaArgs t;
  t.dp = ta.dp;
  t.dq = ta.dq;
  t.ntp = tma_cdiv(ta.dp, PX);
  t.ntq = tma_cdiv(ta.dq, kTmaRows);
  t.sp_log = SP_LOG;
  t.ngp = tma_cdiv(t.ntp, 1 << t.sp_log);
  t.ngq = tma_cdiv(t.ntq, kTmaWarps >> t.sp_log);
  t.ntiles = t.ngp * t.ngq * nbatch * kTmaWarps;
  t.fd_ntq = FastDiv((uint32_t)(t.ngq < 0xffffffffLL ? t.ngq : 1));
  t.fd_ntp = FastDiv((uint32_t)(t.ngp < 0xffffffffLL ? t.ngp : 1));
  t.so_p = ta.so_p;
  t.bso = ta.nb ? ta.bso[0] : 0;
  t.sb_p = ta.sb_p;
  t.sb_q = ta.sb_q;
  t.bsb = ta.nb ? ta.bsb[0] : 0;
  t.batched = nbatch > 1 ? 1 : 0;  // the same rule as tma_encode's rank
  t.err = err;
  auto launch = [&](auto kernel, int SMEM) -> int {
    // per call: the attribute belongs to the current device
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM) != cudaSuccess) {
      (void)cudaGetLastError();
      return -1;
    }
    const int per_sm = blocks_per_sm_smem(reinterpret_cast<const void*>(kernel), kTmaWarps * 32, SMEM);
    int64_t blocks = tma_cdiv(t.ntiles, kTmaWarps);
    const int64_t cap = (int64_t)sm_count() * per_sm;
    if (blocks > cap) blocks = cap;
    kernel<<<(unsigned)(blocks < 1 ? 1 : blocks), kTmaWarps * 32, SMEM, s>>>(tm, op, b, out, t);
    count_tma_launch();
    return launch_check("ew_tiled_tma");
  };
  if constexpr (NIN == 1) {
    return launch(k_ew_tiled_tma<Op, TC, TA, TB, TO, 1, 0, BOXB>, tma_smem_bytes(BOXB));
  } else {
    if (ta.sb_p == 0) return launch(k_ew_tiled_tma<Op, TC, TA, TB, TO, 2, 1, BOXB>, tma_smem_bytes(BOXB));
    return launch(k_ew_tiled_tma<Op, TC, TA, TB, TO, 2, 2, BOXB>, tma_smem_bytes(BOXB));
  }
}

// The TMA form of an EW_TILED plan; returns -1 (nothing launched) when the
// view does not meet its layout rules, so the caller uses k_ew_tiled.
template <class Op, class TC, class TA, class TB, class TO, int NIN>
int run_tiled_tma(const Op& op, const TA* a, const TB* b, TO* out, const TiledArgs& ta, cudaStream_t s) {
  constexpr int SZ = (int)sizeof(TA);
  if constexpr (SZ != 2 && SZ != 4 && SZ != 8) {
    return -1;
  } else {
    constexpr int E = 16 / SZ;
    constexpr int RUN = E * (int)sizeof(TO) < 16 ? E * (int)sizeof(TO) : 16;  // output run alignment
    // TMA coordinates are 32-bit signed
    if (!tiled_tma_enabled() || ta.nb > 1 || ta.dq % E != 0 || ta.dp >= 0x7fffffffLL || ta.dq >= 0x7fffffffLL)
      return -1;
    if (((uintptr_t)a & 15) || ((uintptr_t)out % RUN) || ta.sa_q <= 0 || (ta.sa_q * SZ) % 16 != 0) return -1;
    if ((ta.so_p * (int64_t)sizeof(TO)) % RUN != 0) return -1;
    if (ta.nb == 1 && (ta.bsa[0] <= 0 || (ta.bsa[0] * SZ) % 16 != 0 || (ta.bso[0] * (int64_t)sizeof(TO)) % RUN != 0 ||
                       ta.bshape[0] >= 0x7fffffffLL))
      return -1;
    int* err = tiled_wait_flag();
    if (!err) return -1;
    // Box width and tile grouping per element size, from sweeps on B200
    // (16384^2 2- and 4-byte transposes, 8192^2 int64-transposed + float64
    // row; boxes of 64 / 128 / 256 bytes, groups of 1 x 4 / 2 x 2 / 4 x 1
    // tiles, groups numbered q- or p-fastest): 2-byte elements 256-byte
    // boxes in 4 x 1 groups (178 us, the shared-memory tile kernel 382 us);
    // 8-byte elements 128-byte boxes in 4 x 1 groups (179 us; 2 x 2 groups
    // 185 us, 256-byte boxes 193-199 us). For 4-byte elements the
    // shared-memory tile kernel stays faster (362 us vs 390 us at best).
    if constexpr (SZ == 2) {
      return launch_tiled_tma<Op, TC, TA, TB, TO, NIN, 256, 2>(op, a, b, out, ta, err, s);
    } else if constexpr (SZ == 8) {
      return launch_tiled_tma<Op, TC, TA, TB, TO, NIN, 128, 2>(op, a, b, out, ta, err, s);
    } else {
      return -1;
    }
  }
}

}  // namespace ew
}  // namespace mpb
