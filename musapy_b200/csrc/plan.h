// Host-side planning shared by the elementwise, reduction and scan engines.
//
// musapy's kernels walk every element through offset_nd, a per-element loop
// of 64-bit div/mod over all dims (kernels/include/common.h:42-51,
// reduce_input_offset :64-79). Here that work moves to the host: dims of
// extent 1 are dropped and adjacent dims are merged whenever every operand
// allows it, so the device loops see the fewest dims possible and can pick
// a vectorised or tiled kernel.
#pragma once
#include <stdint.h>
#include <string.h>
#include "mpb_types.h"

namespace mpb {

constexpr int kMaxCollapsed = 12;  // dims left after collapsing (device limit)

struct Geometry {
  int ndim = 0;             // collapsed ndim (>= 1 when numel > 0)
  int nops = 0;             // operands described (inputs followed by output)
  int64_t shape[MPB_MAX_DIMS];
  int64_t st[3][MPB_MAX_DIMS];  // element strides per operand
  int64_t numel = 0;
};

// Collapse `ndim` dims of `shape` for `nops` operands with strides st[k].
// Dims of extent 1 are dropped; dims i, i+1 are merged when
// st[k][i] == st[k][i+1] * shape[i+1] for every operand k.
inline Geometry collapse(int ndim, const int64_t* shape, int nops, const int64_t* const* strides) {
  Geometry g;
  g.nops = nops;
  g.numel = 1;
  for (int i = 0; i < ndim; ++i) g.numel *= shape[i];
  int k = 0;
  for (int i = 0; i < ndim; ++i) {
    if (shape[i] == 1) continue;
    g.shape[k] = shape[i];
    for (int o = 0; o < nops; ++o) g.st[o][k] = strides[o][i];
    ++k;
  }
  if (k == 0 || g.numel == 0) {  // scalar (or empty) -> one dim of extent numel
    g.ndim = 1;
    g.shape[0] = g.numel;
    for (int o = 0; o < nops; ++o) g.st[o][0] = 1;
    return g;
  }
  // merge from the inside out
  int out = k - 1;
  int64_t sh[MPB_MAX_DIMS];
  int64_t st[3][MPB_MAX_DIMS];
  sh[out] = g.shape[k - 1];
  for (int o = 0; o < nops; ++o) st[o][out] = g.st[o][k - 1];
  for (int i = k - 2; i >= 0; --i) {
    bool ok = true;
    for (int o = 0; o < nops && ok; ++o) ok = (g.st[o][i] == st[o][out] * sh[out]);
    if (ok) {
      sh[out] *= g.shape[i];
    } else {
      --out;
      sh[out] = g.shape[i];
      for (int o = 0; o < nops; ++o) st[o][out] = g.st[o][i];
    }
  }
  g.ndim = k - out;
  for (int i = 0; i < g.ndim; ++i) {
    g.shape[i] = sh[out + i];
    for (int o = 0; o < nops; ++o) g.st[o][i] = st[o][out + i];
  }
  return g;
}

// Largest element offset reachable (positive and negative parts) for bounds
// pre-checks and index-width selection.
inline void offset_span(const Geometry& g, int op, int64_t* lo, int64_t* hi) {
  int64_t l = 0, h = 0;
  for (int i = 0; i < g.ndim; ++i) {
    int64_t d = (g.shape[i] - 1) * g.st[op][i];
    if (d < 0) l += d; else h += d;
  }
  *lo = l;
  *hi = h;
}

inline int dtype_size(int dt) {
  switch (dt) {
    case MPB_BOOL: case MPB_I8: case MPB_U8: return 1;
    case MPB_I16: case MPB_U16: case MPB_F16: case MPB_BF16: return 2;
    case MPB_I32: case MPB_U32: case MPB_F32: return 4;
    case MPB_I64: case MPB_U64: case MPB_F64: case MPB_C64: return 8;
    case MPB_C128: return 16;
    default: return 0;
  }
}
inline bool is_complex(int dt) { return dt == MPB_C64 || dt == MPB_C128; }
inline bool is_float(int dt) { return dt == MPB_F16 || dt == MPB_F32 || dt == MPB_F64 || dt == MPB_BF16; }
inline bool is_int(int dt) { return (dt >= MPB_I8 && dt <= MPB_U64); }

// Elementwise kernel classes.
enum EwKind {
  EW_CONTIG = 0,   // 1-D, every input unit-stride or scalar, 16-byte aligned
  EW_ROWS = 1,     // >= 2-D, inner dim unit-stride or broadcast for all, vector aligned
  EW_TILED = 2,    // an input's unit stride lies on an outer dim: smem transpose
  EW_ND = 3,       // general strided, warp-strided scalar access
};

}  // namespace mpb
