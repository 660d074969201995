// Final combine of axis-0 sharded full reductions, shared by the kernels
// that run it after a library collective (shard.cu) and the kernels that
// fuse it with the NVLink record exchange (peer.cu). Run by one thread.
#pragma once
#include <math.h>
#include <stdint.h>
#include "common.cuh"

namespace mpb {

constexpr int kShardMaxRanks = 64;

// recs: n records {value bits, local index} in rank order; offs[r] = global
// flat index of rank r's first element. Rank 0 applies the first-element
// NaN rule, so a (NaN, 0) record from rank 0 decides the answer; every other
// record never holds a NaN. A record with index INT64_MAX is empty (a rank
// without elements). Strict comparison in rank order keeps the first
// occurrence (musapy's sequential strict compare, op_builder.rs:3496-3582).
MPB_D void shard_arg_combine(const int64_t* recs, int n, const int64_t* offs, int is_max, int is_int,
                             int64_t* out_index, double* out_value) {
  int64_t best_i = INT64_MAX;
  double best_d = 0.0;
  int64_t best_v = 0;
  bool have = false;
  for (int r = 0; r < n; ++r) {
    const int64_t vb = recs[2 * r], li = recs[2 * r + 1];
    if (li == INT64_MAX) continue;
    if (is_int) {
      if (!have || (is_max ? vb > best_v : vb < best_v)) {
        best_v = vb;
        best_i = li + offs[r];
        have = true;
      }
    } else {
      const double v = __longlong_as_double(vb);
      if (r == 0 && li == 0 && v != v) {  // NaN first element
        best_d = v;
        best_i = 0;
        have = true;
        break;
      }
      if (!have || (is_max ? v > best_d : v < best_d)) {
        best_d = v;
        best_i = li + offs[r];
        have = true;
      }
    }
  }
  *out_index = have ? best_i : 0;
  if (out_value) *out_value = is_int ? (double)best_v : best_d;
}

// Global f64 sum -> sum and mean (true element count) in the array dtype.
MPB_D void shard_sum_write(double total, double count, int out_dt, void* sum_out, void* mean_out) {
  const double m = total / count;
  if (out_dt == MPB_F32) {
    if (sum_out) *static_cast<float*>(sum_out) = __double2float_rn(total);
    if (mean_out) *static_cast<float*>(mean_out) = __double2float_rn(m);
  } else {
    if (sum_out) *static_cast<double*>(sum_out) = total;
    if (mean_out) *static_cast<double*>(mean_out) = m;
  }
}

}  // namespace mpb
