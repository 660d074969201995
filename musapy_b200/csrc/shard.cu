// Combine steps of axis-0 sharded reductions (one process per GPU).
//
// musapy has no multi-GPU code (docs/adr/ADR.md:896-906); these kernels are
// the device-side halves of the new sharded path: after each rank reduces
// its rows, the host moves one tiny record per rank with one NCCL collective
// and these kernels finish on the device, so no host round trip is needed.
#include <math.h>
#include <stdint.h>
#include "common.cuh"
#include "internal.h"

namespace mpb {
namespace {

constexpr int kMaxRanks = 64;
struct RankOffsets {
  int64_t off[kMaxRanks];
};

// recs: n records {value bits, local index} in rank order (all-gathered).
// Rank 0 applies the first-element NaN rule, so a (NaN, 0) record from rank
// 0 decides the answer; every other record never holds a NaN. Strict
// comparison in rank order keeps the first occurrence.
__global__ void k_arg_combine(const int64_t* __restrict__ recs, int n, RankOffsets ro, int is_max, int is_int,
                              int64_t* __restrict__ out_index, double* __restrict__ out_value) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
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
        best_i = li + ro.off[r];
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
        best_i = li + ro.off[r];
        have = true;
      }
    }
  }
  *out_index = have ? best_i : 0;
  if (out_value) *out_value = is_int ? (double)best_v : best_d;
}

// Sum combine: `total` holds the all-reduced f64 sum; write the sum and the
// mean (true element count) in the array dtype.
__global__ void k_sum_finalize(const double* __restrict__ total, double count, int out_dt, void* sum_out,
                               void* mean_out) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  const double t = *total;
  const double m = t / count;
  if (out_dt == MPB_F32) {
    if (sum_out) *static_cast<float*>(sum_out) = __double2float_rn(t);
    if (mean_out) *static_cast<float*>(mean_out) = __double2float_rn(m);
  } else {
    if (sum_out) *static_cast<double*>(sum_out) = t;
    if (mean_out) *static_cast<double*>(mean_out) = m;
  }
}

}  // namespace
}  // namespace mpb

using namespace mpb;

extern "C" {

int mpb_shard_arg_combine(const int64_t* recs, int nranks, const int64_t* rank_offsets, int is_max, int is_int,
                          int64_t* out_index, double* out_value, cudaStream_t stream) {
  if (nranks < 1 || nranks > kMaxRanks) return fail(MPB_ERR_INVALID, "arg combine: %d ranks (max %d)", nranks, kMaxRanks);
  RankOffsets ro;
  for (int r = 0; r < nranks; ++r) ro.off[r] = rank_offsets[r];
  k_arg_combine<<<1, 32, 0, stream>>>(recs, nranks, ro, is_max, is_int, out_index, out_value);
  return launch_check("shard_arg_combine");
}

int mpb_shard_sum_finalize(const double* total, double count, int out_dtype, void* sum_out, void* mean_out,
                           cudaStream_t stream) {
  if (out_dtype != MPB_F32 && out_dtype != MPB_F64) return fail(MPB_ERR_DTYPE, "sum finalize: dtype %d", out_dtype);
  k_sum_finalize<<<1, 32, 0, stream>>>(total, count, out_dtype, sum_out, mean_out);
  return launch_check("shard_sum_finalize");
}

}  // extern "C"
