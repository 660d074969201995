// Combine steps of axis-0 sharded reductions (one process per GPU).
//
// musapy has no multi-GPU code (docs/adr/ADR.md:896-906); these kernels are
// the device-side halves of the new sharded path: after each rank reduces
// its rows, one tiny record per rank crosses to the other ranks and these
// kernels finish on the device, so no host round trip is needed. They serve
// the NCCL transport (MUSAPY_B200_SHARD_COLLECTIVE=nccl: an all_reduce or
// all_gather moves the records, then one of these kernels combines them);
// the default transport, the peer-memory exchange of peer.cu, fuses the
// same combine (shard_combine.cuh) into its exchange kernel.
#include <math.h>
#include <stdint.h>
#include "common.cuh"
#include "internal.h"
#include "shard_combine.cuh"

namespace mpb {
namespace {

constexpr int kMaxRanks = kShardMaxRanks;
struct RankOffsets {
  int64_t off[kMaxRanks];
};

// recs: n all-gathered records {value bits, local index} in rank order.
__global__ void k_arg_combine(const int64_t* __restrict__ recs, int n, RankOffsets ro, int is_max, int is_int,
                              int64_t* __restrict__ out_index, double* __restrict__ out_value) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  shard_arg_combine(recs, n, ro.off, is_max, is_int, out_index, out_value);
}

// Sum combine: `total` holds the all-reduced f64 sum; write the sum and the
// mean (true element count) in the array dtype.
__global__ void k_sum_finalize(const double* __restrict__ total, double count, int out_dt, void* sum_out,
                               void* mean_out) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  shard_sum_write(*total, count, out_dt, sum_out, mean_out);
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
