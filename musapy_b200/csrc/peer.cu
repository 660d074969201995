// Record exchange between the GPUs of one node over NVLink peer memory.
//
// A sharded full reduction ends with every rank holding one small record
// (an f64 partial sum, or a 16-byte (value, index) argmax record) that all
// ranks need in rank order. A library collective for 8-32 bytes costs tens
// of microseconds of launch and protocol latency; here each rank's kernel
// stores its record straight into every peer's exchange buffer (P2P stores
// through NVSwitch) and reads the other ranks' records from its own buffer -
// one kernel of one warp. The fused forms (mpb_peer_sum_finalize,
// mpb_peer_arg_combine) also finish the reduction in the same kernel, so a
// sharded sum or argmax ends with two launches per rank: the local
// reduction and this one.
//
// Wire format: flag-in-line words. Each 16-byte store carries two 4-byte
// data words, each paired with the exchange's 32-bit sequence number
// {d0, seq, d1, seq}; a reader polls with 16-byte loads until both sequence
// halves match. Every 8-byte {data, flag} half lands atomically, so no
// memory fence and no separate flag store are needed (the scheme of NCCL's
// low-latency protocol, restated here for records of 8-32 bytes).
//
// Exchange buffer (one per rank, cudaMalloc'd, shared by CUDA IPC):
//   slots[2][kPeerMaxRanks][64 bytes]   parity (seq & 1) x writer rank
// Exchange `seq` (1, 2, 3, ... identical on all ranks, one per call) uses
// parity seq & 1. Two parities suffice: a rank starts exchange k+2, which
// overwrites parity k's slots in a peer's buffer, only after it received
// that peer's record of exchange k+1, which the peer sends only after it
// finished reading exchange k. A stale slot holds seq - 2 (or the zeros of
// the fresh buffer; seq starts at 1), never seq, also after the 32-bit
// sequence wraps. Every wait is bounded: after 2 s a rank gives up, records
// MPB_ERR_TIMEOUT in `status`, writes no result and returns (the host checks
// it), so a missing rank cannot hang the GPU.
#include <cstring>
#include "common.cuh"
#include "internal.h"
#include "musapy_b200.h"
#include "shard_combine.cuh"

namespace mpb {
namespace {

constexpr int kPeerMaxRanks = 16;
constexpr int kRecBytes = 32;                // largest record
constexpr int kSlotBytes = 2 * kRecBytes;    // a record as flag-in-line words
constexpr size_t kPeerBufBytes = (size_t)2 * kPeerMaxRanks * kSlotBytes;
constexpr unsigned long long kWaitNs = 2000000000ull;  // per wait, by the global timer
constexpr long long kSpinLimit = 1ll << 26;             // second bound, should the timer stall

struct PeerPtrs {
  char* p[kPeerMaxRanks];
};
struct PeerOffsets {
  int64_t off[kPeerMaxRanks];
};

MPB_D unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

MPB_D size_t slot_off(int par, int writer) { return ((size_t)par * kPeerMaxRanks + writer) * kSlotBytes; }

MPB_D void ll_store(char* dst, uint32_t d0, uint32_t d1, uint32_t seq) {
  asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(dst), "r"(d0), "r"(seq), "r"(d1), "r"(seq)
               : "memory");
}

MPB_D bool ll_load(const char* src, uint32_t seq, uint32_t& d0, uint32_t& d1) {
  uint32_t f0, f1;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(d0), "=r"(f0), "=r"(d1), "=r"(f1)
               : "l"(src)
               : "memory");
  return f0 == seq && f1 == seq;
}

// Lane t < world sends this rank's record (`words` 32-bit words, even) to
// rank t, then receives rank t's record into got[t * words ...]. Returns
// false in the lanes whose wait ran out.
MPB_D bool ll_exchange(const uint32_t* __restrict__ rec, int words, const PeerPtrs& peers, int rank, int world,
                       unsigned long long seq, uint32_t* got) {
  const int t = threadIdx.x;
  if (t >= world) return true;
  const int par = (int)(seq & 1ull);
  const uint32_t s32 = (uint32_t)seq;
  char* dst = peers.p[t] + slot_off(par, rank);
  for (int l = 0; l < words / 2; ++l) ll_store(dst + 16 * l, rec[2 * l], rec[2 * l + 1], s32);
  const char* src = peers.p[rank] + slot_off(par, t);
  const unsigned long long t0 = global_ns();
  long long it = 0;
  for (int l = 0; l < words / 2; ++l) {
    uint32_t d0, d1;
    while (!ll_load(src + 16 * l, s32, d0, d1)) {
      if (++it > kSpinLimit || global_ns() - t0 > kWaitNs) return false;
      __nanosleep(64);
    }
    got[t * words + 2 * l] = d0;
    got[t * words + 2 * l + 1] = d1;
  }
  return true;
}

// One warp: exchange, then `finish` on lane 0 when every lane received.
template <class Finish>
MPB_D void exchange_then(const uint32_t* rec, int words, const PeerPtrs& peers, int rank, int world,
                         unsigned long long seq, int* status, Finish finish) {
  __shared__ __align__(16) uint32_t got[kPeerMaxRanks * (kRecBytes / 4)];
  const bool ok = ll_exchange(rec, words, peers, rank, world, seq, got);
  const bool all_ok = __all_sync(0xffffffffu, ok);
  if (!all_ok) {
    if (threadIdx.x == 0) atomicExch(status, MPB_ERR_TIMEOUT);
    return;
  }
  __syncwarp();
  if (threadIdx.x == 0) finish(got);
}

__global__ void k_peer_allgather(const uint32_t* __restrict__ rec, int words, PeerPtrs peers, int rank, int world,
                                 unsigned long long seq, uint32_t* __restrict__ out, int* status) {
  exchange_then(rec, words, peers, rank, world, seq, status, [&](const uint32_t* got) {
    for (int i = 0; i < world * words; ++i) out[i] = got[i];
  });
}

// The fused exchange kernels below run one rank per block: block b plays
// rank `rank + b`, with its record at rec + b * (record words) and its
// results at out + b. A rank's own launch has one block (b = 0: the rank,
// record and outputs it was given). A launch of `world` blocks on one GPU,
// cooperative so that every block is resident at once, plays all ranks of an
// exchange over buffers of that GPU (mpb_peer_*_emulated): the same code,
// protocol and combine, checkable without several GPUs.

// Records are f64 partial sums (two words); summed in rank order, so every
// rank computes the same value.
__global__ void k_peer_sum_finalize(const uint32_t* __restrict__ partial, PeerPtrs peers, int rank, int world,
                                    unsigned long long seq, double count, int out_dt, void* sum_out, void* mean_out,
                                    int* status) {
  const int b = blockIdx.x;
  const size_t osz = out_dt == MPB_F32 ? 4 : 8;
  char* so = sum_out ? static_cast<char*>(sum_out) + b * osz : nullptr;
  char* mo = mean_out ? static_cast<char*>(mean_out) + b * osz : nullptr;
  exchange_then(partial + 2 * b, 2, peers, rank + b, world, seq, status, [&](const uint32_t* got) {
    double s = 0.0;
    for (int r = 0; r < world; ++r) s += __hiloint2double((int)got[2 * r + 1], (int)got[2 * r]);
    shard_sum_write(s, count, out_dt, so, mo);
  });
}

__global__ void k_peer_arg_combine(const uint32_t* __restrict__ rec, PeerPtrs peers, int rank, int world,
                                   unsigned long long seq, PeerOffsets offs, int is_max, int is_int,
                                   int64_t* out_index, double* out_value, int* status) {
  const int b = blockIdx.x;
  exchange_then(rec + 4 * b, 4, peers, rank + b, world, seq, status, [&](const uint32_t* got) {
    shard_arg_combine(reinterpret_cast<const int64_t*>(got), world, offs.off, is_max, is_int, out_index + b,
                      out_value ? out_value + b : nullptr);
  });
}

// sum of `world` f64 partials in rank order (deterministic, the same on
// every rank), then sum and mean in the array dtype
__global__ void k_sum_parts_finalize(const double* __restrict__ parts, int stride_words, int world, double count,
                                     int out_dt, void* sum_out, void* mean_out) {
  if (threadIdx.x != 0) return;
  double s = 0.0;
  for (int r = 0; r < world; ++r) s += parts[(size_t)r * stride_words];
  shard_sum_write(s, count, out_dt, sum_out, mean_out);
}

int check_ranks(const char* what, int rank, int world) {
  if (world < 1 || world > kPeerMaxRanks || rank < 0 || rank >= world)
    return fail(MPB_ERR_INVALID, "%s: rank %d / world %d out of range (max %d ranks)", what, rank, world,
                kPeerMaxRanks);
  return MPB_OK;
}

int peer_ptrs(const char* what, void* const* peers, int world, unsigned long long seq, PeerPtrs& pp) {
  if (seq == 0) return fail(MPB_ERR_INVALID, "%s: seq starts at 1", what);
  if (!peers) return fail(MPB_ERR_INVALID, "%s: null peer table", what);
  for (int r = 0; r < world; ++r) {
    if (!peers[r]) return fail(MPB_ERR_INVALID, "%s: null buffer for rank %d", what, r);
    if ((uintptr_t)peers[r] & 15) return fail(MPB_ERR_INVALID, "%s: buffer of rank %d not 16-byte aligned", what, r);
    pp.p[r] = static_cast<char*>(peers[r]);
  }
  return MPB_OK;
}

}  // namespace
}  // namespace mpb

using namespace mpb;

extern "C" {

size_t mpb_peer_buffer_bytes(void) { return kPeerBufBytes; }

int mpb_peer_alloc(void** buf, void* ipc_handle) {
  if (!buf || !ipc_handle) return fail(MPB_ERR_INVALID, "mpb_peer_alloc: null pointer");
  void* p = nullptr;
  int rc = cuda_check(cudaMalloc(&p, kPeerBufBytes), "mpb_peer_alloc: cudaMalloc");
  if (rc != MPB_OK) return rc;
  if ((rc = cuda_check(cudaMemset(p, 0, kPeerBufBytes), "mpb_peer_alloc: cudaMemset")) != MPB_OK) {
    cudaFree(p);
    return rc;
  }
  cudaIpcMemHandle_t h;
  if ((rc = cuda_check(cudaIpcGetMemHandle(&h, p), "mpb_peer_alloc: cudaIpcGetMemHandle")) != MPB_OK) {
    cudaFree(p);
    return rc;
  }
  memcpy(ipc_handle, &h, sizeof(h));
  *buf = p;
  return MPB_OK;
}

size_t mpb_peer_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

int mpb_peer_open(const void* ipc_handle, void** peer_buf) {
  if (!ipc_handle || !peer_buf) return fail(MPB_ERR_INVALID, "mpb_peer_open: null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  return cuda_check(cudaIpcOpenMemHandle(peer_buf, h, cudaIpcMemLazyEnablePeerAccess), "mpb_peer_open");
}

int mpb_peer_close(void* peer_buf) { return cuda_check(cudaIpcCloseMemHandle(peer_buf), "mpb_peer_close"); }

int mpb_peer_free(void* buf) { return cuda_check(cudaFree(buf), "mpb_peer_free"); }

int mpb_peer_allgather(const void* rec, int rec_bytes, void* const* peers, int rank, int world, uint64_t seq,
                       void* out, int* status, mpb_stream_t stream) {
  int rc = check_ranks("mpb_peer_allgather", rank, world);
  if (rc) return rc;
  if (rec_bytes <= 0 || rec_bytes > kRecBytes || rec_bytes % 8 != 0)
    return fail(MPB_ERR_INVALID, "mpb_peer_allgather: record size %d must be 8, 16, 24 or 32 bytes", rec_bytes);
  if (!rec || !out || !status) return fail(MPB_ERR_INVALID, "mpb_peer_allgather: null pointer");
  if (((uintptr_t)rec | (uintptr_t)out) & 7) return fail(MPB_ERR_INVALID, "mpb_peer_allgather: records must be 8-byte aligned");
  PeerPtrs pp{};
  if ((rc = peer_ptrs("mpb_peer_allgather", peers, world, seq, pp))) return rc;
  k_peer_allgather<<<1, 32, 0, (cudaStream_t)stream>>>(static_cast<const uint32_t*>(rec), rec_bytes / 4, pp, rank,
                                                       world, (unsigned long long)seq, static_cast<uint32_t*>(out),
                                                       status);
  return launch_check("peer_allgather");
}

int mpb_peer_sum_finalize(const double* partial, void* const* peers, int rank, int world, uint64_t seq, double count,
                          int out_dtype, void* sum_out, void* mean_out, int* status, mpb_stream_t stream) {
  int rc = check_ranks("mpb_peer_sum_finalize", rank, world);
  if (rc) return rc;
  if (out_dtype != MPB_F32 && out_dtype != MPB_F64)
    return fail(MPB_ERR_DTYPE, "mpb_peer_sum_finalize: output dtype must be f32 or f64");
  if (!partial || !status) return fail(MPB_ERR_INVALID, "mpb_peer_sum_finalize: null pointer");
  PeerPtrs pp{};
  if ((rc = peer_ptrs("mpb_peer_sum_finalize", peers, world, seq, pp))) return rc;
  k_peer_sum_finalize<<<1, 32, 0, (cudaStream_t)stream>>>(reinterpret_cast<const uint32_t*>(partial), pp, rank, world,
                                                          (unsigned long long)seq, count, out_dtype, sum_out,
                                                          mean_out, status);
  return launch_check("peer_sum_finalize");
}

int mpb_peer_arg_combine(const int64_t* record, void* const* peers, int rank, int world, uint64_t seq,
                         const int64_t* rank_offsets, int is_max, int is_int, int64_t* out_index, double* out_value,
                         int* status, mpb_stream_t stream) {
  int rc = check_ranks("mpb_peer_arg_combine", rank, world);
  if (rc) return rc;
  if (!record || !rank_offsets || !out_index || !status)
    return fail(MPB_ERR_INVALID, "mpb_peer_arg_combine: null pointer");
  PeerPtrs pp{};
  if ((rc = peer_ptrs("mpb_peer_arg_combine", peers, world, seq, pp))) return rc;
  PeerOffsets po{};
  for (int r = 0; r < world; ++r) po.off[r] = rank_offsets[r];
  k_peer_arg_combine<<<1, 32, 0, (cudaStream_t)stream>>>(reinterpret_cast<const uint32_t*>(record), pp, rank, world,
                                                         (unsigned long long)seq, po, is_max, is_int, out_index,
                                                         out_value, status);
  return launch_check("peer_arg_combine");
}

int mpb_peer_sum_finalize_emulated(const double* partials, void* const* bufs, int world, uint64_t seq, double count,
                                   int out_dtype, void* sum_out, void* mean_out, int* status, mpb_stream_t stream) {
  int rc = check_ranks("mpb_peer_sum_finalize_emulated", 0, world);
  if (rc) return rc;
  if (out_dtype != MPB_F32 && out_dtype != MPB_F64)
    return fail(MPB_ERR_DTYPE, "mpb_peer_sum_finalize_emulated: output dtype must be f32 or f64");
  if (!partials || !status) return fail(MPB_ERR_INVALID, "mpb_peer_sum_finalize_emulated: null pointer");
  PeerPtrs pp{};
  if ((rc = peer_ptrs("mpb_peer_sum_finalize_emulated", bufs, world, seq, pp))) return rc;
  const uint32_t* rec = reinterpret_cast<const uint32_t*>(partials);
  int rank0 = 0;
  unsigned long long sq = (unsigned long long)seq;
  void* args[] = {(void*)&rec, (void*)&pp, (void*)&rank0, (void*)&world, (void*)&sq, (void*)&count,
                  (void*)&out_dtype, (void*)&sum_out, (void*)&mean_out, (void*)&status};
  const cudaError_t e = cudaLaunchCooperativeKernel((const void*)k_peer_sum_finalize, dim3(world), dim3(32), args, 0,
                                                    (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_check(e, "peer_sum_finalize_emulated");
  return launch_check("peer_sum_finalize_emulated");
}

int mpb_peer_arg_combine_emulated(const int64_t* records, void* const* bufs, int world, uint64_t seq,
                                  const int64_t* rank_offsets, int is_max, int is_int, int64_t* out_index,
                                  double* out_value, int* status, mpb_stream_t stream) {
  int rc = check_ranks("mpb_peer_arg_combine_emulated", 0, world);
  if (rc) return rc;
  if (!records || !rank_offsets || !out_index || !status)
    return fail(MPB_ERR_INVALID, "mpb_peer_arg_combine_emulated: null pointer");
  PeerPtrs pp{};
  if ((rc = peer_ptrs("mpb_peer_arg_combine_emulated", bufs, world, seq, pp))) return rc;
  PeerOffsets po{};
  for (int r = 0; r < world; ++r) po.off[r] = rank_offsets[r];
  const uint32_t* rec = reinterpret_cast<const uint32_t*>(records);
  int rank0 = 0;
  unsigned long long sq = (unsigned long long)seq;
  void* args[] = {(void*)&rec, (void*)&pp, (void*)&rank0, (void*)&world, (void*)&sq, (void*)&po,
                  (void*)&is_max, (void*)&is_int, (void*)&out_index, (void*)&out_value, (void*)&status};
  const cudaError_t e = cudaLaunchCooperativeKernel((const void*)k_peer_arg_combine, dim3(world), dim3(32), args, 0,
                                                    (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_check(e, "peer_arg_combine_emulated");
  return launch_check("peer_arg_combine_emulated");
}

int mpb_shard_sum_parts_finalize(const double* parts, int stride_bytes, int world, double count, int out_dtype,
                                 void* sum_out, void* mean_out, mpb_stream_t stream) {
  if (out_dtype != MPB_F32 && out_dtype != MPB_F64)
    return fail(MPB_ERR_DTYPE, "mpb_shard_sum_parts_finalize: output dtype must be f32 or f64");
  if (stride_bytes % 8 != 0 || world < 1) return fail(MPB_ERR_INVALID, "mpb_shard_sum_parts_finalize: bad layout");
  k_sum_parts_finalize<<<1, 32, 0, (cudaStream_t)stream>>>(parts, stride_bytes / 8, world, count, out_dtype, sum_out,
                                                           mean_out);
  return launch_check("sum_parts_finalize");
}

}  // extern "C"
