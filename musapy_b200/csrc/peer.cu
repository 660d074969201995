// Record exchange between the GPUs of one node over NVLink peer memory.
//
// A sharded full reduction ends with every rank holding one small record
// (an f64 partial sum, or a 16-byte (value, index) argmax record) that all
// ranks need in rank order. A library collective for 8-32 bytes costs tens
// of microseconds of launch and protocol latency; here each rank's kernel
// stores its record straight into every peer's exchange buffer (P2P stores
// through NVSwitch), raises a per-rank flag there, and waits for the other
// ranks' flags in its own buffer - one kernel, one block, a few microseconds.
//
// Exchange buffer (one per rank, cudaMalloc'd, shared by CUDA IPC):
//   records[2][kPeerMaxRanks][32 bytes]  parity (seq & 1) x writer rank
//   flags  [2][kPeerMaxRanks] uint64     last seq each writer completed
// Exchange `seq` (1, 2, 3, ... identical on all ranks, one per call) uses
// parity seq & 1. Two parities suffice: a rank starts exchange k+2, which
// overwrites parity k's records in a peer's buffer, only after it saw that
// peer's flag for k+1, and the peer raises it only after it finished reading
// exchange k. Every wait is bounded: after ~2 s a rank gives up, records
// MPB_ERR_TIMEOUT in `status` and returns (the host checks it), so a missing
// rank cannot hang the GPU.
#include <cstring>
#include "common.cuh"
#include "internal.h"
#include "musapy_b200.h"

namespace mpb {
namespace {

constexpr int kPeerMaxRanks = 16;
constexpr int kRecBytes = 32;
constexpr size_t kRecordsOff = 0;
constexpr size_t kFlagsOff = 2 * kPeerMaxRanks * kRecBytes;
constexpr size_t kPeerBufBytes = kFlagsOff + 2 * kPeerMaxRanks * sizeof(unsigned long long);
constexpr long long kSpinLimit = 1ll << 24;  // x ~128 ns sleeps: ~2 s

struct PeerPtrs {
  char* p[kPeerMaxRanks];
};

MPB_D size_t rec_off(int par, int writer) { return kRecordsOff + ((size_t)par * kPeerMaxRanks + writer) * kRecBytes; }
MPB_D size_t flag_off(int par, int writer) {
  return kFlagsOff + ((size_t)par * kPeerMaxRanks + writer) * sizeof(unsigned long long);
}

MPB_D void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
MPB_D unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__global__ void k_peer_allgather(const uint4* __restrict__ rec, int rec_words, PeerPtrs peers, int rank, int world,
                                 unsigned long long seq, uint4* __restrict__ out, int* status) {
  const int t = threadIdx.x;
  const int par = (int)(seq & 1ull);
  if (t < world) {
    // my record into rank t's buffer, then my flag there
    uint4* dst = reinterpret_cast<uint4*>(peers.p[t] + rec_off(par, rank));
    for (int w = 0; w < rec_words; ++w) dst[w] = rec[w];
    __threadfence_system();
    st_release_sys(reinterpret_cast<unsigned long long*>(peers.p[t] + flag_off(par, rank)), seq);
  }
  if (t < world) {
    // rank t's record in my buffer
    const char* mine = peers.p[rank];
    const unsigned long long* f = reinterpret_cast<const unsigned long long*>(mine + flag_off(par, t));
    long long it = 0;
    bool ok = true;
    while (ld_acquire_sys(f) < seq) {
      if (++it > kSpinLimit) {
        ok = false;
        break;
      }
      __nanosleep(128);
    }
    if (!ok) {
      atomicExch(status, MPB_ERR_TIMEOUT);
    } else {
      const uint4* src = reinterpret_cast<const uint4*>(mine + rec_off(par, t));
      for (int w = 0; w < rec_words; ++w) out[(size_t)t * rec_words + w] = src[w];
    }
  }
}

// sum of `world` f64 partials in rank order (deterministic, the same on
// every rank), then sum and mean in the array dtype
__global__ void k_sum_parts_finalize(const double* __restrict__ parts, int stride_words, int world, double count,
                                     int out_dt, void* sum_out, void* mean_out) {
  if (threadIdx.x != 0) return;
  double s = 0.0;
  for (int r = 0; r < world; ++r) s += parts[(size_t)r * stride_words];
  const double m = s / count;
  if (out_dt == MPB_F32) {
    *static_cast<float*>(sum_out) = (float)s;
    *static_cast<float*>(mean_out) = (float)m;
  } else {
    *static_cast<double*>(sum_out) = s;
    *static_cast<double*>(mean_out) = m;
  }
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
  if (world < 1 || world > kPeerMaxRanks || rank < 0 || rank >= world)
    return fail(MPB_ERR_INVALID, "mpb_peer_allgather: rank %d / world %d out of range (max %d ranks)", rank, world,
                kPeerMaxRanks);
  if (rec_bytes <= 0 || rec_bytes > kRecBytes || rec_bytes % 16 != 0)
    return fail(MPB_ERR_INVALID, "mpb_peer_allgather: record size %d must be 16 or 32 bytes", rec_bytes);
  if (seq == 0) return fail(MPB_ERR_INVALID, "mpb_peer_allgather: seq starts at 1");
  if (!rec || !peers || !out || !status) return fail(MPB_ERR_INVALID, "mpb_peer_allgather: null pointer");
  if (((uintptr_t)rec | (uintptr_t)out) & 15) return fail(MPB_ERR_INVALID, "mpb_peer_allgather: records must be 16-byte aligned");
  PeerPtrs pp{};
  for (int r = 0; r < world; ++r) {
    if (!peers[r]) return fail(MPB_ERR_INVALID, "mpb_peer_allgather: null buffer for rank %d", r);
    pp.p[r] = static_cast<char*>(peers[r]);
  }
  k_peer_allgather<<<1, 32, 0, (cudaStream_t)stream>>>(static_cast<const uint4*>(rec), rec_bytes / 16, pp, rank,
                                                       world, (unsigned long long)seq, static_cast<uint4*>(out),
                                                       status);
  return launch_check("peer_allgather");
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
