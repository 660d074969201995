/*
 * libmusapy_b200 - musapy's stride-aware elementwise and reduction engine
 * for NVIDIA B200 (sm_100a). Public C-ABI.
 *
 * Two families of entry points:
 *
 *  1. Extended entry points (mpb_*): one call per musapy operator, a dtype tag
 *     per operand (promotion casts are fused into the kernels), an int status
 *     return, caller-owned scratch. These are what the Python surface
 *     (musapy_b200) binds, and what a host layer in any language should bind.
 *     They replace the per-dtype kernel wrappers that musapy's operator layer
 *     calls from rust/musapy-ops/src/op_builder.rs (launch_binary! ...
 *     launch_argreduce_partial!, :38-223, and the cast/cumsum dispatch at
 *     :968-1045 and :3321-3330).
 *
 *  2. Reference-named kernel symbols (musapy_<op>_<dtype>_v2 / _v3), declared
 *     in include/musapy_kernels_v2.h: the exact set and signatures of
 *     rust/musapy-ops/src/kernels.rs:16-343, so a CUDA build of musapy's Rust
 *     layers can link this library unchanged.
 *
 * Conventions (shared with musapy's kernel contract, docs/adr/ADR.md:322-338):
 *  - strides and offsets are in ELEMENTS and may be 0 (broadcast) or negative
 *    (flipped views); each data pointer addresses the logical element
 *    [0, ..., 0] of its view (the view offset is already applied);
 *  - outputs are C-contiguous;
 *  - shape / stride arrays are host memory read during the call only;
 *  - every launch is asynchronous on `stream`; the library never allocates
 *    device memory (scratch is passed in) and never synchronises, except
 *    mpb_cumsum_status which reads a status word back;
 *  - dtype tags follow musapy's Dtype enum order
 *    (rust/musapy-core/src/dtype.rs:25-41), see enum mpb_dtype.
 */
#ifndef MUSAPY_B200_H
#define MUSAPY_B200_H

#include <stddef.h>
#include <stdint.h>

#include "mpb_types.h"

#ifdef __cplusplus
extern "C" {
#endif

/* cudaStream_t without requiring the CUDA headers. */
typedef struct CUstream_st* mpb_stream_t;

/* ---------------------------------------------------------------- status */

/* Message describing the last non-OK status returned on this thread. */
const char* mpb_last_error(void);
/* ABI version of this header (bumped on incompatible changes). */
int mpb_version(void);
/* Multiprocessor count of the current device (148 on B200; 148 without a device). */
int mpb_num_sms(void);
/* Number of kernels this library has launched in the process so far. */
unsigned long long mpb_launch_count(void);

/* ------------------------------------------------------- host-side helpers */

/* Result dtype of a binary op: rust/musapy-core/src/dtype.rs:302-338
 * (`promote`); all_gpu=1 selects the narrow-first rule musapy applies when
 * every input lives on the device. Returns -1 when no promotion exists. */
int mpb_promote(int a_dtype, int b_dtype, int all_gpu);

/* NumPy broadcast of two shapes: rust/musapy-ops/src/broadcast.rs:24-58
 * (`broadcast_shape`). Writes max(na, nb) extents to `out`; returns that
 * ndim, or -1 when the shapes are incompatible. */
int mpb_broadcast_shape(int na, const int64_t* a_shape, int nb, const int64_t* b_shape, int64_t* out);

/* Strides of an operand against a broadcast target:
 * rust/musapy-ops/src/broadcast.rs:71-92 (`broadcast_strides`). */
void mpb_broadcast_strides(int ndim, const int64_t* shape, const int64_t* strides, int target_ndim,
                           const int64_t* target, int64_t* out);

/* The engine's dimension collapsing (replaces the per-element offset_nd of
 * kernels/include/common.h:42-51): drops extent-1 dims and merges adjacent
 * dims that every operand allows. `strides` holds nops x ndim values;
 * writes the collapsed shape and nops x result strides; returns the
 * collapsed ndim (>= 1), or -1 on bad arguments. Host only. */
int mpb_collapse(int ndim, const int64_t* shape, int nops, const int64_t* strides, int64_t* out_shape,
                 int64_t* out_strides);

/* Kernel class the reduction planner picks (1 row_warp, 2 row_block,
 * 3 row_split, 4 col, 5 col_split, 6 gen; 0 empty) and the output count M,
 * reduced length L and split count. Host only; negative status on error. */
int mpb_reduce_plan(int ndim, const int64_t* shape, const int64_t* strides, int in_dtype, uint64_t axes_mask,
                    int64_t* M, int64_t* L, int64_t* splits);

/* mpb_reduce_plan for reduction `op` (an mpb_red_op) of an input at address
 * `a` (the column kernels' vector width depends on the op and on the
 * address's alignment), also giving the outputs each thread of a column
 * kernel (kinds 4 and 5) reduces: 1, or 2/4/8 when every group of them is
 * one aligned 8- or 16-byte load at every reduced step. No counterpart in
 * the reference (its column kernels take one output per thread). Host only;
 * `a` is not dereferenced. */
int mpb_reduce_plan_at(int op, int ndim, const int64_t* shape, const int64_t* strides, const void* a, int in_dtype,
                       uint64_t axes_mask, int64_t* M, int64_t* L, int64_t* splits, int* outputs_per_thread);

/* ------------------------------------------------------------ elementwise */

/* out = op(a[, b]) over `shape`, for every mpb_ew_op:
 *   MPB_ADD..MPB_POW   binary arithmetic; replaces musapy_{add,sub,mul,div,pow}
 *                      _{f32,f64,c64,c128}_v2 (rust/musapy-ops/src/kernels.rs:19-28,
 *                      :102-109) plus the cast temporaries of op_builder.rs:410-417
 *   MPB_EQ..MPB_GE     comparisons, out_dtype MPB_BOOL (kernels.rs:84-95, :114-117)
 *   MPB_SIN..MPB_NEG   unary math (kernels.rs:31-44, :110-113)
 *   MPB_CLAMP          p0 = lo, p1 = hi (kernels.rs:47-48)
 *   MPB_CAST           dtype conversion / strided copy (kernels.rs:51-81, :119-124)
 *   MPB_FILL           out = p0 (+ i*p1 for complex); a and b unused
 * a_strides / b_strides are already broadcast to `shape` (0 on broadcast
 * dims); b is NULL for unary ops. compute_dtype is the promoted dtype the op
 * is evaluated in; a and b are read in their own dtypes and converted in
 * registers. */
int mpb_elementwise(int op, int ndim, const int64_t* shape, const void* a, int a_dtype, const int64_t* a_strides,
                    const void* b, int b_dtype, const int64_t* b_strides, void* out, int out_dtype,
                    int compute_dtype, double p0, double p1, mpb_stream_t stream);

/* Transposed-view elementwise ops (an input with unit stride on an outer
 * dim) run through TMA tile loads when the view's layout allows it (16-byte
 * aligned base and strides, 2-, 4- or 8-byte elements); mpb_ew_set_tma(0)
 * routes them to the shared-memory tile kernel instead, (1) back, (-1)
 * queries. Returns the previous setting. No counterpart in musapy. */
int mpb_ew_set_tma(int enable);

/* TMA-tiled kernel launches in this process so far. */
uint64_t mpb_ew_tma_launches(void);

/* Synchronous: *timed_out = 1 when a TMA tile wait gave up (2 s) since the
 * last call on this device (the op's output is then incomplete), else 0;
 * clears the flag. No counterpart in musapy. */
int mpb_ew_wait_status(int* timed_out);

/* -------------------------------------------------------------- reductions */

/* Device scratch (bytes) mpb_reduce needs for this request; 0 when none. */
size_t mpb_reduce_scratch_bytes(int op, int ndim, const int64_t* shape, const int64_t* strides, const void* a,
                                int in_dtype, uint64_t axes_mask, int compute_dtype);

/* Reduce the dims set in axes_mask (bit d = dim d) with an mpb_red_op.
 * Replaces the naive / small_axis / partial / mid / final kernel families of
 * kernels.rs:139-180, :222-304 and the host path choice of
 * op_builder.rs:2310-3139 with one call. The output is C-contiguous over the
 * kept dims in order. nan_first_rule=1 applies musapy's CPU rule for
 * max/min/argmax/argmin (a NaN is the answer only when it is the first
 * element). Multiple axes reduce in one pass; argmax/argmin over several axes
 * report the flat index over those axes (reduction.rs:186-223). Integer
 * inputs narrower than 64 bits must be widened to int64 by the caller (as
 * musapy's cast_array does); MPB_R_ARGMAX_REC / _ARGMIN_REC write a 16-byte
 * {value bits, index} record per output for cross-shard combining. */
int mpb_reduce(int op, int ndim, const int64_t* shape, const int64_t* strides, const void* a, int in_dtype,
               uint64_t axes_mask, void* out, int out_dtype, int compute_dtype, int nan_first_rule, void* scratch,
               size_t scratch_bytes, mpb_stream_t stream);

/* Same as mpb_reduce but with no scratch argument: the scratch comes from an
 * array built into the library (256 KiB per GPU, held from the library's
 * load on that GPU until the process exits). No counterpart in musapy. It
 * exists for callers that cannot allocate device memory: an application that
 * embeds this library and owns the whole device budget through its own pool,
 * or a latency-critical loop in which cudaMalloc / cudaFree must not run
 * because they can synchronise the device. It allocates nothing. No request
 * is refused for its size: the reduction splits across CTAs only as far as
 * its partials fit in the 256 KiB (a reduction with more than 16384 outputs
 * runs unsplit, which needs no scratch). Where that limit changes the split,
 * float sums and means may differ from mpb_reduce's in the last bits;
 * otherwise both run the same plan and agree bit for bit. All calls on a GPU
 * share the array and it keeps the last call's contents (nothing in it needs
 * to start at zero), so calls that can overlap on the GPU race: order them on
 * one stream or with events. The first call on each device looks up the
 * array's device address with that device current; make that first call
 * before any stream capture begins (later uncaptured calls look it up again,
 * so a device reset is picked up). */
int mpb_reduce_noalloc(int op, int ndim, const int64_t* shape, const int64_t* strides, const void* a, int in_dtype,
                       uint64_t axes_mask, void* out, int out_dtype, int compute_dtype, int nan_first_rule,
                       mpb_stream_t stream);

/* ------------------------------------------------------------------ cumsum */

/* Device scratch (bytes) mpb_cumsum needs; 0 when none. */
size_t mpb_cumsum_scratch_bytes(int ndim, const int64_t* shape, const int64_t* strides, const void* a, int in_dtype,
                                int axis, void* out, int out_dtype);

/* Inclusive prefix sum along `axis`; out_dtype is the compute dtype (f32,
 * f64, or i64 for integer inputs). Replaces musapy_cumsum_{i64,f32,f64}_v3
 * (kernels.rs:185-187) without its 256^3 length limit. The scratch is
 * cleared by the call itself. */
int mpb_cumsum(int ndim, const int64_t* shape, const int64_t* strides, const void* a, int in_dtype, int axis,
               void* out, int out_dtype, void* scratch, size_t scratch_bytes, mpb_stream_t stream);

/* Synchronises `stream` and reads the status word a look-back cumsum left in
 * its scratch: MPB_OK, or MPB_ERR_TIMEOUT when a bounded wait gave up. */
int mpb_cumsum_status(const void* scratch, mpb_stream_t stream);

/* ---------------------------------------------------------------- creation */

/* Fills `out` (n contiguous elements of `dtype`) with start + i*step, each
 * value evaluated in f64 (multiply, then add, each rounded) and converted once
 * with Rust `as` semantics, as the CPU path of ms.arange does
 * (creation.rs:469-501 and :324-348). Replaces musapy_arange_{f32,f64,i64,i32}
 * (kernels.rs, init.mu:86-97), which compute in the element type; every dtype
 * is accepted. The caller derives n from start/stop/step (arange_len,
 * creation.rs:624-633). */
int mpb_arange(void* out, int dtype, int64_t n, double start, double step, mpb_stream_t stream);

/* n evenly spaced values from start to stop inclusive: step = (stop - start) /
 * (n - 1) in f64, element i = start + i*step as in mpb_arange; n == 1 gives
 * start (creation.rs:508-521 and :350-377). Replaces musapy_linspace_{f32,f64}
 * (init.mu:102-115). */
int mpb_linspace(void* out, int dtype, int64_t n, double start, double stop, mpb_stream_t stream);

/* rows x cols matrix (C-contiguous) of zeros with ones where col - row == k
 * (creation.rs:457-461, init.mu:47-56). Replaces musapy_eye_{f32,f64,i64,i32}
 * (init.mu:121-134); every dtype is accepted. */
int mpb_eye(void* out, int dtype, int64_t rows, int64_t cols, int64_t k, mpb_stream_t stream);

/* --------------------------------------------------- host <-> device copies */

/* Copies `bytes` from pageable (or any) host memory to device memory `dst`
 * on `stream`, through a ring of pinned staging slots with the host-side
 * copies spread over a few threads and overlapped with the DMA of the
 * previous chunk; a page-locked source (cudaHostAlloc / cudaHostRegister) is
 * moved by one DMA with no staging. Returns once the host source has been read completely (it
 * may be reused at once); the device copy completes in stream order. Replaces
 * the list-based host transfer of ms.array (rust/musapy-python/src/ops.rs:
 * 354-625) and the plain musaMemcpy behind it (musa_ffi.rs). The device is the
 * current CUDA device. */
int mpb_copy_h2d(void* dst, const void* src, size_t bytes, mpb_stream_t stream);

/* Copies `bytes` of device memory `src` to host memory `dst` after the work
 * already queued on `stream`, and returns when `dst` holds the data. Same
 * staging ring as mpb_copy_h2d, the DMA of chunk k+4 overlapping the host
 * copy of chunk k; a page-locked destination gets one DMA, no staging. Replaces Array.tolist's transfer (array.rs:451-488). */
int mpb_copy_d2h(void* dst, const void* src, size_t bytes, mpb_stream_t stream);

/* ---------------------------------------------------- axis-0 sharding (new) */

/* Device combine of per-rank argmax/argmin records (MPB_R_ARG*_REC output,
 * all-gathered in rank order) into one global flat index; rank_offsets[r] is
 * the flat index of rank r's first element. No counterpart in musapy, which
 * has no multi-GPU path. */
int mpb_shard_arg_combine(const int64_t* records, int nranks, const int64_t* rank_offsets, int is_max, int is_int,
                          int64_t* out_index, double* out_value, mpb_stream_t stream);

/* Writes sum and mean (true global count) of an all-reduced f64 total in the
 * array dtype (MPB_F32 or MPB_F64). No counterpart in musapy. */
int mpb_shard_sum_finalize(const double* total, double count, int out_dtype, void* sum_out, void* mean_out,
                           mpb_stream_t stream);

/* ------------------------------------------- peer record exchange (new) */

/* Record exchange over NVLink peer memory between the ranks of one node, the
 * last step of a sharded full reduction. No counterpart in musapy, which has
 * no multi-GPU path. Each rank allocates one exchange buffer
 * (mpb_peer_alloc: cudaMalloc of mpb_peer_buffer_bytes() bytes, zeroed, plus
 * its CUDA IPC handle of mpb_peer_handle_bytes() bytes), the handles are
 * exchanged out of band, and each rank opens the others (mpb_peer_open). */
size_t mpb_peer_buffer_bytes(void);
size_t mpb_peer_handle_bytes(void);
int mpb_peer_alloc(void** buf, void* ipc_handle);
int mpb_peer_open(const void* ipc_handle, void** peer_buf);
int mpb_peer_close(void* peer_buf);
int mpb_peer_free(void* buf);

/* Exchange number `seq` (1, 2, ... the same sequence on every rank): stores
 * this rank's `rec_bytes` (8, 16, 24 or 32) record into every rank's buffer
 * (peers[r] is rank r's buffer as mapped here, peers[rank] the local one),
 * then waits until all `world` records of this exchange have arrived and
 * writes them to `out` in rank order (world x rec_bytes, 8-byte aligned).
 * Records travel as flag-in-line words (each 8-byte half of a 16-byte
 * store is {4 data bytes, 32-bit seq}), so no fence or flag store is
 * needed. Waits are bounded (~2 s): on expiry *status (device int) becomes
 * MPB_ERR_TIMEOUT and the kernel returns without writing `out`. At most 16
 * ranks. */
int mpb_peer_allgather(const void* rec, int rec_bytes, void* const* peers, int rank, int world, uint64_t seq,
                       void* out, int* status, mpb_stream_t stream);

/* The exchange of mpb_peer_allgather fused with the finish of a sharded
 * sum: `partial` is this rank's f64 partial sum; the `world` partials are
 * summed in rank order (the same value on every rank) and the sum and mean
 * (over `count` elements) written in MPB_F32 or MPB_F64. One kernel. No
 * counterpart in musapy. */
int mpb_peer_sum_finalize(const double* partial, void* const* peers, int rank, int world, uint64_t seq, double count,
                          int out_dtype, void* sum_out, void* mean_out, int* status, mpb_stream_t stream);

/* The exchange fused with the finish of a sharded argmax / argmin: `record`
 * is this rank's {value bits, local index} (MPB_R_ARG*_REC output); the
 * records are combined in rank order as mpb_shard_arg_combine does
 * (rank_offsets[r] = flat index of rank r's first element). One kernel. No
 * counterpart in musapy. */
int mpb_peer_arg_combine(const int64_t* record, void* const* peers, int rank, int world, uint64_t seq,
                         const int64_t* rank_offsets, int is_max, int is_int, int64_t* out_index, double* out_value,
                         int* status, mpb_stream_t stream);

/* The two fused exchanges above with all `world` ranks played on ONE GPU:
 * one cooperative launch of `world` blocks (every block resident at once),
 * block r acting as rank r with exchange buffer bufs[r] (zeroed
 * mpb_peer_buffer_bytes() buffers on this GPU), record partials[r] /
 * records[2r..2r+1] and results sum_out[r], mean_out[r] (f32 or f64 per
 * out_dtype) / out_index[r], out_value[r]. The kernels, wire format, waits
 * and combine are those of the per-rank calls; only the launch differs.
 * For checking the multi-rank exchange and combine where fewer GPUs than
 * ranks exist (ranks that wait on one another must never be separate
 * launches on one GPU). No counterpart in musapy. */
int mpb_peer_sum_finalize_emulated(const double* partials, void* const* bufs, int world, uint64_t seq, double count,
                                   int out_dtype, void* sum_out, void* mean_out, int* status, mpb_stream_t stream);
int mpb_peer_arg_combine_emulated(const int64_t* records, void* const* bufs, int world, uint64_t seq,
                                  const int64_t* rank_offsets, int is_max, int is_int, int64_t* out_index,
                                  double* out_value, int* status, mpb_stream_t stream);

/* Sum of `world` f64 partials (stride_bytes apart) in rank order, then sum
 * and mean (over `count` elements) in MPB_F32 or MPB_F64. No counterpart in
 * musapy. */
int mpb_shard_sum_parts_finalize(const double* parts, int stride_bytes, int world, double count, int out_dtype,
                                 void* sum_out, void* mean_out, mpb_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* MUSAPY_B200_H */
