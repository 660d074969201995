"""Axis-0 sharding across the GPUs of one node (one process per GPU).

musapy is single-device (docs/adr/ADR.md:896-906); this module is the new
multi-GPU path. A ``ShardedArray`` holds this rank's contiguous block of rows
of a global array; broadcast operands (a row vector) are replicated.

* elementwise ops run on each shard independently (no communication);
* reductions over non-leading axes stay local;
* full reductions reduce the local shard on the GPU and move one 8- or
  16-byte record per rank over NVLink with ONE exchange - by default a
  peer-memory kernel (PeerExchange: P2P stores of flag-in-line words into
  every rank's IPC-shared buffer, bounded waits) that also finishes the
  reduction in rank order, or NCCL (all_reduce for sum/mean, all_gather for
  argmax/argmin, then a one-thread device combine) with
  MUSAPY_B200_SHARD_COLLECTIVE=nccl - so no host round trip is needed.

The process group is torch.distributed's (backend "nccl" on GPUs, "gloo" in
the CPU tests of the combine logic).
"""
from __future__ import annotations

import numpy as np
import torch
import torch.distributed as dist

from . import dtypes as _dt
from . import errors, ops
from . import streams as _streams
from ._lib import LIB, NATIVE, RED_OPS, check, i64arr
from .array import Array, empty


def shard_rows(n_rows: int, world: int, rank: int) -> tuple[int, int]:
    """[start, stop) rows of `rank`: contiguous blocks, the first n % world
    ranks one row larger."""
    base, extra = divmod(n_rows, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


class ShardedArray:
    """This rank's rows [row0, row0 + local.shape[0]) of a global array."""

    def __init__(self, local: Array, global_shape: tuple, row0: int, group=None) -> None:
        self.local = local
        self.global_shape = tuple(global_shape)
        self.row0 = int(row0)
        self.group = group

    @property
    def dtype(self) -> _dt.Dtype:
        return self.local.dtype

    @property
    def global_size(self) -> int:
        n = 1
        for s in self.global_shape:
            n *= s
        return n


class PeerExchange:
    """Small-record exchange over NVLink peer memory (mpb_peer_allgather and
    the fused mpb_peer_sum_finalize / mpb_peer_arg_combine):
    one exchange buffer per rank shared by CUDA IPC, one kernel per exchange,
    sequence numbers kept identical on all ranks by calling exchanges in the
    same order everywhere (as collectives already must be)."""

    def __init__(self, dev: int, group=None) -> None:
        """Collective: every rank of `group` constructs it together. Raises
        InteropError on every rank when any rank cannot share or map the
        buffers (the ranks agree before and after mapping)."""
        import ctypes

        self.dev, self.group = dev, group
        self.world, self.rank = _world(group)
        self.seq = 0
        self._buf = ctypes.c_void_p()
        self._opened = []
        handle = ctypes.create_string_buffer(int(LIB.mpb_peer_handle_bytes()))
        with torch.cuda.device(dev):
            ok = LIB.mpb_peer_alloc(ctypes.byref(self._buf), handle) == 0
        gathered = [None] * self.world
        dist.all_gather_object(gathered, (ok, handle.raw if ok else b""), group=group)
        if not all(g[0] for g in gathered):
            self._release()
            raise errors.InteropError("peer exchange: a rank could not allocate or share its buffer")
        ptrs = []
        with torch.cuda.device(dev):
            for r, (_, h) in enumerate(gathered):
                if r == self.rank:
                    ptrs.append(self._buf.value)
                    continue
                p = ctypes.c_void_p()
                hb = ctypes.create_string_buffer(h, len(h))
                if LIB.mpb_peer_open(hb, ctypes.byref(p)) != 0:
                    ok = False
                    break
                self._opened.append(p.value)
                ptrs.append(p.value)
        oks = [None] * self.world
        dist.all_gather_object(oks, ok, group=group)
        if not all(oks):
            self._release()
            raise errors.InteropError("peer exchange: a rank could not map the other ranks' buffers")
        self._ptrs = (ctypes.c_void_p * self.world)(*ptrs)
        self.status = torch.zeros(1, dtype=torch.int32, device=f"cuda:{dev}")
        self._status_ptr = self.status.data_ptr()
        # The fused exchanges run here, ordered after the local reduction by
        # an event: the rank's next pass starts while its exchange waits for
        # the other ranks (their records arrive over NVLink meanwhile).
        self.side = torch.cuda.Stream(device=dev)
        self.side_handle = self.side.cuda_stream
        self.side_ms = _streams._wrap(dev, self.side)
        self.ready = torch.cuda.Event()  # recorded on the main stream behind each local reduction

    def _release(self) -> None:
        with torch.cuda.device(self.dev):
            for p in self._opened:
                LIB.mpb_peer_close(p)
            self._opened = []

    def allgather(self, rec: torch.Tensor, out: torch.Tensor, stream: int) -> None:
        """rec: 16 or 32 bytes on this rank's device; out: world x that, in rank order."""
        self.seq += 1
        check(LIB.mpb_peer_allgather(rec.data_ptr(), rec.nbytes, self._ptrs, self.rank, self.world, self.seq,
                                     out.data_ptr(), self.status.data_ptr(), stream), "peer exchange")

    def sum_finalize(self, partial_ptr: int, count: float, out_dtype: int, sum_ptr: int, mean_ptr: int,
                     stream: int) -> None:
        """Exchange the f64 partials (`partial_ptr`: this rank's, on the device)
        and write the global sum and mean (one kernel)."""
        self.seq += 1
        check(LIB.mpb_peer_sum_finalize(partial_ptr, self._ptrs, self.rank, self.world, self.seq, count,
                                        out_dtype, sum_ptr, mean_ptr, self._status_ptr, stream),
              "peer exchange")

    def arg_combine(self, rec_ptr: int, starts, is_max: bool, is_int: bool, index_ptr: int, value_ptr: int,
                    stream: int) -> None:
        """Exchange the (value, index) records and write the global index (one
        kernel); `starts`: the ranks' first flat indices (a list or an int64
        ctypes array)."""
        self.seq += 1
        if isinstance(starts, (list, tuple)):
            starts = i64arr(starts)
        check(LIB.mpb_peer_arg_combine(rec_ptr, self._ptrs, self.rank, self.world, self.seq, starts,
                                       1 if is_max else 0, 1 if is_int else 0, index_ptr, value_ptr,
                                       self._status_ptr, stream), "peer exchange")

    def check(self) -> None:
        """Raise if any exchange gave up waiting for a rank (synchronises the
        device, side stream included)."""
        torch.cuda.synchronize(self.dev)
        if int(self.status.item()) != 0:
            raise errors.StreamError(f"peer exchange on cuda:{self.dev}: a rank did not arrive within the wait limit")

    def close(self) -> None:
        """Collective: every rank synchronises, meets at a barrier (so no
        exchange kernel is still writing into anyone's buffer), then unmaps."""
        torch.cuda.synchronize(self.dev)
        dist.barrier(group=self.group)
        self._release()
        dist.barrier(group=self.group)
        if self._buf.value:  # nobody maps it any more
            with torch.cuda.device(self.dev):
                LIB.mpb_peer_free(self._buf)
            self._buf.value = None


def _on_side(ex: PeerExchange, dev: int, outs, launch) -> None:
    """Run `launch(stream_handle)` on the exchange's side stream after the
    work queued so far on the current stream (the local reduction that wrote
    the record), with the ms stream bookkeeping of the outputs `outs`: the
    side stream waits for their users on other streams and becomes their last
    user (in the steady state the side stream already is, and nothing but the
    event is needed)."""
    main = torch.cuda.current_stream(dev)
    ex.ready.record(main)
    ex.side.wait_event(ex.ready)
    side = ex.side_ms
    for o in outs:
        buf = o._buf
        last = getattr(buf, "_mpb_stream", None)
        if last is side:
            continue
        if last is not None and last._handle != side._handle:
            ex.side.wait_stream(last._torch)
        buf.record_stream(ex.side)
        buf._mpb_stream = side
    launch(ex.side_handle)


def join_exchanges(dev: int) -> None:
    """Make the current stream of `dev` wait for every record exchange queued
    so far (e.g. before timing ends or before reading results with torch)."""
    main = torch.cuda.current_stream(dev)
    for (d, _), ex in _EXCHANGES.items():
        if d == dev and ex is not None:
            main.wait_stream(ex.side)


_EXCHANGES: dict = {}
_MISSING = object()


def peer_exchange(dev: int, group=None) -> PeerExchange | None:
    """The node's peer exchange for (dev, group), created on first use by all
    ranks together; None when there is a single rank or when the transport is
    NCCL (MUSAPY_B200_SHARD_COLLECTIVE=nccl)."""
    import os

    key = (dev, id(group))
    ex = _EXCHANGES.get(key, _MISSING)
    if ex is not _MISSING:
        return ex
    world, _ = _world(group)
    if world <= 1 or os.environ.get("MUSAPY_B200_SHARD_COLLECTIVE", "peer") == "nccl":
        return None
    if dist.get_backend(group) != "nccl":  # CPU process groups (gloo) have no device buffers
        _EXCHANGES[key] = None
        return None
    try:
        ex = PeerExchange(dev, group)
    except errors.InteropError as e:  # every rank takes this branch together
        import warnings

        warnings.warn(f"{e}; full reductions use NCCL collectives", RuntimeWarning)
        ex = None
    _EXCHANGES[key] = ex
    return ex


def close_exchanges() -> None:
    """Collective teardown of every peer exchange (call on all ranks before
    destroy_process_group)."""
    for key in list(_EXCHANGES):
        ex = _EXCHANGES.pop(key)
        if ex is not None:
            ex.close()


def _world(group) -> tuple[int, int]:
    if dist.is_available() and dist.is_initialized():
        return dist.get_world_size(group), dist.get_rank(group)
    return 1, 0


def add(x: ShardedArray, row: Array, out: Array | None = None) -> ShardedArray:
    """Broadcast add of a replicated operand; local, no communication."""
    return ShardedArray(ops.add(x.local, row, out=out), x.global_shape, x.row0, x.group)


def sum_axis(x: ShardedArray, axis: int, out: Array | None = None) -> ShardedArray:
    """Reduction over a non-leading axis: local per shard."""
    if axis % len(x.global_shape) == 0:
        raise errors.ShapeError("sum over the sharded axis needs a collective: use sum_all")
    return ShardedArray(ops.sum(x.local, axis=axis, out=out), x.global_shape[:axis] + x.global_shape[axis + 1:],
                        x.row0, x.group)


class _Slots:
    """Two alternating record slots: a slot is written by the local reduction
    on the current stream only after the exchange that last read it (on the
    side stream) is done."""

    def __init__(self, dev: int, n: int, dtype) -> None:
        self.buf = torch.zeros((2, n), dtype=dtype, device=f"cuda:{dev}")
        self.views = [self.buf[0], self.buf[1]]
        self.ptrs = [v.data_ptr() for v in self.views]
        self.read_done = [torch.cuda.Event(), torch.cuda.Event()]
        self.used = [False, False]
        self.side_recorded = False
        self.k = 0

    def next(self, dev: int) -> int:
        """Index of the slot to write next (the current stream waits for the
        exchange that read it last)."""
        self.k ^= 1
        if self.used[self.k]:
            torch.cuda.current_stream(dev).wait_event(self.read_done[self.k])
        return self.k

    def read_by(self, ex: PeerExchange) -> None:
        self.read_done[self.k].record(ex.side)
        self.used[self.k] = True
        if not self.side_recorded:
            # a combine object made for one call alone is freed on return:
            # its slots must outlive the side stream's use of them
            self.buf.record_stream(ex.side)
            self.side_recorded = True


class _Local:
    """A local full reduction's plan and scratch, cached per layout (the
    reduction runs on the current stream, so one scratch serves every call)."""

    def __init__(self) -> None:
        self.key = None
        self.nbytes = 0
        self.scratch = None
        self.scratch_ptr = None

    def prepare(self, dev: int, op: int, a: Array, in_code: int, mask: int, cd_code: int) -> None:
        key = (op, a._shape, a._strides, in_code, mask, cd_code, a.data_ptr & 15)
        if key == self.key:
            return
        n = NATIVE.reduce_scratch_bytes(op, a._shape, a._strides, a.data_ptr, in_code, mask, cd_code)
        if n and (self.scratch is None or self.scratch.numel() < n):
            self.scratch = torch.empty(n, dtype=torch.uint8, device=f"cuda:{dev}")
            self.scratch_ptr = self.scratch.data_ptr()
        self.nbytes = n
        self.key = key


class _SumCombine:
    """Scratch of a full sum/mean: the local f64 partial (first of two
    doubles: the NCCL route all-reduces it in place; the peer route
    alternates between two slots) and the results."""

    def __init__(self, dev: int, out_dt: _dt.Dtype, world: int = 1) -> None:
        self.partial = torch.zeros(2, dtype=torch.float64, device=f"cuda:{dev}")
        self.slots = _Slots(dev, 2, torch.float64)
        self.local = _Local()
        self.sum_out = empty((), out_dt, dev)
        self.mean_out = empty((), out_dt, dev)


def sum_all(x: ShardedArray, combine: _SumCombine | None = None) -> tuple[Array, Array]:
    """Global sum and mean of a float array: local f32/f64 sum written as f64,
    one exchange of 8 bytes per rank (peer kernel with the finish fused, or
    an NCCL all_reduce), mean over the true global element count. Pass the
    same `combine` on every call of a loop: its plan, scratch and records are
    reused (this call's host cost is part of every sharded step)."""
    a = x.local
    if a.dtype.code not in (_dt.F32, _dt.F64):
        raise errors.DtypeError("sum_all: float32/float64 shards only")
    dev = a._dev
    c = combine or _SumCombine(dev, a.dtype)
    cd = a.dtype
    mask = (1 << a.ndim) - 1
    op = RED_OPS["sum"]
    stream = _streams.current_stream(dev).cuda_stream
    ex = peer_exchange(dev, x.group)
    if ex is not None:
        k = c.slots.next(dev)
        partial, partial_ptr = c.slots.views[k], c.slots.ptrs[k]
    else:
        partial, partial_ptr = c.partial, c.partial.data_ptr()
    if a.size == 0:  # a rank without rows (more ranks than rows) contributes 0
        with torch.cuda.stream(_streams.current_stream(dev).torch_stream):
            partial.zero_()
    else:
        c.local.prepare(dev, op, a, a.dtype.code, mask, cd.code)
        check(NATIVE.reduce(op, a._shape, a._strides, a.data_ptr, a.dtype.code, mask, partial_ptr, _dt.F64, cd.code,
                            1, c.local.scratch_ptr if c.local.nbytes else None, c.local.nbytes, stream), "sum_all")
    if ex is not None:
        # partials of all ranks over NVLink, summed in rank order on every
        # rank, on the exchange's side stream
        _on_side(ex, dev, (c.sum_out, c.mean_out),
                 lambda h: ex.sum_finalize(partial_ptr, float(x.global_size), a.dtype.code, c.sum_out.data_ptr,
                                           c.mean_out.data_ptr, h))
        c.slots.read_by(ex)
        return c.sum_out, c.mean_out
    world, _ = _world(x.group)
    if world > 1:
        dist.all_reduce(c.partial, op=dist.ReduceOp.SUM, group=x.group)
    check(LIB.mpb_shard_sum_finalize(c.partial.data_ptr(), float(x.global_size), a.dtype.code,
                                     c.sum_out.data_ptr, c.mean_out.data_ptr, stream), "sum_all")
    return c.sum_out, c.mean_out


class _ArgCombine:
    def __init__(self, dev: int, world: int) -> None:
        self.rec = torch.empty(2, dtype=torch.int64, device=f"cuda:{dev}")
        self.slots = _Slots(dev, 2, torch.int64)
        self.local = _Local()
        self.all = torch.empty(2 * world, dtype=torch.int64, device=f"cuda:{dev}")
        self.index = empty((), _dt.int64, dev)
        self.value = torch.empty(1, dtype=torch.float64, device=f"cuda:{dev}")
        self.value_ptr = self.value.data_ptr()
        self.starts_key = None
        self.starts = None
        self.value_recorded = False

    def rank_starts(self, x: ShardedArray, world: int):
        """The ranks' first flat indices as an int64 ctypes array (cached)."""
        a = x.local
        row_elems = a.size // max(1, a.shape[0]) if a.ndim else 1
        key = (x.global_shape, world, row_elems)
        if key != self.starts_key:
            self.starts = i64arr([shard_rows(x.global_shape[0], world, r)[0] * row_elems for r in range(world)])
            self.starts_key = key
        return self.starts


def argreduce_all(x: ShardedArray, is_max: bool = True, combine: _ArgCombine | None = None) -> Array:
    """Global argmax/argmin (flat index, first occurrence, musapy's NaN rule):
    local (value, index) record, one exchange of 16 bytes per rank (peer
    kernel with the combine fused, or an NCCL all_gather and a device
    combine), in rank order. Pass the same `combine` on every call of a loop
    (plan, scratch, records and rank offsets are reused)."""
    a = x.local
    dev = a._dev
    world, rank = _world(x.group)
    c = combine or _ArgCombine(dev, world)
    src = a if a.dtype.code in (_dt.F32, _dt.F64, _dt.F16, _dt.BF16, _dt.I64, _dt.U64) else ops.astype(a, _dt.int64)
    mask = (1 << src.ndim) - 1
    stream = _streams.current_stream(dev).cuda_stream
    op = RED_OPS["argmax_rec" if is_max else "argmin_rec"]
    ex = peer_exchange(dev, x.group)
    if ex is not None:
        k = c.slots.next(dev)
        rec, rec_ptr = c.slots.views[k], c.slots.ptrs[k]
    else:
        rec, rec_ptr = c.rec, c.rec.data_ptr()
    if src.size == 0:  # a rank without rows sends the empty record {0, INT64_MAX}
        with torch.cuda.stream(_streams.current_stream(dev).torch_stream):
            rec[0] = 0
            rec[1] = np.iinfo(np.int64).max
    else:
        # only the shard holding global element 0 applies the first-element NaN rule
        c.local.prepare(dev, op, src, src.dtype.code, mask, src.dtype.code)
        check(NATIVE.reduce(op, src._shape, src._strides, src.data_ptr, src.dtype.code, mask, rec_ptr, _dt.I64,
                            src.dtype.code, 1 if x.row0 == 0 else 0,
                            c.local.scratch_ptr if c.local.nbytes else None, c.local.nbytes, stream), "argreduce_all")
    is_int = src.dtype.code in (_dt.I64, _dt.U64)
    if ex is not None:
        starts = c.rank_starts(x, world)
        # c.value is a torch tensor outside the ms bookkeeping: torch users of
        # it call join_exchanges first
        _on_side(ex, dev, (c.index,),
                 lambda h: ex.arg_combine(rec_ptr, starts, is_max, is_int, c.index.data_ptr, c.value_ptr, h))
        c.slots.read_by(ex)
        if not c.value_recorded:
            c.value.record_stream(ex.side)
            c.value_recorded = True
        return c.index
    if world > 1:
        dist.all_gather_into_tensor(c.all, c.rec, group=x.group)
        recs = c.all
        starts = c.rank_starts(x, world)
    else:
        recs = c.rec
        starts = i64arr([0])
    check(LIB.mpb_shard_arg_combine(recs.data_ptr(), world, starts, 1 if is_max else 0, 1 if is_int else 0,
                                    c.index.data_ptr, c.value_ptr, stream), "argreduce_all")
    return c.index


def combine_records_host(recs: np.ndarray, starts, is_max: bool, is_int: bool) -> int:
    """Host restatement of the device combine (k_arg_combine), used by the
    CPU tests of the sharded logic: recs is int64 [world, 2]."""
    best_i, best_v, have = 0, None, False
    for r, (vb, li) in enumerate(recs.tolist()):
        if li == np.iinfo(np.int64).max:
            continue
        v = vb if is_int else float(np.array([vb], np.int64).view(np.float64)[0])
        if not is_int and r == 0 and li == 0 and v != v:
            return 0
        if not have or (v > best_v if is_max else v < best_v):
            best_v, best_i, have = v, li + starts[r], True
    return best_i if have else 0
