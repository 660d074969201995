"""Host logic of the axis-0 sharded path on CPU: row partitioning, and the
cross-rank combine of (value, index) records and f64 partial sums, run as two
gloo ranks and checked against the oracle on the whole array."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_shard_rows_partition():
    from musapy_b200.shard import shard_rows

    for n in (1, 7, 8, 65536, 65537):
        for w in (1, 2, 3, 4, 8):
            spans = [shard_rows(n, w, r) for r in range(w)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1


def _local_record(x: np.ndarray, is_max: bool, nan_rule: bool):
    """What a rank's device reduction writes: best (value, local index) over
    non-NaN values with first occurrence, or (NaN, 0) when the rule applies
    and element 0 is NaN; index INT64_MAX when nothing qualifies."""
    flat = x.reshape(-1)
    if nan_rule and flat.size and np.isnan(flat[0]):
        return np.array([np.array([np.nan]).view(np.int64)[0], 0], np.int64)
    ok = ~np.isnan(flat)
    if not ok.any():
        return np.array([0, np.iinfo(np.int64).max], np.int64)
    vals = np.where(ok, flat, -np.inf if is_max else np.inf)
    i = int(np.argmax(vals) if is_max else np.argmin(vals))
    return np.array([np.array([float(flat[i])]).view(np.int64)[0], i], np.int64)


def _worker(rank, world, port, x, results):
    import torch
    import torch.distributed as dist

    from musapy_b200.shard import combine_records_host, shard_rows

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    r0, r1 = shard_rows(x.shape[0], world, rank)
    local = x[r0:r1]
    # sum: f64 partial, one all_reduce
    part = torch.tensor([float(local.astype(np.float64).sum())], dtype=torch.float64)
    dist.all_reduce(part)
    # argmax / argmin: one all_gather of 16-byte records
    out = {}
    for is_max in (True, False):
        rec = torch.from_numpy(_local_record(local, is_max, r0 == 0))
        allr = [torch.zeros(2, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(allr, rec)
        starts = [shard_rows(x.shape[0], world, r)[0] * x.shape[1] for r in range(world)]
        out[is_max] = combine_records_host(torch.stack(allr).numpy(), starts, is_max, False)
    results[rank] = (float(part[0]), out[True], out[False])
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("case", ["random", "ties_across_ranks", "nan_first", "nan_elsewhere"])
def test_two_rank_combine_matches_oracle(oracle, case):
    rng = np.random.default_rng(5)
    x = rng.random((9, 16), dtype=np.float32) * 2 - 1
    if case == "ties_across_ranks":
        x[2, 3] = x[7, 1] = 5.0
        x[1, 0] = x[8, 15] = -5.0
    if case == "nan_first":
        x[0, 0] = np.nan
    if case == "nan_elsewhere":
        x[6, 0] = np.nan  # first element of rank 1's shard
        x[3, 3] = np.nan
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, x, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    for r in range(2):
        total, amax, amin = results[r]
        np.testing.assert_allclose(total, x.astype(np.float64).sum(), rtol=1e-12)
        assert amax == int(oracle.reduce("argmax", x, None)), (case, amax)
        assert amin == int(oracle.reduce("argmin", x, None)), (case, amin)
