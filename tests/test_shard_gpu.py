"""Sharded path on 2 GPUs (one process per GPU, NCCL): broadcast add and
axis-1 sums stay local, full sum/mean and argmax/argmin combine across ranks;
results checked on rank 0 against the oracle on the whole array. Skipped with
fewer than 2 GPUs."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from tests.helpers import assert_bits_equal

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, x, row, out_q, transport="peer"):
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["MUSAPY_B200_SHARD_COLLECTIVE"] = transport
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device(f"cuda:{rank}"))
    import musapy_b200 as ms
    from musapy_b200 import shard as sh

    ms.set_default_device(f"cuda:{rank}")

    r0, r1 = sh.shard_rows(x.shape[0], world, rank)
    xs = sh.ShardedArray(ms.from_numpy(x[r0:r1], device=rank), x.shape, r0)
    rd = ms.from_numpy(row, device=rank)
    y = sh.add(xs, rd)
    rs = sh.sum_axis(y, 1)
    s, m = sh.sum_all(xs)
    amax = sh.argreduce_all(xs, True)
    amin = sh.argreduce_all(xs, False)
    res = (y.local.numpy(), rs.local.numpy(), float(s.item()), float(m.item()), int(amax.item()), int(amin.item()))
    # many exchanges in a row (sequence numbers, both buffer parities)
    seq = []
    for _ in range(25):
        s2, _m2 = sh.sum_all(xs)
        seq.append((float(s2.item()), int(sh.argreduce_all(xs, True).item())))
    # exchanges queued back to back with no host wait in between: x and -x
    # alternate, each result copied on the current stream (ordered after the
    # exchange by the stream bookkeeping) and read at the end
    xn = sh.ShardedArray(ms.neg(xs.local), x.shape, r0)
    queued = []
    for i in range(30):
        src = xs if i % 2 == 0 else xn
        s3, _m3 = sh.sum_all(src)
        a3 = sh.argreduce_all(src, True)
        queued.append((ms.astype(s3, "f64"), ms.astype(a3, "i64")))
    queued = [(float(v.item()), int(w.item())) for v, w in queued]
    for ex in sh._EXCHANGES.values():
        if ex is not None:
            ex.check()
    out_q.put((rank, r0, r1, res, seq, queued))
    sh.close_exchanges()
    dist.barrier(device_ids=[rank])
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("transport", ["peer", "nccl"])
@pytest.mark.parametrize("case", ["random", "nan_first", "nan_in_rank1", "ties"])
def test_sharded_ops_two_gpus(oracle, case, transport):
    rng = np.random.default_rng(5)
    x = rng.random((1024, 4096), dtype=np.float32) * 2 - 1
    row = rng.random(4096, dtype=np.float32) * 2 - 1
    if case == "nan_first":
        x[0, 0] = np.nan
    if case == "nan_in_rank1":
        x[512, 0] = np.nan
        x[700, 5] = np.nan
    if case == "ties":
        x[3, 3] = x[900, 1] = 9.0
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, x, row, q, transport)) for r in range(2)]
    for p in procs:
        p.start()
    got = [q.get(timeout=180) for _ in range(2)]
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    want_y = oracle.binary("add", x, row)
    seqs = [[repr(t) for t in g[4]] for g in got]  # repr: NaN-safe comparison
    assert seqs[0] == seqs[1], "ranks disagree on repeated exchanges"
    assert len(set(seqs[0])) == 1, "repeated full reductions differ"
    amax_neg = int(oracle.reduce("argmax", -x, None))
    for rank, r0, r1, (y, rs, s, m, amax, amin), _, queued in got:
        for i, (qs, qa) in enumerate(queued):
            ws, wa = (s, amax) if i % 2 == 0 else (-s, amax_neg)
            assert repr(qs) == repr(ws) and qa == wa, (case, transport, rank, i, qs, ws, qa, wa)
    for rank, r0, r1, (y, rs, s, m, amax, amin), _, _q in got:
        assert_bits_equal(y, want_y[r0:r1], f"sharded add rank {rank}")
        want_rs = oracle.reduce("sum", want_y[r0:r1], axis=1)
        ok = np.abs(rs.astype(np.float64) - want_rs) <= 1e-5 * np.abs(want_y[r0:r1]).astype(np.float64).sum(1)
        assert (ok | (np.isnan(rs) & np.isnan(want_rs))).all()
        truth = np.sum(x.astype(np.float64))
        if case.startswith("nan"):
            assert np.isnan(s) and np.isnan(m)
        else:
            assert abs(s - truth) <= 1e-5 * np.abs(x).astype(np.float64).sum()
            assert abs(m - truth / x.size) <= 1e-5 * np.abs(x).astype(np.float64).mean()
        assert amax == int(oracle.reduce("argmax", x, None)), (case, rank)
        assert amin == int(oracle.reduce("argmin", x, None)), (case, rank)
