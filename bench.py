"""Benchmark: HBM GB/s of musapy's broadcast add and axis sums on B200.

Workload: a float32 (65536, 32768) array, uniform[-1, 1) from numpy PCG64
seed 5, sharded on axis 0 across the GPUs of one node (one process per GPU),
and a replicated (32768,) row vector drawn after it. One step is the hot
path over the whole array:

    y   = x + row                 broadcast add           (local)
    r   = sum(y, axis=1)          axis sum                (local)
    s,m = sum(x), mean(x)         full reduction          (8-byte record per rank)
    i   = argmax(x)               full arg reduction      (16-byte record per rank)

With several ranks each full reduction ends with one record exchange over
NVLink: the peer-memory exchange kernel (csrc/peer.cu) stores the rank's
record into every peer's buffer and finishes the reduction in the same
kernel (NCCL collectives with MUSAPY_B200_SHARD_COLLECTIVE=nccl).

`value` = algorithmic bytes of all ranks / step time (each input read once,
each output written once), max over ranks; `e2e` is the same metric with the
step's input copied from pinned host memory through the library's transfer
entry points (mpb_copy_h2d / mpb_copy_d2h) and its results copied back inside
the timed region. Total work is fixed as N grows (strong scaling). At one GPU
the line also carries `config.suite`: every op of the other workloads of the
benchmark set (the CPU-runnable broadcast add, the mixed-dtype strided and
transcendental chain, the 3-D reductions and cumsums, the low-precision and
complex elementwise ops), timed through the API in the same run.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

ROWS, COLS, SEED = 1 << 16, 1 << 15, 5
METRIC = "HBM GB/s & % of peak: broadcast add and axis-sum at 1/2/4/8 B200"
WORKLOAD = ("config5: f32 (65536, 32768) uniform[-1,1) seed 5 sharded on axis 0 + replicated (32768,) row; "
            "step = broadcast add -> sum(axis=1) -> sum/mean(all) -> argmax(all)")


def env_int(name: str, default: int) -> int:
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


def shard_rows(n_rows: int, world: int, rank: int):
    base, extra = divmod(n_rows, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def gen_rows(r0: int, r1: int, cols: int, out=None):
    """Rows [r0, r1) of the config-5 matrix from one PCG64 stream (seed 5),
    generated chunk by chunk: each float32 draw consumes half of a 64-bit
    PCG64 step, so the stream is advanced to row r0 directly."""
    import numpy as np

    bg = np.random.PCG64(SEED)
    bg.advance((r0 * cols) // 2)
    rng = np.random.Generator(bg)
    n = r1 - r0
    if out is None:
        out = np.empty((n, cols), dtype=np.float32)
    chunk = max(1, (1 << 24) // cols)
    for i in range(0, n, chunk):
        j = min(n, i + chunk)
        out[i:j] = rng.random((j - i, cols), dtype=np.float32) * 2 - 1
    return out


def gen_row_vector(rows: int, cols: int):
    import numpy as np

    bg = np.random.PCG64(SEED)
    bg.advance((rows * cols) // 2)
    return np.random.Generator(bg).random(cols, dtype=np.float32) * 2 - 1


def gen_rows_parallel(r0: int, r1: int, cols: int, out, threads: int = 0):
    """gen_rows over several host threads: each block of rows advances its
    own copy of the stream, so the result is the same matrix."""
    import concurrent.futures as cf

    threads = threads or min(32, os.cpu_count() or 1)
    n = r1 - r0
    per = max(1, -(-n // (threads * 4)))
    jobs = [(r0 + i, min(r1, r0 + i + per)) for i in range(0, n, per)]
    with cf.ThreadPoolExecutor(max_workers=threads) as ex:
        list(ex.map(lambda j: gen_rows(j[0], j[1], cols, out=out[j[0] - r0:j[1] - r0]), jobs))
    return out


def host_info() -> dict:
    """The GPU box's host: logical CPUs, the CPUs this process may run on,
    the CPU model and the memory available."""
    model = None
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    model = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    try:
        usable = len(os.sched_getaffinity(0))
    except Exception:
        usable = os.cpu_count()
    mem = None
    try:
        import psutil

        mem = round(psutil.virtual_memory().available / 2**30, 1)
    except Exception:
        pass
    return {"nproc": os.cpu_count(), "usable_cpus": usable, "cpu_model": model, "mem_available_gib": mem}


def step_bytes(rows: int, cols: int) -> dict:
    n = rows * cols * 4
    return {
        "add": n + cols * 4 + n,          # read x, read row, write y
        "sum_axis1": n + rows * 4,        # read y, write row sums
        "sum_all": n,                     # read x (sum and mean share the pass)
        "argmax": n,                      # read x
    }


def measured_peak() -> tuple[float, str]:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            v = float(json.load(f)["hbm_gbs"])
        return v, "measured"
    except Exception:
        return 6650.0, "fallback"


def add_traffic(rows: int):
    """DRAM bytes (read + write) of one broadcast-add launch over `rows` rows,
    from the committed ncu captures (profiles/ncu_traffic.json): a capture of
    that very launch size when there is one, else the line through captures
    at two sizes (slope per row + a constant part, e.g. output still dirty in
    L2 when the kernel ends). Returns (bytes or None, how)."""
    p = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    try:
        with open(p) as f:
            caps = json.load(f).get("captures", [])
    except Exception:
        return None, "no capture"
    pts = {}
    for c in caps:
        try:
            pts[int(c["rows"])] = int(c["dram_bytes_read"]) + int(c["dram_bytes_write"])
        except (KeyError, TypeError, ValueError):
            continue
    if rows in pts:
        return pts[rows], f"ncu capture of this launch ({rows} rows)"
    if len(pts) >= 2:
        (r0, b0), (r1, b1) = sorted(pts.items())[-2:]
        slope = (b1 - b0) / (r1 - r0)
        return int(round(b0 + slope * (rows - r0))), f"line through ncu captures at {r0} and {r1} rows"
    return None, "fewer than two captures"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self) -> None:
        self.proc = None

    def start(self) -> None:
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self, gpus) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out, _ = self.proc.communicate()
        mhz, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                idx = int(f[0])
            except ValueError:
                continue
            if idx not in gpus:
                continue
            try:
                mhz.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                pass
            for name, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(mhz) if mhz else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(mhz)}


# --------------------------------------------------------------- CPU legs
def cpu_sample(rows: int, cols: int, threads: int, steps: int, warmup: int) -> dict:
    """The oracle port (the reference CPU path restated) on a bounded sample:
    the first `rows` rows of the same matrix, the same step."""
    import numpy as np

    from oracle import oracle as O

    O.build()
    O.set_threads(threads)
    x = gen_rows(0, rows, cols)
    row = gen_row_vector(ROWS, cols)
    b = step_bytes(rows, cols)

    def one():
        y = O.binary("add", x, row)
        O.reduce("sum", y, axis=1)
        O.reduce("sum", x, None)
        O.reduce("mean", x, None)
        O.reduce("argmax", x, None)

    for _ in range(warmup):
        one()
    t0 = time.perf_counter()
    for _ in range(steps):
        one()
    dt = (time.perf_counter() - t0) / steps
    total = sum(b.values())
    return {"value": total / dt / 1e9, "unit": "GB/s", "cores": threads, "seconds_per_step": dt,
            "host": host_info(),
            "sample": f"first {rows} of {ROWS} rows ({rows * cols} f32 elements), same step, "
                      f"{'1 thread (scalar port)' if threads == 1 else f'{threads} OpenMP threads'}"}


def run_reference(args) -> None:
    """The reference CPU path of the step (the oracle port: musapy's CPU loops
    restated, each output computed in the reference's order; all host
    threads) on the full workload when the host has the memory for it (x and
    y, 16 GiB), else on the first --sample-rows rows. Warm-up steps run on a
    2048-row slice (they only warm the threads and the allocator)."""
    rank = env_int("RANK", 0)
    if rank != 0:
        return
    import numpy as np

    from oracle import oracle as O

    O.build()
    threads = O.max_threads()
    O.set_threads(threads)
    host = host_info()
    need_gib = 2 * ROWS * COLS * 4 / 2**30 + 2
    full = host["mem_available_gib"] is None or host["mem_available_gib"] > need_gib + 8
    rows = ROWS if full else args.sample_rows
    x = np.empty((rows, COLS), dtype=np.float32)
    gen_rows_parallel(0, rows, COLS, x)
    row = gen_row_vector(ROWS, COLS)
    y = np.empty_like(x)
    y.fill(0.0)  # first-touch page faults outside the timed steps

    def one(xs, ys):
        O.binary("add", xs, row, out=ys)
        O.reduce("sum", ys, axis=1)
        O.reduce("sum", xs, None)
        O.reduce("mean", xs, None)
        O.reduce("argmax", xs, None)

    for _ in range(max(0, args.warmup)):
        one(x[:2048], y[:2048])
    steps = max(1, args.steps)
    t0 = time.perf_counter()
    for _ in range(steps):
        one(x, y)
    dt = (time.perf_counter() - t0) / steps
    value = sum(step_bytes(rows, COLS).values()) / dt / 1e9
    sample = (f"the full workload ({rows} x {COLS} f32), same step" if full else
              f"first {rows} of {ROWS} rows (host memory {host['mem_available_gib']} GiB < the {need_gib:.0f} GiB "
              f"the full workload needs)")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": steps, "warmup": args.warmup,
        "ms_per_step": round(dt * 1e3, 3), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "rows": rows, "cols": COLS, "same_config": full,
                   "warmup_sample": "warm-up steps on the first 2048 rows"},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": sample + f", {threads} OpenMP threads", "host": host},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------- GPU leg
def run_b200(args) -> None:
    import numpy as np
    import torch
    import torch.distributed as dist

    world = env_int("WORLD_SIZE", 1)
    rank = env_int("RANK", 0)
    local = env_int("LOCAL_RANK", 0)
    if world != args.gpus:
        if world == 1 and args.gpus > 1:
            raise SystemExit("--gpus N > 1 must be launched with torchrun (one process per GPU)")
    torch.cuda.set_device(local)
    import datetime

    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device(f"cuda:{local}"))
    import musapy_b200 as ms
    from musapy_b200 import shard as sh

    ms.set_default_device(f"cuda:{local}")
    rows, cols = args.rows, COLS
    r0, r1 = shard_rows(rows, world, rank)
    nloc = r1 - r0
    dev = local
    stream = torch.cuda.current_stream(dev)

    # host data (pinned) and the device copies
    host_x = torch.empty((nloc, cols), dtype=torch.float32, pin_memory=True)
    gen_rows(r0, r1, cols, out=host_x.numpy())
    host_row = torch.from_numpy(gen_row_vector(rows, cols)).pin_memory()
    x = ms.empty((nloc, cols), "f32", dev)
    row = ms.empty((cols,), "f32", dev)
    x.torch().copy_(host_x, non_blocking=True)
    row.torch().copy_(host_row, non_blocking=True)
    y = ms.empty((nloc, cols), "f32", dev)
    rowsum = ms.empty((nloc,), "f32", dev)
    xs = sh.ShardedArray(x, (rows, cols), r0)
    ys = sh.ShardedArray(y, (rows, cols), r0)
    sc = sh._SumCombine(dev, ms.float32)
    ac = sh._ArgCombine(dev, world)
    torch.cuda.synchronize()

    nev = 5

    def step(evs=None):
        if evs is not None:
            evs[0].record(stream)
        sh.add(xs, row, out=y)
        if evs is not None:
            evs[1].record(stream)
        sh.sum_axis(ys, 1, out=rowsum)
        if evs is not None:
            evs[2].record(stream)
        sh.sum_all(xs, sc)
        if evs is not None:
            evs[3].record(stream)
        sh.argreduce_all(xs, True, ac)
        if evs is not None:
            evs[4].record(stream)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    barrier()

    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(nev)] for _ in range(args.steps)]
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler()
    if local == 0:
        clocks.start()
        time.sleep(0.4)
    torch.cuda.synchronize()
    barrier()
    launches0 = ms._lib.launch_count()
    t_start.record(stream)
    h0 = time.perf_counter()
    for k in range(args.steps):
        step(evs[k])
    host_ms = (time.perf_counter() - h0) * 1e3 / args.steps  # host time to enqueue one step
    sh.join_exchanges(dev)  # the last record exchanges end inside the timed region
    t_end.record(stream)
    torch.cuda.synchronize()
    launches = ms._lib.launch_count() - launches0
    barrier()
    ms_total = t_start.elapsed_time(t_end)
    op_ms = {name: statistics.mean(e[i].elapsed_time(e[i + 1]) for e in evs)
             for i, name in enumerate(["add", "sum_axis1", "sum_all", "argmax"])}
    clk = clocks.stop(set(range(world))) if local == 0 else None

    # e2e through the library's own transfer entry points: the step's input
    # from pinned host memory to the device (mpb_copy_h2d: one DMA for
    # page-locked memory), the step, the results back (mpb_copy_d2h); both
    # calls return once their copy is done
    from musapy_b200._lib import LIB, check

    host_rowsum = torch.empty((nloc,), dtype=torch.float32, pin_memory=True)
    # one pinned buffer per result in the result's own dtype: a plain D2H copy,
    # no conversion kernel on the device
    host_sum = torch.empty(1, dtype=sc.sum_out.torch().dtype, pin_memory=True)
    host_mean = torch.empty(1, dtype=sc.mean_out.torch().dtype, pin_memory=True)
    host_index = torch.empty(1, dtype=ac.index.torch().dtype, pin_memory=True)
    sraw = stream.cuda_stream
    copies_in = [(x.data_ptr, host_x.data_ptr(), host_x.nbytes), (row.data_ptr, host_row.data_ptr(), host_row.nbytes)]
    copies_out = [(host_rowsum.data_ptr(), rowsum.data_ptr, host_rowsum.nbytes),
                  (host_sum.data_ptr(), sc.sum_out.data_ptr, host_sum.nbytes),
                  (host_mean.data_ptr(), sc.mean_out.data_ptr, host_mean.nbytes),
                  (host_index.data_ptr(), ac.index.data_ptr, host_index.nbytes)]
    e2e_steps = max(1, min(args.steps, args.e2e_steps))

    def e2e_step():
        for d, h, n in copies_in:
            check(LIB.mpb_copy_h2d(d, h, n, sraw), "e2e input copy")
        step()
        sh.join_exchanges(dev)
        for h, d, n in copies_out:
            check(LIB.mpb_copy_d2h(h, d, n, sraw), "e2e result copy")

    e2e_step()  # warm-up: the transfer entry points' first call sets up their events
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / e2e_steps
    h2d = sum(n for _, _, n in copies_in)
    d2h = sum(n for _, _, n in copies_out)

    # max over ranks of the step time, total bytes over ranks
    b_local = step_bytes(nloc, cols)
    vals = torch.tensor([ms_total / args.steps, e2e_ms], dtype=torch.float64, device=f"cuda:{dev}")
    per_rank = None
    if world > 1:
        mine = torch.tensor([ms_total / args.steps] + [op_ms[k] for k in ("add", "sum_axis1", "sum_all", "argmax")],
                            dtype=torch.float64, device=f"cuda:{dev}")
        allr = torch.empty((world, mine.numel()), dtype=torch.float64, device=f"cuda:{dev}")
        dist.all_gather_into_tensor(allr, mine)
        per_rank = [[round(v, 4) for v in r] for r in allr.cpu().tolist()]
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    t_step, t_e2e = float(vals[0]), float(vals[1])
    total_bytes = sum(step_bytes(rows, cols).values())
    value = total_bytes / (t_step * 1e-3) / 1e9
    e2e_value = total_bytes / (t_e2e * 1e-3) / 1e9

    peak, peak_kind = measured_peak()
    add_bytes = b_local["add"]
    achieved = add_bytes / (op_ms["add"] * 1e-3) / 1e9
    traffic, traffic_how = add_traffic(nloc)

    suite = None
    if world == 1 and not args.no_suite:
        del x, y, xs, ys, host_x
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        clocks_s = ClockSampler()
        clocks_s.start()
        time.sleep(0.3)
        suite = {"ops": device_suite(args, peak), "inputs": SUITE_INPUTS}
        torch.cuda.synchronize()
        suite["clocks"] = clocks_s.stop({local})

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_sample(args.sample_rows, cols, 1, 1, 0)

    if world > 1:
        for ex in list(sh._EXCHANGES.values()):
            if ex is not None:
                ex.check()  # a peer-exchange wait that gave up invalidates the run
        sh.close_exchanges()
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": max(3, args.warmup), "ms_per_step": round(t_step, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "rows": rows, "cols": cols, "parallelism": f"axis0-shard{world}",
                   "global_batch": rows, "l2": "inputs 8 GiB > 126 MB L2: no flush needed",
                   "per_op_ms": {k: round(v, 4) for k, v in op_ms.items()},
                   "host_enqueue_ms_per_step": round(host_ms, 4),
                   "per_op_gbs": {k: round(b_local[k] / (v * 1e-3) / 1e9, 1) for k, v in op_ms.items()},
                   "per_op_frac": {k: round(b_local[k] / (v * 1e-3) / 1e9 / peak, 4) for k, v in op_ms.items()}},
        "roofline": {"bound": "hbm", "kernel": "k_ew_rows (broadcast add)", "achieved": round(achieved, 1),
                     "peak": peak, "peak_kind": peak_kind, "unit": "GB/s", "frac": round(achieved / peak, 4),
                     "bytes_per_launch": add_bytes, "traffic": traffic, "traffic_source": traffic_how},
        "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d * world,
                "d2h_bytes_per_step": d2h * world, "ms_per_step": round(t_e2e, 3)},
        "gpu_launches": int(launches),
        "clocks": clk,
    }
    if per_rank is not None:
        line["config"]["per_rank_ms"] = {"columns": ["step", "add", "sum_axis1", "sum_all", "argmax"],
                                         "ranks": per_rank,
                                         "note": "device time per rank (CUDA events); ops on the main stream, "
                                                 "the record exchanges overlap on a side stream"}
    if suite is not None:
        line["config"]["suite"] = suite
    if cpu is not None:
        line["cpu_baseline"] = {"value": round(cpu["value"], 4), "unit": "GB/s", "cores": cpu["cores"],
                                "kind": "port", "sample": cpu["sample"], "host": cpu["host"]}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------- per-config suite
def config_inputs(name: str, scale: int = 1):
    """Seeded inputs of BASELINE configs 1-4 (numpy PCG64; seeds 0, 2, 1, 4).
    `scale` > 1 divides the large extents (C2's chain, C3's leading dim, C4's
    lengths) for small profiling runs; 1 is the benchmark's size."""
    import numpy as np

    if name == "C1":
        rng = np.random.default_rng(0)
        a = rng.random((4096, 1), dtype=np.float32) * 2 - 1
        b = rng.random(4096, dtype=np.float32) * 2 - 1
        return {"a": a, "b": b}
    if name == "C2":
        rng = np.random.default_rng(2)
        A = rng.integers(-1000, 1001, (8192, 8192), dtype=np.int64)
        row = rng.standard_normal(8192)
        x = rng.standard_normal((1 << 28) // scale, dtype=np.float32)
        return {"A": A, "row": row, "x": x}
    if name == "C3":
        rng = np.random.default_rng(1)
        return {"x": rng.standard_normal((64 // scale, 4096, 4096), dtype=np.float32)}
    if name == "C4":
        rng = np.random.default_rng(4)
        n, m = (1 << 30) // scale, (1 << 27) // scale
        x = rng.standard_normal(n, dtype=np.float32)
        a = (0.1 + 3.9 * rng.random(n, dtype=np.float32)).astype(np.float16)
        b = (-2 + 4 * rng.random(n, dtype=np.float32)).astype(np.float16)
        re, im = rng.standard_normal((2, m), dtype=np.float32)
        re2, im2 = rng.standard_normal((2, m), dtype=np.float32)
        return {"x": x, "a": a, "b": b, "z1": (re + 1j * im).astype(np.complex64),
                "z2": (re2 + 1j * im2).astype(np.complex64)}
    raise KeyError(name)


def run_suite(args) -> None:
    import gc

    import numpy as np

    import torch

    import musapy_b200 as ms

    ms.set_default_device("cuda:0")
    peak, peak_kind = measured_peak()
    stream = torch.cuda.current_stream()

    def timeit(fn, nbytes, iters=None):
        iters = iters or args.steps
        for _ in range(max(3, args.warmup)):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n0 = ms._lib.launch_count()
        e0.record(stream)
        for _ in range(iters):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        ms_per = e0.elapsed_time(e1) / iters
        return ms_per, nbytes / (ms_per * 1e-3) / 1e9, (ms._lib.launch_count() - n0) // iters

    def timeit_graph(fn, nbytes, reps=20):
        """Device time per call with the calls replayed from a CUDA graph, so
        the host-side cost of each API call (Python, argument checks) drops out
        and only the kernels' own time remains."""
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(3):
                fn()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for _ in range(reps):
                fn()
        for _ in range(max(3, args.warmup)):
            g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            g.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        ms_per = e0.elapsed_time(e1) / (args.steps * reps)
        del g
        return ms_per, nbytes / (ms_per * 1e-3) / 1e9

    O = None
    if args.suite_cpu:
        from oracle import oracle as O

        O.build()
        O.set_threads(1)

    def cpu_leg(cpu):
        """The reference CPU path (the oracle port, one thread, as the
        reference's CPU loops are) on a bounded sample of the same op:
        (callable, algorithmic bytes of the sample, description)."""
        fn, nb, desc = cpu
        fn()
        reps, t0 = 0, time.perf_counter()
        while True:
            fn()
            reps += 1
            el = time.perf_counter() - t0
            if el > 1.0 or reps >= 5:
                break
        sec = el / reps
        return {"value": round(nb / sec / 1e9, 4), "unit": "GB/s", "cores": 1, "kind": "port",
                "sample": desc, "ms": round(sec * 1e3, 2)}

    def emit(cfg, op, nbytes, fn, note="", graph=False, cpu=None, iters=None):
        t, gbs, launches = timeit(fn, nbytes, iters)
        line = {"config": cfg, "op": op, "ms": round(t, 4), "gbs": round(gbs, 1),
                "frac": round(gbs / peak, 4), "bytes": int(nbytes), "launches": launches,
                "peak": peak, "peak_kind": peak_kind, "note": note, "scale": args.scale}
        if graph:
            tg, gg = timeit_graph(fn, nbytes)
            line["graph"] = {"ms": round(tg, 4), "gbs": round(gg, 1), "frac": round(gg / peak, 4)}
        if cpu is not None and O is not None:
            line["cpu_baseline"] = cpu_leg(cpu)
        print(json.dumps(line), flush=True)

    cfgs = args.suite.split(",")
    if "C1" in cfgs:
        d = config_inputs("C1")
        a, b = ms.from_numpy(d["a"]), ms.from_numpy(d["b"])
        c = ms.add(a, b)
        r = ms.sum(c, axis=1)
        ch = c.numpy()
        emit("C1", "add (4096,1)+(4096,)", 4096 * 4 * 2 + 4096 * 4096 * 4, lambda: ms.add(a, b, out=c),
             note="64 MB output: per-call host cost is a large part of ms; graph = kernels alone", graph=True,
             cpu=(lambda: O.binary("add", d["a"], d["b"]), 4096 * 4 * 2 + 4096 * 4096 * 4, "whole op"),
             iters=max(args.steps, 200))
        emit("C1", "sum axis=1", 4096 * 4096 * 4 + 4096 * 4, lambda: ms.sum(c, axis=1, out=r), graph=True,
             cpu=(lambda: O.reduce("sum", ch, 1), 4096 * 4096 * 4 + 4096 * 4, "whole op"), iters=max(args.steps, 200))
    if "C2" in cfgs:
        d = config_inputs("C2", args.scale)
        A, row, x = ms.from_numpy(d["A"]), ms.from_numpy(d["row"]), ms.from_numpy(d["x"])
        As, rs, xs = d["A"][:512], d["row"][:512], d["x"][: 1 << 22]
        del d
        At = ms.transpose(A)
        o = ms.add(At, row)
        emit("C2", "add i64^T (8192,8192) + f64 row -> f64", 8192 * 8192 * 8 * 2 + 8192 * 8,
             lambda: ms.add(At, row, out=o),
             cpu=(lambda: O.binary("add", As.T, rs), 512 * 8192 * 16 + 512 * 8, "A[:512]^T + row[:512]"))
        s = ms.sin(x)
        e = ms.exp(s)
        cl = ms.clamp(e, -0.5, 0.5)
        n = x.size
        ss = xs if O is None else O.unary("sin", xs)
        es = ss if O is None else O.unary("exp", ss)
        emit("C2", "sin f32 2^28", n * 8, lambda: ms.sin(x, out=s),
             cpu=(lambda: O.unary("sin", xs), (1 << 22) * 8, "first 2^22 elements"))
        emit("C2", "exp f32 2^28", n * 8, lambda: ms.exp(s, out=e),
             cpu=(lambda: O.unary("exp", ss), (1 << 22) * 8, "first 2^22 elements"))
        emit("C2", "clamp f32 2^28", n * 8, lambda: ms.clamp(e, -0.5, 0.5, out=cl),
             cpu=(lambda: O.clamp(es, -0.5, 0.5), (1 << 22) * 8, "first 2^22 elements"))
        del A, At, o, s, e, cl, x, row
    if "C3" in cfgs:
        xh = config_inputs("C3", args.scale)["x"]
        x = ms.from_numpy(xh)
        n = xh.nbytes
        P = xh.shape[0]
        # CPU samples: 2 of the 64 planes for axis 2 / argmax / cumsum, 128 of
        # the 4096 rows of every plane for axis 0 and (0, 2)
        s2, s0 = xh[:2], np.ascontiguousarray(xh[:, :128])
        samp = {2: (s2, s2.nbytes, "x[:2]"), 0: (s0, s0.nbytes, "x[:, :128]"), (0, 2): (s0, s0.nbytes, "x[:, :128]")}
        for axis, oelems in [(2, P * 4096), (0, 4096 * 4096), ((0, 2), 4096)]:
            for op in ("sum", "max", "mean"):
                out = getattr(ms, op)(x, axis=axis)
                f = (lambda op=op, axis=axis: getattr(ms, op)(x, axis=axis)) if isinstance(axis, tuple) else \
                    (lambda op=op, axis=axis, out=out: getattr(ms, op)(x, axis=axis, out=out))
                sx, sb, sd = samp[axis]
                emit("C3", f"{op} axis={axis}", n + oelems * 4, f,
                     cpu=(lambda op=op, axis=axis, sx=sx: O.reduce(op, sx, axis), sb, sd))
        am = ms.argmax(x, axis=1)
        emit("C3", "argmax axis=1", n + P * 4096 * 8, lambda: ms.argmax(x, axis=1, out=am),
             cpu=(lambda: O.reduce("argmax", s2, 1), s2.nbytes + 2 * 4096 * 8, "x[:2]"))
        cs = ms.cumsum(x, axis=-1)
        emit("C3", "cumsum axis=-1", 2 * n, lambda: ms.cumsum(x, axis=-1, out=cs),
             cpu=(lambda: O.cumsum(s2, -1), 2 * s2.nbytes, "x[:2] (running-sum form)"))
        del x, cs, am, xh, s2, s0
    if "C4" in cfgs:
        d = config_inputs("C4", args.scale)
        n = d["x"].size
        x = ms.from_numpy(d["x"])
        m = 1 << 22
        xs_, as_, bs_, z1s, z2s = d["x"][:m], d["a"][:m], d["b"][:m], d["z1"][:m], d["z2"][:m]
        xbs = xs_ if O is None else O.cast(xs_, O.BF16)
        xb = x.astype("bf16")
        back = xb.astype("f32")
        emit("C4", "astype f32->bf16 2^30", n * 6, lambda: ms.astype(x, "bf16", out=xb),
             cpu=(lambda: O.cast(xs_, O.BF16), m * 6, "first 2^22 elements"))
        emit("C4", "astype bf16->f32 2^30", n * 6, lambda: ms.astype(xb, "f32", out=back),
             cpu=(lambda: O.cast(xbs, O.F32), m * 6, "first 2^22 elements"))
        del x, xb, back
        a, b = ms.from_numpy(d["a"]), ms.from_numpy(d["b"])
        p = ms.pow(a, b)
        emit("C4", "pow f16 2^30", n * 6, lambda: ms.pow(a, b, out=p),
             cpu=(lambda: O.binary("pow", as_, bs_), m * 6, "first 2^22 elements"))
        del p
        lt = ms.lt(a, b)
        emit("C4", "lt f16 -> bool 2^30", n * 5, lambda: ms.lt(a, b, out=lt),
             cpu=(lambda: O.compare("lt", as_, bs_), m * 5, "first 2^22 elements"))
        emit("C4", "eq f16 -> bool 2^30", n * 5, lambda: ms.eq(a, b, out=lt),
             cpu=(lambda: O.compare("eq", as_, bs_), m * 5, "first 2^22 elements"))
        del a, b, lt
        z1, z2 = ms.from_numpy(d["z1"]), ms.from_numpy(d["z2"])
        z = ms.mul(z1, z2)
        emit("C4", "mul c64 2^27", d["z1"].size * 24, lambda: ms.mul(z1, z2, out=z),
             cpu=(lambda: O.binary("mul", z1s, z2s), m * 24, "first 2^22 elements"))
        del z1, z2, z, d
    if "SCAN" in cfgs:
        # cumsum of 2^30 / scale f32 N(0,1): flattened (one decoupled look-back
        # scan) and along rows of 4096 (one CTA per row)
        n = (1 << 30) // args.scale
        x = ms.empty((n,), "f32")
        x.torch().normal_(generator=torch.Generator(device="cuda").manual_seed(1))
        c = ms.cumsum(x)
        emit("SCAN", f"cumsum axis=None f32 {n}", 8 * n, lambda: ms.cumsum(x, out=c))
        xr = ms.reshape(x, (n // 4096, 4096))
        cr = ms.cumsum(xr, axis=-1)
        emit("SCAN", f"cumsum axis=-1 f32 ({n // 4096}, 4096)", 8 * n, lambda: ms.cumsum(xr, axis=-1, out=cr))
        del x, c, xr, cr
    if "VIEWS" in cfgs:
        # contiguous() of transposed 16384^2 views (the padded-tile kernel for
        # 4-byte elements, TMA tiles for 2-byte ones); small enough to profile
        q = 16384
        for dt_, esz in (("f32", 4), ("f16", 2)):
            v = ms.reshape(ms.arange(q * q, dtype=dt_), (q, q))
            t = ms.contiguous(ms.transpose(v))
            emit("VIEWS", f"contiguous(transpose) {dt_} (16384,16384)", 2 * q * q * esz,
                 lambda v=v, t=t: ms.contiguous(ms.transpose(v), out=t))
            del v, t
    if "NEXT" in cfgs:
        # the rows around the hot path: contiguous copies of views, creation
        # kernels, host <-> device transfers (device-side bytes = read + write)
        q = 16384
        x = ms.arange(q * q, dtype="f32")
        x2 = ms.reshape(x, (q, q))
        t = ms.contiguous(ms.transpose(x2))
        emit("NEXT", "contiguous(transpose) f32 (16384,16384)", 2 * q * q * 4,
             lambda: ms.contiguous(ms.transpose(x2), out=t))
        f = ms.contiguous(ms.flip(x, 0))
        emit("NEXT", "contiguous(flip) f32 2^28", 2 * q * q * 4, lambda: ms.contiguous(ms.flip(x, 0), out=f))
        w = ms.reshape(x, (q // 2, 2 * q))
        half = ms.contiguous(ms.slice(w, [[0, q // 2, 1], [0, 2 * q, 2]]))
        emit("NEXT", "contiguous(x[:, ::2]) f32 (8192,32768)->(8192,16384)", 2 * (q * q // 2) * 4,
             lambda: ms.contiguous(ms.slice(w, [[0, q // 2, 1], [0, 2 * q, 2]]), out=half))
        del t, f, half, w, x2
        # one rank's local full reductions in the 8-GPU config-5 run (1 GiB)
        s1 = ms.sum(x)
        emit("NEXT", "sum all f32 2^28 (8-GPU shard size)", q * q * 4, lambda: ms.sum(x, out=s1), graph=True)
        a1 = ms.argmax(x)
        emit("NEXT", "argmax all f32 2^28 (8-GPU shard size)", q * q * 4, lambda: ms.argmax(x, out=a1), graph=True)
        n = 1 << 30
        emit("NEXT", "arange f32 2^30", n * 4, lambda: ms.arange(0, n, 1, dtype="f32"))
        emit("NEXT", "linspace f64 2^28", (1 << 28) * 8, lambda: ms.linspace(-1.0, 1.0, 1 << 28))
        emit("NEXT", "eye f32 (32768,32768)", 32768 * 32768 * 4, lambda: ms.eye(32768, dtype="f32"))
        host = np.ones(1 << 28, dtype=np.float32)
        import time as _time

        for name, fn in (("from_numpy 1 GiB f32 (pageable host)", lambda: ms.from_numpy(host)),
                         ("Array.numpy() 1 GiB f32", lambda: x.numpy())):
            fn()
            torch.cuda.synchronize()
            t0 = _time.perf_counter()
            for _ in range(3):
                fn()
            torch.cuda.synchronize()
            dt_ms = (_time.perf_counter() - t0) / 3 * 1e3
            nb = (1 << 28) * 4
            print(json.dumps({"config": "NEXT", "op": name, "ms": round(dt_ms, 3),
                              "gbs": round(nb / (dt_ms * 1e-3) / 1e9, 2), "bytes": nb,
                              "note": "wall clock, PCIe-bound"}), flush=True)
        del x, host
    gc.collect()
    torch.cuda.empty_cache()


SUITE_INPUTS = ("the CPU-runnable broadcast add from its numpy seed; the other workloads' inputs drawn on the "
                "device by torch's seeded generator with the same shapes, dtypes and value distributions as their "
                "numpy-seeded versions (the parity tests check those): N(0,1), uniform ints in [-1000, 1000], "
                "uniform[0.1,4) and uniform[-2,2) f16, complex64 with N(0,1) parts. CUDA events over back-to-back "
                "API calls after warm-up; every input except the broadcast add's is larger than the L2; that one "
                "(64 MB) is also replayed from a CUDA graph, which drops the per-call host cost")


def device_suite(args, peak: float) -> list:
    """Every op of the benchmark set's other workloads, timed through the
    public API on the current GPU (ms per call, GB/s of algorithmic bytes,
    fraction of the measured HBM peak)."""
    import numpy as np
    import torch

    import musapy_b200 as ms

    stream = torch.cuda.current_stream()
    iters = max(10, args.steps)
    out = []

    def timeit(fn, n):
        for _ in range(max(3, args.warmup)):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        l0 = ms._lib.launch_count()
        e0.record(stream)
        for _ in range(n):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / n, (ms._lib.launch_count() - l0) // n

    def graph_ms(fn, reps=20):
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(3):
                fn()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for _ in range(reps):
                fn()
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(iters):
            g.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        del g
        return e0.elapsed_time(e1) / (iters * reps)

    def emit(cfg, op, nbytes, fn, n=None, graph=False):
        t, launches = timeit(fn, n or iters)
        gbs = nbytes / (t * 1e-3) / 1e9
        e = {"config": cfg, "op": op, "ms": round(t, 4), "gbs": round(gbs, 1), "frac": round(gbs / peak, 4),
             "bytes": int(nbytes), "launches": launches}
        if graph:
            tg = graph_ms(fn)
            gg = nbytes / (tg * 1e-3) / 1e9
            e["graph"] = {"ms": round(tg, 4), "gbs": round(gg, 1), "frac": round(gg / peak, 4)}
        out.append(e)

    def dev(shape, dtype):
        a = ms.empty(shape, dtype)
        return a, a.torch()

    gen = torch.Generator(device="cuda")

    # C1: (4096,1) + (4096,) f32 from numpy seed 0, then sum(axis=1)
    d = config_inputs("C1")
    a, b = ms.from_numpy(d["a"]), ms.from_numpy(d["b"])
    c = ms.add(a, b)
    r = ms.sum(c, axis=1)
    emit("C1", "add (4096,1)+(4096,) f32", 4096 * 8 + 4096 * 4096 * 4, lambda: ms.add(a, b, out=c), n=200,
         graph=True)
    emit("C1", "sum axis=1 (4096,4096) f32", 4096 * 4096 * 4 + 4096 * 4, lambda: ms.sum(c, axis=1, out=r), n=200,
         graph=True)
    del a, b, c, r

    # C2: int64 (8192,8192) read transposed + f64 row; f32 chain on 2^28
    gen.manual_seed(2)
    A, At_ = dev((8192, 8192), "i64")
    At_.random_(-1000, 1001, generator=gen)
    row, rt = dev((8192,), "f64")
    rt.normal_(generator=gen)
    x, xt = dev((1 << 28,), "f32")
    xt.normal_(generator=gen)
    AT = ms.transpose(A)
    o = ms.add(AT, row)
    emit("C2", "add int64^T (8192,8192) + f64 row -> f64", 8192 * 8192 * 16 + 8192 * 8, lambda: ms.add(AT, row, out=o))
    s_ = ms.sin(x)
    e_ = ms.exp(s_)
    cl = ms.clamp(e_, -0.5, 0.5)
    n = 1 << 28
    emit("C2", "sin f32 2^28", n * 8, lambda: ms.sin(x, out=s_))
    emit("C2", "exp f32 2^28", n * 8, lambda: ms.exp(s_, out=e_))
    emit("C2", "clamp f32 2^28", n * 8, lambda: ms.clamp(e_, -0.5, 0.5, out=cl))
    del A, At_, row, rt, x, xt, AT, o, s_, e_, cl

    # C3: f32 (64,4096,4096) N(0,1)
    gen.manual_seed(1)
    x, xt = dev((64, 4096, 4096), "f32")
    xt.normal_(generator=gen)
    nb = 64 * 4096 * 4096 * 4
    for axis, outs in ((2, 64 * 4096), (0, 4096 * 4096), ((0, 2), 4096)):
        for op in ("sum", "max", "mean"):
            f = getattr(ms, op)
            res = f(x, axis=axis)
            emit("C3", f"{op} axis={axis}", nb + outs * 4, lambda f=f, axis=axis, res=res: f(x, axis=axis, out=res))
    am = ms.argmax(x, axis=1)
    emit("C3", "argmax axis=1 -> int64", nb + 64 * 4096 * 8, lambda: ms.argmax(x, axis=1, out=am))
    del am
    cs = ms.cumsum(x, axis=-1)
    emit("C3", "cumsum axis=-1 (262144 rows of 4096)", 2 * nb, lambda: ms.cumsum(x, axis=-1, out=cs))
    del cs
    cf = ms.cumsum(x)
    emit("C3", "cumsum axis=None (2^30, one decoupled look-back scan)", 2 * nb, lambda: ms.cumsum(x, out=cf))
    del cf, x, xt

    # C4: 2^30 casts / f16 pow / compares, complex64 mul of 2^27
    gen.manual_seed(4)
    n = 1 << 30
    x, xt = dev((n,), "f32")
    xt.normal_(generator=gen)
    xb = x.astype("bf16")
    back = xb.astype("f32")
    emit("C4", "astype f32->bf16 2^30", n * 6, lambda: ms.astype(x, "bf16", out=xb))
    emit("C4", "astype bf16->f32 2^30", n * 6, lambda: ms.astype(xb, "f32", out=back))
    del x, xt, xb, back
    a, at = dev((n,), "f16")
    at.uniform_(0.1, 4.0, generator=gen)
    b, bt = dev((n,), "f16")
    bt.uniform_(-2.0, 2.0, generator=gen)
    p = ms.pow(a, b)
    emit("C4", "pow f16 2^30", n * 6, lambda: ms.pow(a, b, out=p))
    del p
    lt = ms.lt(a, b)
    emit("C4", "lt f16 -> bool 2^30", n * 5, lambda: ms.lt(a, b, out=lt))
    emit("C4", "eq f16 -> bool 2^30", n * 5, lambda: ms.eq(a, b, out=lt))
    del a, at, b, bt, lt
    m = 1 << 27
    z1, z1t = dev((m,), "c64")
    torch.view_as_real(z1t).normal_(generator=gen)
    z2, z2t = dev((m,), "c64")
    torch.view_as_real(z2t).normal_(generator=gen)
    z = ms.mul(z1, z2)
    emit("C4", "mul c64 2^27", m * 24, lambda: ms.mul(z1, z2, out=z))
    del z1, z1t, z2, z2t, z

    # the transposed copies of the views row (contiguous() of a transpose)
    q = 16384
    for dt_, esz in (("f32", 4), ("f16", 2)):
        v, vt = dev((q, q), dt_)
        vt.normal_(generator=gen)
        t = ms.contiguous(ms.transpose(v))
        emit("views", f"contiguous(transpose) {dt_} (16384,16384)", 2 * q * q * esz,
             lambda v=v, t=t: ms.contiguous(ms.transpose(v), out=t))
        del v, vt, t
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    del np
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--rows", type=int, default=ROWS, help="global rows (default: config 5)")
    ap.add_argument("--sample-rows", type=int, default=2048, help="rows of the CPU sample")
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-suite", action="store_true", help="skip the per-op table of the other workloads")
    ap.add_argument("--suite", default="", help="comma list of C1..C4, SCAN, VIEWS, NEXT: time every op of those configs")
    ap.add_argument("--scale", type=int, default=1,
                    help="with --suite: divide the large extents of C2-C4 by this power of two (profiling runs)")
    ap.add_argument("--suite-cpu", action="store_true",
                    help="with --suite: also time the reference CPU path (oracle port, 1 thread) on a sample")
    args = ap.parse_args()
    if args.suite:
        run_suite(args)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
