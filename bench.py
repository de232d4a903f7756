"""Benchmark: bit-exact sf16 elementwise ops on B200 (Gelem/s), with the wide
8192^3 and chain 512^3 matmuls measured beside it.

One step = the five status-reporting sf16 ops (add, sub, mul, fma, div) over
2^26-element inputs resident in HBM, each op's exact event counts reduced on
the device (and all-reduced over ranks when N > 1: the status exchange).
``value`` = elements processed by all ranks / max-over-ranks device time.
``e2e`` = the same ops on codes in pinned HOST memory (int16, the device
word's width): the host->device copies of every step's inputs, the kernels,
the device->host copies of the result codes and the read of the status
counts are all inside the timed region (chunked over two streams so copies
overlap kernels).  ``e2e_plugin_int64`` is the reference's own plug-in
contract, ``Device.run`` on int64 NumPy arrays returning int64 codes and
boolean masks, once per op.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

N > 1 is launched with torchrun; each rank runs its own 2^26 elements (weak
scaling, no data-path collective; only the status counts are all-reduced).
``--impl reference`` times the reference's host implementation of the same
ops (the oracle's NumPy restatement of src/sf/_vectorized.py, the reference's
own code path being NumPy) on this host's cores, on rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

OPS = ("add", "sub", "mul", "fma", "div")
N_ELEM = 1 << 26
BYTES_PER_ELEM = {"add": 6, "sub": 6, "mul": 6, "div": 6, "fma": 8}   # int16 reads + write
METRIC = "bit-exact sf16 matmul TOPS + elementwise Gelem/s at 1/2/4/8 B200 vs host CPU"


def _env_int(k, d):
    try:
        return int(os.environ.get(k, d))
    except ValueError:
        return d


def peaks():
    p = os.path.join(HERE, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d.get("hbm_gbs", 6650.0), "measured"
    return 6650.0, "fallback"


def traffic_from_profiles(kernel_key):
    """DRAM bytes per launch recorded by ncu (profiles/ncu_traffic.txt:
    '<key> <bytes per launch>' lines), or None."""
    p = os.path.join(HERE, "profiles", "ncu_traffic.txt")
    if not os.path.exists(p):
        return None
    for line in open(p):
        parts = line.split()
        if len(parts) >= 2 and parts[0] == kernel_key:
            try:
                return float(parts[1])
            except ValueError:
                return None
    return None


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.p = None

    def start(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                       "-lms", "200", "-i", str(self.idx)], stdout=subprocess.PIPE,
                                      stderr=subprocess.DEVNULL, text=True)
        except (OSError, FileNotFoundError):
            self.p = None

    def stop(self):
        if self.p is None:
            return None
        time.sleep(0.25)
        self.p.terminate()
        try:
            out, _ = self.p.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.p.kill()
            out, _ = self.p.communicate()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax), "reasons": sorted(reasons),
                "samples": len(sm)}


def cpu_sample(n_sample):
    """The oracle's NumPy ops (the reference's own NumPy formulation) on
    n_sample elements of the same workload, single-threaded."""
    from oracle import sfref
    from superfloat.python_b200 import workloads
    x, y, z, d = workloads.elementwise(n_sample, 0)
    args = {"add": (x, y), "sub": (x, y), "mul": (x, y), "fma": (x, y, z), "div": (x, d)}
    t0 = time.perf_counter()
    for op in OPS:
        sfref.ew(op, 16, *args[op])
    return time.perf_counter() - t0


def _cpu_pool_worker(n):
    return cpu_sample(n)


def host_cores() -> int:
    """CPUs this process may run on: the affinity mask, capped by a cgroup v2
    CPU quota when one is set (a container can see more cores than it gets)."""
    try:
        n = len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        n = os.cpu_count() or 1
    try:
        quota, period = open("/sys/fs/cgroup/cpu.max").read().split()[:2]
        if quota != "max":
            n = min(n, max(1, int(int(quota) / int(period))))
    except (OSError, ValueError):
        pass
    return max(1, n)


def run_reference(args, rank, world):
    if rank != 0:
        return 0
    import multiprocessing as mp
    cores = host_cores()
    n_sample = 1 << 22                             # per process per step
    ctx = mp.get_context("spawn")
    with ctx.Pool(cores) as pool:
        for _ in range(args.warmup):
            pool.map(_cpu_pool_worker, [n_sample] * cores)
        times = []
        for _ in range(args.steps):
            t0 = time.perf_counter()
            pool.map(_cpu_pool_worker, [n_sample] * cores)
            times.append(time.perf_counter() - t0)
    elems = len(OPS) * n_sample * cores
    ms = 1e3 * statistics.median(times)
    v = elems / (ms / 1e3) / 1e9
    line = {"metric": METRIC, "value": v, "unit": "Gelem/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int64", "data": "synthetic",
            "config": {"workload": "sf16 elementwise add/sub/mul/fma/div with status, seeded (2^26 generator)",
                       "sample_elements_per_op": n_sample * cores, "processes": cores},
            "impl": "reference",
            "cpu_baseline": {"value": v, "unit": "Gelem/s", "cores": cores, "kind": "port",
                             "sample": f"{n_sample} elements x 5 ops per process, {cores} spawn processes"},
            "e2e": {"value": v, "unit": "Gelem/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--elements", type=int, default=N_ELEM)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-matmul", action="store_true")
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--matmul-only", type=int, default=0, metavar="SIZE",
                    help="time only the wide and chain matmuls, wide at SIZE^3 (a small case for profiling)")
    ap.add_argument("--wide", action="store_true", help="with --gpt2-only: the accumulate=\"wide\" conversion")
    ap.add_argument("--chain-only", action="store_true",
                    help="time only the proven chain kernel on the GPT-2-small projection shapes")
    ap.add_argument("--sweep-only", action="store_true", help="time only the exhaustive sf16 pair sweep")
    ap.add_argument("--gpt2-only", type=int, default=0, metavar="TOKENS",
                    help="time only the converted GPT-2-small forward on 8 x TOKENS ids")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    rank, world, local = _env_int("RANK", 0), _env_int("WORLD_SIZE", 1), _env_int("LOCAL_RANK", 0)
    if args.impl == "reference":
        return run_reference(args, rank, world)

    import torch
    import torch.distributed as dist
    from superfloat.python_b200 import FORMATS, B200Device, _lib, workloads
    torch.cuda.set_device(local)
    if args.matmul_only:
        print(json.dumps(bench_matmuls(B200Device(local), FORMATS[16], torch, args.matmul_only)), flush=True)
        return 0
    if args.chain_only:
        print(json.dumps(bench_chain_shapes(torch)), flush=True)
        return 0
    if args.sweep_only:
        print(json.dumps(bench_sweep(torch, None, 0, 1)), flush=True)
        return 0
    if args.gpt2_only and args.wide:
        print(json.dumps(bench_gpt2(torch, seq=args.gpt2_only, accumulate="wide")), flush=True)
        return 0
    if args.gpt2_only:
        print(json.dumps(bench_gpt2(torch, seq=args.gpt2_only)), flush=True)
        return 0
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    dev = B200Device(local)
    fmt = FORMATS[16]
    n = args.elements
    x, y, z, d = workloads.elementwise(n, seed=rank)
    tx, ty, tz, td = (dev.upload(v) for v in (x, y, z, d))
    outs = {op: torch.empty(n, dtype=torch.int16, device=dev.torch_device) for op in OPS}
    counts = torch.zeros(len(OPS), _lib.N_COUNTS, dtype=torch.int64, device=dev.torch_device)
    targs = {"add": (tx, ty), "sub": (tx, ty), "mul": (tx, ty), "fma": (tx, ty, tz), "div": (tx, td)}
    stream = torch.cuda.current_stream()

    # one count buffer per step, zeroed by the step itself.  The element ranges
    # are independent, so no rank needs another's counts during the run: every
    # step's counters are summed over the ranks in one all-reduce at the end of
    # the timed region (a per-step all-reduce ran beside the next step's first
    # kernel on NCCL's stream and slowed it)
    allbufs = torch.zeros(max(args.steps, args.warmup), len(OPS), _lib.N_COUNTS, dtype=torch.int64,
                          device=dev.torch_device)
    bufs = list(allbufs.unbind(0))

    def step(evs=None, buf=None):
        buf.zero_()
        for i, op in enumerate(OPS):
            if evs is not None:
                evs[op][0].record(stream)
            dev.run_device(op, fmt, *targs[op], out=outs[op], counts=buf[i])
            if evs is not None:
                evs[op][1].record(stream)

    def drain():
        if world > 1:
            dist.all_reduce(allbufs)

    for i in range(args.warmup):
        step(buf=bufs[i])
    drain()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    per_op = {op: [] for op in OPS}
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t_start.record(stream)
    evs_all = []
    for i in range(args.steps):
        evs = {op: (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for op in OPS}
        step(evs, bufs[i])
        evs_all.append(evs)
    drain()                                  # the status reduction is part of the timed work
    t_end.record(stream)
    counts = bufs[args.steps - 1]
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = sampler.stop() if sampler else None
    ms_total = t_start.elapsed_time(t_end)
    for evs in evs_all:
        for op in OPS:
            per_op[op].append(evs[op][0].elapsed_time(evs[op][1]))
    t = torch.tensor([ms_total], dtype=torch.float64, device=dev.torch_device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_total = float(t.item())
    ms_step = ms_total / args.steps
    elems = len(OPS) * n * world * args.steps
    value = elems / (ms_total / 1e3) / 1e9

    # status check: the step's counts are the oracle's on a sample (sanity, rank 0)
    cnt = counts.cpu().numpy()

    hbm, peak_kind = peaks()
    mean_ms = {op: statistics.mean(v) for op, v in per_op.items()}
    dom = max(mean_ms, key=mean_ms.get)
    achieved = BYTES_PER_ELEM[dom] * n / (mean_ms[dom] / 1e3) / 1e9
    traffic = traffic_from_profiles(f"ew_{dom}_{n}")
    roofline = {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                "traffic": traffic, "kernel": f"ew_kernel<{dom}>", "peak_kind": peak_kind,
                "per_op_GBps": {op: BYTES_PER_ELEM[op] * n / (mean_ms[op] / 1e3) / 1e9 for op in OPS},
                "algorithmic_bytes_per_launch": BYTES_PER_ELEM[dom] * n}

    line = {"metric": METRIC, "value": value, "unit": "Gelem/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int16", "data": "synthetic",
            "config": {"workload": "sf16 elementwise add/sub/mul/fma/div with exact status counts, "
                                   f"{n} elements per op per rank (seeded 2^26 generator)",
                       "elements_per_op_per_rank": n, "l2": "inputs larger than L2 (3 x 128 MiB per op)",
                       "parallelism": f"element-range shards x{world}, status all-reduce"},
            "gpu_launches": len(OPS) * args.steps, "roofline": roofline,
            "status_counts_last_step": {op: {"overflow": int(cnt[i][0]), "underflow": int(cnt[i][1]),
                                             "divide": int(cnt[i][2])} for i, op in enumerate(OPS)}}
    if clocks:
        line["clocks"] = clocks

    # end to end: codes in pinned host memory, copies inside the timed region
    if not args.no_e2e:
        from superfloat.python_b200._hostpath import HostPipeline, plugin_run
        pipe = HostPipeline(dev)
        hx = {}
        for name, v in (("x", x), ("y", y), ("z", z), ("d", d)):
            t = torch.empty(n, dtype=torch.int16, pin_memory=True)
            t.copy_(torch.from_numpy(v))
            hx[name] = t
        hargs = {"add": ("x", "y"), "sub": ("x", "y"), "mul": ("x", "y"), "fma": ("x", "y", "z"), "div": ("x", "d")}
        hout = {op: torch.empty(n, dtype=torch.int16, pin_memory=True) for op in OPS}
        for op in OPS:                               # warm-up of the host path
            pipe.run(op, fmt, *(hx[a] for a in hargs[op]), out=hout[op])
        e2e_steps = max(1, min(5, args.steps))
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        t0 = time.perf_counter()
        for _ in range(e2e_steps):
            for op in OPS:
                pipe.run(op, fmt, *(hx[a] for a in hargs[op]), out=hout[op])   # returns after the counts are read
        dt = torch.tensor([time.perf_counter() - t0], dtype=torch.float64, device=dev.torch_device)
        if world > 1:
            dist.all_reduce(dt, op=dist.ReduceOp.MAX)
        dt = float(dt.item())
        h2d = sum(2 * n * len(hargs[op]) for op in OPS)
        d2h = sum(2 * n + 8 * _lib.N_COUNTS for op in OPS)
        line["e2e"] = {"value": len(OPS) * n * world * e2e_steps / dt / 1e9, "unit": "Gelem/s",
                       "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                       "path": "int16 codes in pinned host memory -> chunked H2D / sfb_elementwise / D2H on two "
                               "streams, status counts read back every op"}
        # the reference's Device.run contract: int64 NumPy codes in, int64 codes + boolean masks out
        xs = {"add": (x, y), "sub": (x, y), "mul": (x, y), "fma": (x, y, z), "div": (x, d)}
        plugin_run(dev, pipe, "add", fmt, x[:4096], y[:4096])
        t0 = time.perf_counter()
        for op in OPS:
            plugin_run(dev, pipe, op, fmt, *xs[op])
        dtp = time.perf_counter() - t0
        line["e2e_plugin_int64"] = {"value": len(OPS) * n / dtp / 1e9, "unit": "Gelem/s",
                                    "path": "B200Device.run contract: int64 NumPy codes in, int64 codes and "
                                            "boolean event masks out (host narrowing / widening included)"}

    # CPU baseline on rank 0, N = 1
    if rank == 0 and world == 1 and not args.no_cpu:
        n_sample = 1 << 22
        cpu_sample(1 << 16)
        reps = 3
        ts = [cpu_sample(n_sample) for _ in range(reps)]
        v = len(OPS) * n_sample / statistics.median(ts) / 1e9
        line["cpu_baseline"] = {"value": v, "unit": "Gelem/s", "cores": 1, "kind": "port",
                                "sample": f"{n_sample} elements x 5 ops, NumPy, median of {reps}"}

    # the exhaustive pair sweep beside it, row-sharded over all ranks: not part of `value`
    if not args.no_sweep:
        sw = bench_sweep(torch, dist, rank, world, cpu=(rank == 0 and world == 1 and not args.no_cpu))
        if rank == 0:
            line["sweep"] = sw

    # the matmuls beside it: not part of `value`.  The wide one row-sharded over all
    # ranks; chain 512^3 and the converted GPT-2 forward on rank 0 at N = 1.
    if not args.no_matmul:
        mm = bench_matmuls(dev, fmt, torch, rank=rank, world=world, dist=dist)
        if rank == 0 and world == 1:
            mm["chain_gpt2_projections"] = bench_chain_shapes(torch)
            mm["gpt2_small_convert"] = bench_gpt2(torch)
            mm["gpt2_small_convert_wide"] = bench_gpt2(torch, accumulate="wide")
        if rank == 0:
            line["matmul"] = mm

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


def bench_matmuls(dev, fmt, torch, n=8192, rank=0, world=1, dist=None):
    """The wide n^3 matmul (MX v4.9.2, shift 0), rows of A split over the
    ranks with B replicated: device time of the compute as the max over
    ranks, then the all-gather of the int16 row blocks timed apart; the
    gathered output's checksum on rank 0.  Chain 512^3 on rank 0."""
    from superfloat.python_b200 import _shard, workloads
    res = {}
    stream = torch.cuda.current_stream()
    A, B = workloads.wide_square(n, n, n, 0)
    cuts = _shard.row_cuts(n, world)
    lo, hi = cuts[rank], cuts[rank + 1]
    tA, tB = dev.upload(A[lo:hi]), dev.upload(B)
    del A, B
    out = torch.empty(hi - lo, n, dtype=torch.int16, device=dev.torch_device)
    cnt = torch.zeros(8, dtype=torch.int64, device=dev.torch_device)
    for _ in range(2):
        dev.run_device("matmul_wide", fmt, tA, tB, out=out, counts=cnt, shift=0)
    _shard.gather_rows(out, cuts, dist, world)               # the first collective of this size sets NCCL up
    e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
    reps = 3
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0.record(stream)
    for _ in range(reps):
        dev.run_device("matmul_wide", fmt, tA, tB, out=out, counts=cnt, shift=0)
    e1.record(stream)
    full = _shard.gather_rows(out, cuts, dist, world)
    e2.record(stream)
    torch.cuda.synchronize()
    ms = _shard.max_over_ranks(e0.elapsed_time(e1) / reps, "cuda", dist, world)
    gms = _shard.max_over_ranks(e1.elapsed_time(e2), "cuda", dist, world)
    cnt.zero_()
    dev.run_device("matmul_wide", fmt, tA, tB, out=out, counts=cnt, shift=0)
    _shard.sum_counts(cnt, dist, world)
    res[f"wide_{n}"] = {"ms": ms, "TOPS": 2 * n ** 3 / (ms / 1e3) / 1e12, "unit": "sf16 TOPS (2*M*N*K/s)",
                        "gather_ms": gms, "sharding": f"rows of A over {world} GPU(s), B replicated",
                        "overflow_outputs": int(cnt[0]), "underflow_outputs": int(cnt[1])}
    if rank == 0:
        import hashlib
        res[f"wide_{n}"]["codes_sha256"] = hashlib.sha256(full.cpu().numpy().astype("<i2").tobytes()).hexdigest()[:16]
    del tA, tB, out, full
    if rank != 0:
        return res
    # chain 512^3
    A, B = workloads.chain_square(512, 0)
    tA, tB = dev.upload(A), dev.upload(B)
    out = torch.empty(512, 512, dtype=torch.int16, device=dev.torch_device)
    for _ in range(3):
        dev.run_device("matmul", fmt, tA, tB, out=out, counts=cnt)
    torch.cuda.synchronize()
    reps = 20
    e0.record(stream)
    for _ in range(reps):
        dev.run_device("matmul", fmt, tA, tB, out=out, counts=cnt)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    res["chain_512"] = {"ms": ms, "TOPS": 2 * 512 ** 3 / (ms / 1e3) / 1e12, "unit": "sf16 TOPS (2*M*N*K/s)"}
    return res


def bench_sweep(torch, dist, rank, world, bits=16, cpu=False):
    """Every sf16 code pair through add, sub, mul and div (4 x 65535^2 =
    1.7e10 pairs), the a-rows split evenly over the ranks; each row folds
    into two 64-bit digests on the device.  Device time is the max over
    ranks; rank 0 gathers the row digests and checks their sha256 against
    the reference's (tests/golden/sweep.json) when that file is present."""
    from superfloat.python_b200 import _shard, sweep
    M = (1 << (bits - 1)) - 1
    n = 2 * M + 1
    cuts = _shard.row_cuts(n, world, -M)
    lo, hi = cuts[rank], cuts[rank + 1]
    for op in sweep.OPS:                                   # warm-up on a few rows
        sweep.run_device(op, bits, lo, min(hi, lo + 64))
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    outs = {op: sweep.run_device(op, bits, lo, hi) for op in sweep.OPS}
    e1.record()
    torch.cuda.synchronize()
    ms = _shard.max_over_ranks(e0.elapsed_time(e1), "cuda", dist, world)
    res = {"ms": ms, "value": len(sweep.OPS) * n * n / (ms / 1e3) / 1e9, "unit": "Gpairs/s (add, sub, mul, div)",
           "pairs": len(sweep.OPS) * n * n, "bits": bits, "sharding": f"a-rows over {world} GPU(s)"}
    golden = os.path.join(os.path.dirname(os.path.abspath(__file__)), "tests", "golden", "sweep.json")
    ref = json.load(open(golden))["widths"][str(bits)] if os.path.exists(golden) else None
    match = True
    for op, (rc, rf, cnt) in outs.items():
        rows = _shard.gather_rows(torch.stack([rc, rf], 1), cuts, dist, world)
        _shard.sum_counts(cnt, dist, world)
        if rank == 0:
            rows = rows.cpu().numpy()
            sha = sweep.digest(rows[:, 0].view(np.uint64), rows[:, 1].view(np.uint64))
            c = cnt.cpu().numpy()
            ok = ref is not None and sha == ref[op]["sha"] and all(
                int(c[i]) == ref[op][f"n_{e}"] for i, e in enumerate(("overflow", "underflow", "divide", "invalid")))
            match &= ok
            res[op] = {"sha256": sha[:16], "overflow": int(c[0]), "underflow": int(c[1]), "divide": int(c[2])}
    if rank == 0:
        res["digests_match_reference"] = bool(match) if ref is not None else None
    if cpu:
        from oracle import sfref
        rows = np.arange(-3, 3)
        b = np.arange(-M, M + 1)
        ka, kb = np.repeat(rows, n), np.tile(b, rows.size)
        t0 = time.perf_counter()
        for op in sweep.OPS:
            sfref.ew(op, bits, ka, kb)
        dt = time.perf_counter() - t0
        res["cpu_baseline"] = {"value": len(sweep.OPS) * ka.size / dt / 1e9, "unit": "Gpairs/s", "cores": 1,
                               "kind": "port", "sample": f"{rows.size} a-rows x {n} b, 4 ops, NumPy oracle"}
    return res


GPT2_SHAPES = ((4096, 768, 2304), (4096, 768, 768), (4096, 768, 3072), (4096, 3072, 768), (4096, 768, 50257))


def bench_chain_shapes(torch, reps=10):
    """sfb_linear_chain in proven mode (the converted layer's chain, bias-free,
    float32 output) on the GPT-2-small projection shapes at 8 x 512 tokens:
    activation codes in [-40, 40] and weight codes over the full sf16 range
    (seed 0), which the L1 bound proves clip-free.  Products per second and
    INT lane-instructions per second against SMs x 128 lanes x clock."""
    from superfloat.python_b200 import _lib
    _lib.load()
    g = torch.Generator(device="cuda").manual_seed(0)
    props = torch.cuda.get_device_properties(0)
    res = {}
    for (R, K, N) in GPT2_SHAPES:
        X = torch.randint(-40, 41, (R, K), dtype=torch.int16, device="cuda", generator=g)
        WT = torch.randint(-32767, 32768, (K, N), dtype=torch.int16, device="cuda", generator=g)
        s = torch.ones(N, dtype=torch.float64, device="cuda")
        y = torch.empty(R, N, dtype=torch.float32, device="cuda")
        cnt = torch.zeros(_lib.N_COUNTS, dtype=torch.int64, device="cuda")

        def f():
            _lib.linear_chain(16, X, WT, None, 1.0, s, True, y, None, None, None, cnt, R, N, K, K, N)
        for _ in range(3):
            f()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            f()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / reps
        res[f"{R}x{K}x{N}"] = {"ms": ms, "Tproducts_per_s": R * K * N / (ms / 1e3) / 1e12}
        del X, WT, y
    res["note"] = (f"{props.multi_processor_count} SMs; proven-mode kernel, two outputs per 32-bit word; "
                   "issue-bound on the INT pipes")
    return res


def bench_gpt2(torch, batch=8, seq=512, reps=3, accumulate="chain"):
    """sft.convert(dtype=sf16) GPT-2-small (12 layers, d_model 768, 12 heads,
    FFN 3072, vocab 50257; random init, seed 0) forward on batch x seq token
    ids, on the GPU; 49 SF layers (chain accumulation, headroom "bound")."""
    import warnings
    from transformers import GPT2Config, GPT2LMHeadModel
    import superfloat.python_b200.torch as sft
    torch.manual_seed(0)
    cfg = GPT2Config(n_layer=12, n_embd=768, n_head=12, n_inner=3072, vocab_size=50257, n_positions=1024)
    kw = {"accumulate": "wide", "attention": False} if accumulate == "wide" else {}
    model = sft.convert(GPT2LMHeadModel(cfg).eval(), dtype="sf16", **kw).cuda()
    ids = torch.randint(0, 50257, (batch, seq), generator=torch.Generator().manual_seed(0)).cuda()
    with torch.no_grad(), warnings.catch_warnings():
        warnings.simplefilter("ignore")
        model(ids)                                        # prepares the weights (cached per weight)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            model(ids)
        e1.record()
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    R = batch * seq
    products = R * (768 * 2304 + 768 * 768 + 768 * 3072 + 3072 * 768) * 12 + R * 768 * 50257
    st = sft.last_status(model)
    return {"ms_per_forward": ms, "tokens_per_s": R / (ms / 1e3), "sf_layers": len(st),
            "sf16_TOPS": 2 * products / (ms / 1e3) / 1e12, "saturated": sum(v.saturated or 0 for v in st.values()),
            "workload": f"GPT-2-small sft.convert(sf16, accumulate={accumulate!r}) forward, {batch} x {seq} tokens, "
                        "float parts on the GPU"}


if __name__ == "__main__":
    sys.exit(main())
