"""Benchmark: bit-exact sf16 elementwise ops on B200 (Gelem/s), with the wide
8192^3 and chain 512^3 matmuls, the converted GPT-2-small forward and the
exhaustive sf16 pair sweep measured beside it.

One step = the five status-reporting sf16 ops (add, sub, mul, fma, div) over
2^26-element inputs resident in HBM, each op's exact event counts reduced on
the device (and all-reduced over ranks when N > 1: the status exchange).
Each timed step is one CUDA graph replay (the step's counter reset and the
five launches, captured once per step buffer), so host launch overhead does
not gap the device.  ``value`` = elements processed by all ranks /
max-over-ranks device time.  ``e2e`` = the same ops on codes in pinned HOST
memory (int16, the device word's width): the host->device copies of every
step's inputs, the kernels, the device->host copies of the result codes and
the read of the status counts are all inside the timed region (chunked over
four streams so copies overlap kernels).  ``e2e_plugin_int64`` is the
reference's own plug-in contract, ``Device.run`` on int64 NumPy arrays
returning int64 codes and boolean masks, once per op.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

N > 1 is launched with torchrun; each rank runs its own 2^26 elements (weak
scaling, no data-path collective; only the status counts are all-reduced).
``--impl reference`` times the reference's host implementation of the same
ops (its own src/sf/_vectorized.py when the reference is installed, else the
oracle's NumPy restatement) on this host's cores, on rank 0 only.
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


def _profile_value(fname, key, col=1):
    """A number recorded from an ncu capture in profiles/<fname> (lines of
    '<key> <value> ...'), or None."""
    p = os.path.join(HERE, "profiles", fname)
    if not os.path.exists(p):
        return None
    for line in open(p):
        parts = line.split()
        if len(parts) > col and parts[0] == key:
            try:
                return float(parts[col])
            except ValueError:
                return None
    return None


def traffic_from_profiles(kernel_key):
    """DRAM bytes per launch recorded by ncu (profiles/ncu_traffic.txt)."""
    return _profile_value("ncu_traffic.txt", kernel_key)


def insts_from_profiles(kernel_key):
    """Warp instructions per launch recorded by ncu (profiles/ncu_inst.txt,
    smsp__inst_executed.sum of one launch of the same workload)."""
    return _profile_value("ncu_inst.txt", kernel_key)


def issue_roofline(torch, kernel, keys, ms, clocks):
    """Roofline of an integer kernel that is bound by instruction issue: the
    warp instructions its launches execute (ncu, profiles/ncu_inst.txt) over
    their CUDA-event time, against one warp instruction per scheduler per
    clock (SMs x 4 x the highest SM clock seen)."""
    insts = [insts_from_profiles(k) for k in keys]
    if any(v is None for v in insts):
        return None
    sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    mhz = (clocks or {}).get("sm_max_mhz") or 1965.0
    peak = sms * 4 * mhz * 1e6 / 1e12
    achieved = sum(insts) / (ms / 1e3) / 1e12
    return {"bound": "int", "achieved": achieved, "peak": peak, "unit": "T warp-instructions/s",
            "frac": achieved / peak, "traffic": None, "kernel": kernel,
            "peak_kind": f"{sms} SMs x 4 schedulers x 1 warp-instruction per clock at {mhz:.0f} MHz",
            "warp_instructions": sum(insts), "source": "ncu smsp__inst_executed.sum, profiles/ncu_inst.txt"}


def int8_peak(torch, n=8192, reps=10):
    """Dense int8 GEMM rate of this GPU in this run: torch._int_mm (cuBLASLt)
    on n^3, CUDA events, int8 TOPS (2 n^3 / t)."""
    g = torch.Generator(device="cuda").manual_seed(0)
    a = torch.randint(-128, 128, (n, n), dtype=torch.int8, device="cuda", generator=g)
    b = torch.randint(-128, 128, (n, n), dtype=torch.int8, device="cuda", generator=g)
    for _ in range(3):
        torch._int_mm(a, b)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record()
    for _ in range(reps):
        torch._int_mm(a, b)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    del a, b
    return 2 * n ** 3 / (ms / 1e3) / 1e12


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


def _cpu_pool_worker(n):
    return cpu_sample(n)


def reference_site():
    """The directory holding the reference package ``sf`` (an offline install
    under baseline/_ref, or SF_REFERENCE_SITE), or None."""
    for d in (os.environ.get("SF_REFERENCE_SITE"), os.path.join(HERE, "baseline", "_ref")):
        if d and os.path.isfile(os.path.join(d, "sf", "__init__.py")):
            return d
    return None


def _import_reference():
    site = reference_site()
    if site is None:
        return None
    if site not in sys.path:
        sys.path.insert(0, site)
    import tempfile
    os.environ.setdefault("SF_CACHE_DIR", os.path.join(tempfile.gettempdir(), "sf_bench_cache"))
    import sf
    return sf


def cpu_ops():
    """(fn(op, *codes), kind): the reference's own sf._vectorized ops
    (src/sf/_vectorized.py:94-131) when the reference is installed, else the
    oracle's NumPy restatement of them."""
    sf = _import_reference()
    if sf is not None:
        from sf import _vectorized as vec
        from sf._format import FORMATS
        f16 = FORMATS[16]
        return (lambda op, *xs: getattr(vec, op)(f16, *xs)), "reference"
    from oracle import sfref
    return (lambda op, *xs: sfref.ew(op, 16, *xs)), "port"


def cpu_sample(n_sample):
    """The five ops on n_sample elements of the same workload, single-threaded
    (the reference's own code when installed, else the oracle port)."""
    from superfloat.python_b200 import workloads
    fn, _ = cpu_ops()
    x, y, z, d = workloads.elementwise(n_sample, 0)
    args = {"add": (x, y), "sub": (x, y), "mul": (x, y), "fma": (x, y, z), "div": (x, d)}
    t0 = time.perf_counter()
    for op in OPS:
        fn(op, *args[op])
    return time.perf_counter() - t0


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


def cpu_matmul_baselines():
    """CPU baselines of the matmul, GPT-2 and sweep configs, each on a bounded
    sample of its workload, timed with the reference's own code when it is
    installed (else the oracle's restatement, or the reference's own C
    accumulator built into oracle/_ref).  Runs in a child process
    (``bench.py --cpu-baselines``): the reference and this package both
    register a TorchDynamo backend named ``superfloat``."""
    from superfloat.python_b200 import workloads
    sf = _import_reference()
    res = {}
    # chain 512^3: src/sf/_linalg.py:61-81, one core (NumPy's K-loop)
    A, B = workloads.chain_square(512, 0)
    if sf is not None:
        from sf import _linalg
        from sf._format import FORMATS
        f16 = FORMATS[16]
        t0 = time.perf_counter()
        _linalg.matmul_codes(f16, A, B)
        kind, what = "reference", "sf._linalg.matmul_codes"
    else:
        from oracle import sfref
        t0 = time.perf_counter()
        sfref.matmul_chain(16, A, B)
        kind, what = "port", "the oracle's NumPy restatement of _linalg.matmul_codes"
    dt = time.perf_counter() - t0
    res["chain_512"] = {"value": 2 * 512 ** 3 / dt / 1e12, "unit": "sf16 TOPS (2*M*N*K/s)", "cores": 1,
                        "kind": kind, "sample": f"{what} on the whole 512^3 workload, {dt:.2f} s"}
    # wide 8192^3: a 64-row slice (rows are independent), src/sf/_linalg.py:330-348 with
    # the compiled _fastmx loop (src/sf/_fastmx.py:176-198) on its own thread count
    rows = 64
    A, B = workloads.wide_square(8192, 8192, 8192, 0)
    A = np.ascontiguousarray(A[:rows])
    if sf is not None:
        from sf import _fastmx, _linalg
        threads = _fastmx._threads() if _fastmx.available() else 1
        t0 = time.perf_counter()
        _linalg.matmul_wide_codes(f16, A, B, 0)
        kind, what = "reference", f"sf._linalg.matmul_wide_codes (compiled _fastmx loop, {threads} threads)"
    else:
        from oracle import native
        threads = min(8, host_cores())
        t0 = time.perf_counter()
        if native.ref_available():
            native.ref_wide_acc(16, A, B, threads=threads)
            kind, what = "reference", f"the reference's own C accumulator (oracle/_ref), {threads} threads"
        else:
            native.wide_acc(16, A, B)
            kind, what = "port", "the oracle's C accumulator"
    dt = time.perf_counter() - t0
    res["wide_8192"] = {"value": 2 * rows * 8192 * 8192 / dt / 1e12, "unit": "sf16 TOPS (2*M*N*K/s)",
                        "cores": threads, "kind": kind,
                        "sample": f"{what}, rows 0..{rows - 1} of 8192 ({dt:.1f} s), extrapolated by rows"}
    del A, B
    # the converted GPT-2-small: the reference's own sft.convert forward on 1 x 16 tokens
    if sf is not None:
        import warnings
        import torch
        import sf.torch as sft
        from transformers import GPT2Config, GPT2LMHeadModel
        torch.manual_seed(0)
        cfg = GPT2Config(n_layer=12, n_embd=768, n_head=12, n_inner=3072, vocab_size=50257, n_positions=1024)
        model = sft.convert(GPT2LMHeadModel(cfg).eval(), dtype="sf16")
        tokens = 16
        ids = torch.randint(0, 50257, (1, tokens), generator=torch.Generator().manual_seed(0))
        torch.set_num_threads(1)
        with torch.no_grad(), warnings.catch_warnings():
            warnings.simplefilter("ignore")
            t0 = time.perf_counter()
            model(ids)
            dt = time.perf_counter() - t0
        res["gpt2_small_convert"] = {
            "value": tokens / dt, "unit": "tokens/s", "cores": 1, "kind": "reference",
            "sample": f"the reference's sft.convert(sf16) GPT-2-small forward on 1 x {tokens} tokens ({dt:.1f} s; "
                      "host path, one core), taken as linear in tokens (its cost per token at 64 tokens is about 0.8x "
                      "that at 8)"}
    else:
        res["gpt2_small_convert"] = None
    # the exhaustive sweep: a few a-rows through the four ops
    fn, kind = cpu_ops()
    M = 32767
    arows = np.arange(-128, 128)
    b = np.arange(-M, M + 1)
    ka, kb = np.repeat(arows, b.size), np.tile(b, arows.size)
    t0 = time.perf_counter()
    for op in ("add", "sub", "mul", "div"):
        fn(op, ka, kb)
    dt = time.perf_counter() - t0
    res["sweep"] = {"value": 4 * ka.size / dt / 1e9, "unit": "Gpairs/s", "cores": 1, "kind": kind,
                    "sample": f"{arows.size} a-rows x {b.size} b, add/sub/mul/div ({dt:.2f} s)"}
    return res


def run_cpu_baselines_child():
    """``bench.py --cpu-baselines`` in a child process; None when it fails."""
    try:
        p = subprocess.run([sys.executable, os.path.abspath(__file__), "--cpu-baselines"], capture_output=True,
                           text=True, timeout=600, cwd=HERE)
        return json.loads(p.stdout.strip().splitlines()[-1]) if p.returncode == 0 else None
    except (subprocess.TimeoutExpired, ValueError, IndexError):
        return None


def elementwise_config(n, world):
    """The ``config`` of the headline line; the reference arm prints the same dict."""
    return {"workload": "sf16 elementwise add/sub/mul/fma/div with exact status counts, "
                        f"{n} elements per op per rank (seeded 2^26 generator)",
            "elements_per_op_per_rank": n, "l2": "inputs larger than L2 (3 x 128 MiB per op)",
            "parallelism": f"element-range shards x{world}, status all-reduce"}


def run_reference(args, rank, world):
    if rank != 0:
        return 0
    import multiprocessing as mp
    cores = host_cores()
    n_sample = 1 << 22                             # per process per step
    _, kind = cpu_ops()
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
    what = ("the reference's own sf._vectorized ops" if kind == "reference"
            else "the oracle's NumPy restatement of sf._vectorized")
    line = {"metric": METRIC, "value": v, "unit": "Gelem/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int64", "data": "synthetic",
            "config": elementwise_config(args.elements, world),
            "impl": "reference",
            "cpu_baseline": {"value": v, "unit": "Gelem/s", "cores": cores, "kind": kind,
                             "sample": f"{what}: {n_sample} elements x 5 ops per process and step, {cores} spawn "
                                       f"processes (a bounded sample of the {args.elements}-element workload)"},
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
    ap.add_argument("--cpu-baselines", action="store_true",
                    help="print the CPU baselines of the matmul / GPT-2 / sweep configs (a child process)")
    ap.add_argument("--gpt2-only", type=int, default=0, metavar="TOKENS",
                    help="time only the converted GPT-2-small forward on 8 x TOKENS ids")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    rank, world, local = _env_int("RANK", 0), _env_int("WORLD_SIZE", 1), _env_int("LOCAL_RANK", 0)
    if args.impl == "reference":
        return run_reference(args, rank, world)
    if args.cpu_baselines:
        print(json.dumps(cpu_matmul_baselines()), flush=True)
        return 0

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

    def step(evs=None, buf=None, st=None, only=None):
        buf.zero_()
        # the timed op last: its closing event then falls on the step boundary
        order = [op for op in OPS if op != only] + ([only] if only else [])
        for op in order:
            i = OPS.index(op)
            timed = evs is not None and (only is None or op == only)
            if timed:
                evs[op][0].record(st or stream)
            dev.run_device(op, fmt, *targs[op], out=outs[op], counts=buf[i], stream=st)
            if timed:
                evs[op][1].record(st or stream)

    def drain():
        if world > 1:
            dist.all_reduce(allbufs)

    # warm-up: eager steps with every op's launch bracketed by events (each
    # op's kernel time, and which op's launch is longest)
    warm_evs = []
    for i in range(max(1, args.warmup)):
        evs = {op: (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for op in OPS}
        step(evs, bufs[i])
        warm_evs.append(evs)
    drain()
    torch.cuda.synchronize()
    warm = {op: [evs[op][0].elapsed_time(evs[op][1]) for evs in warm_evs] for op in OPS}
    # the first step carries the first launches' set-up: left out when there are more
    warm_ms = {op: statistics.median(v[1:] if len(v) > 1 else v) for op, v in warm.items()}
    dom = max(OPS, key=warm_ms.get)

    # one CUDA graph per timed step (the step's counter buffer zeroed and the
    # five launches), so the host's launch overhead stays out of the device's
    # way.  The longest op runs last in every step; in every fourth step its
    # launch is bracketed by events inside the graph for its kernel time over
    # the timed region (an event node between two launches holds the next one
    # back by a few microseconds: around every launch of every step they cost
    # ~10% of the step, around the one op of every step ~2.5%); the other
    # ops' kernel times come from the warm-up.
    graphs, dom_evs = [], []
    side = torch.cuda.Stream(device=dev.torch_device)
    side.wait_stream(stream)
    with torch.cuda.stream(side):                       # a warm-up off the capturing stream
        step(buf=bufs[0], st=side)
    torch.cuda.synchronize()
    for i in range(args.steps):
        g = torch.cuda.CUDAGraph()
        sampled = i % 4 == 0
        evs = {dom: (torch.cuda.Event(enable_timing=True, external=True),
                     torch.cuda.Event(enable_timing=True, external=True))} if sampled else None
        with torch.cuda.graph(g):
            step(evs, bufs[i], st=torch.cuda.current_stream(), only=dom)
        graphs.append(g)
        if sampled:
            dom_evs.append(evs[dom])
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t_start.record(stream)
    for i in range(args.steps):
        graphs[i].replay()
    drain()                                  # the status reduction is part of the timed work
    t_end.record(stream)
    counts = bufs[args.steps - 1]
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = sampler.stop() if sampler else None
    ms_total = t_start.elapsed_time(t_end)
    dom_ms = statistics.mean(e0.elapsed_time(e1) for e0, e1 in dom_evs)
    del graphs
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
    achieved = BYTES_PER_ELEM[dom] * n / (dom_ms / 1e3) / 1e9
    traffic = traffic_from_profiles(f"ew_{dom}_{n}")
    roofline = {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                "traffic": traffic, "kernel": f"ew_kernel<{dom}>", "peak_kind": peak_kind,
                "launch_ms": dom_ms,
                "launch_ms_source": f"CUDA events around this op's launch inside the graphs of timed steps "
                                    f"0, 4, 8, ... ({len(dom_evs)} of {args.steps})",
                "per_op_GBps_warmup": {op: BYTES_PER_ELEM[op] * n / (warm_ms[op] / 1e3) / 1e9 for op in OPS},
                "per_op_source": "median of the warm-up steps after the first, events around every launch",
                "algorithmic_bytes_per_launch": BYTES_PER_ELEM[dom] * n}

    line = {"metric": METRIC, "value": value, "unit": "Gelem/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int16", "data": "synthetic",
            "config": elementwise_config(n, world),
            "gpu_launches": len(OPS) * args.steps, "roofline": roofline,
            "status_counts_last_step": {op: {"overflow": int(cnt[i][0]), "underflow": int(cnt[i][1]),
                                             "divide": int(cnt[i][2])} for i, op in enumerate(OPS)}}
    if clocks:
        line["clocks"] = clocks

    # end to end: codes in pinned host memory, copies inside the timed region
    if not args.no_e2e:
        from superfloat.python_b200._hostpath import HostPipeline, MultiOpPipeline
        hx = {}
        for name, v in (("x", x), ("y", y), ("z", z), ("d", d)):
            t = torch.empty(n, dtype=torch.int16, pin_memory=True)
            t.copy_(torch.from_numpy(v))
            hx[name] = t
        hargs = {"add": ("x", "y"), "sub": ("x", "y"), "mul": ("x", "y"), "fma": ("x", "y", "z"), "div": ("x", "d")}
        hout = {op: torch.empty(n, dtype=torch.int16, pin_memory=True) for op in OPS}
        e2e_steps = max(1, min(5, args.steps))

        def timed_host(fn):
            fn()                                         # warm-up of the host path
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            t0 = time.perf_counter()
            for _ in range(e2e_steps):
                fn()                                     # returns after the counts are read
            dt = torch.tensor([time.perf_counter() - t0], dtype=torch.float64, device=dev.torch_device)
            if world > 1:
                dist.all_reduce(dt, op=dist.ReduceOp.MAX)
            return float(dt.item())

        # the step's four operands copied in once per chunk, the five ops, the five results copied out;
        # each step's counts are read while the next step's copies run
        multi = MultiOpPipeline(dev, ("x", "y", "z", "d"), [(op, hargs[op]) for op in OPS])

        def e2e_steps_run():
            pending = None
            for _ in range(e2e_steps):
                nxt = multi.run_async(fmt, hx, [hout[op] for op in OPS])
                if pending is not None:
                    pending.result()
                pending = nxt
            pending.result()

        multi.run(fmt, hx, [hout[op] for op in OPS])            # warm-up of the host path
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        t0 = time.perf_counter()
        e2e_steps_run()
        dt = torch.tensor([time.perf_counter() - t0], dtype=torch.float64, device=dev.torch_device)
        if world > 1:
            dist.all_reduce(dt, op=dist.ReduceOp.MAX)
        dt = float(dt.item())
        h2d = 4 * 2 * n
        d2h = len(OPS) * (2 * n + 8 * _lib.N_COUNTS)
        line["e2e"] = {"value": len(OPS) * n * world * e2e_steps / dt / 1e9, "unit": "Gelem/s",
                       "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                       "copy_GBps_per_rank": {"h2d": h2d * e2e_steps / dt / 1e9, "d2h": d2h * e2e_steps / dt / 1e9},
                       "copy_GBps_all_ranks": (h2d + d2h) * e2e_steps * world / dt / 1e9,
                       "path": "int16 codes in pinned host memory -> MultiOpPipeline: per 8M-code chunk the four "
                               "operands copied in once, add/sub/mul/fma/div on the device, the five results "
                               "copied out, four streams; every step's status counts read back while the next "
                               "step's copies run"}
        # each op with its own copies of its operands (HostPipeline, one call per op)
        pipe = HostPipeline(dev)
        dt1 = timed_host(lambda: [pipe.run(op, fmt, *(hx[a] for a in hargs[op]), out=hout[op]) for op in OPS])
        line["e2e_inputs_per_op"] = {"value": len(OPS) * n * world * e2e_steps / dt1 / 1e9, "unit": "Gelem/s",
                                     "h2d_bytes_per_step": sum(2 * n * len(hargs[op]) for op in OPS),
                                     "path": "HostPipeline, one call per op: each op copies its own operands in"}
        # the reference's Device.run contract: int64 NumPy codes in, int64 codes + boolean masks out,
        # timed on every rank (each rank its own 2^26 elements) with its share of the host's cores
        xs = {"add": (x, y), "sub": (x, y), "mul": (x, y), "fma": (x, y, z), "div": (x, d)}
        threads = torch.get_num_threads()
        torch.set_num_threads(max(1, host_cores() // world))
        dev.run("add", fmt, x, y)                        # warm-up: allocates the staging buffers
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        t0 = time.perf_counter()
        for op in OPS:
            dev.run(op, fmt, *xs[op])
        dtp = torch.tensor([time.perf_counter() - t0], dtype=torch.float64, device=dev.torch_device)
        if world > 1:
            dist.all_reduce(dtp, op=dist.ReduceOp.MAX)
        torch.set_num_threads(threads)
        line["e2e_plugin_int64"] = {"value": len(OPS) * n * world / float(dtp.item()) / 1e9, "unit": "Gelem/s",
                                    "threads_per_rank": max(1, host_cores() // world),
                                    "path": "B200Device.run, the reference's Device contract: int64 NumPy codes "
                                            "in, int64 codes and boolean event masks out (host narrowing / "
                                            "widening included), all ranks, max-over-ranks wall time"}

    # CPU baseline on rank 0, N = 1
    if rank == 0 and world == 1 and not args.no_cpu:
        n_sample = 1 << 22
        cpu_sample(1 << 16)
        reps = 3
        ts = [cpu_sample(n_sample) for _ in range(reps)]
        v = len(OPS) * n_sample / statistics.median(ts) / 1e9
        _, kind = cpu_ops()
        what = "the reference's own sf._vectorized" if kind == "reference" else "the oracle's NumPy restatement"
        line["cpu_baseline"] = {"value": v, "unit": "Gelem/s", "cores": 1, "kind": kind,
                                "sample": f"{what}: {n_sample} elements x 5 ops, one core, median of {reps}"}

    # CPU baselines of the other configs (rank 0, N = 1), in a child process
    cpu_mm = run_cpu_baselines_child() if rank == 0 and world == 1 and not args.no_cpu else None

    # the exhaustive pair sweep beside it, row-sharded over all ranks: not part of `value`
    if not args.no_sweep:
        sw = bench_sweep(torch, dist, rank, world)
        if rank == 0:
            if cpu_mm:
                sw["cpu_baseline"] = cpu_mm.get("sweep")
            rl = issue_roofline(torch, "sweep_kernel<op, 16> (add, sub, mul, div)",
                                [f"sweep_{op}_16" for op in ("add", "sub", "mul", "div")], sw["ms"] * world, clocks)
            sw["roofline"] = rl                # per GPU: 1 / world of the instructions in sw["ms"]
            line["sweep"] = sw

    # the matmuls beside it: not part of `value`.  The wide one row-sharded over all
    # ranks; chain 512^3 and the converted GPT-2 forward on rank 0 at N = 1.
    if not args.no_matmul:
        mm = bench_matmuls(dev, fmt, torch, rank=rank, world=world, dist=dist)
        if rank == 0 and world == 1:
            mm["chain_gpt2_projections"] = bench_chain_shapes(torch)
            mm["gpt2_small_convert"] = bench_gpt2(torch)
            mm["gpt2_small_convert_wide"] = bench_gpt2(torch, accumulate="wide")
        if rank == 0 and cpu_mm:
            for key in ("chain_512", "wide_8192", "gpt2_small_convert"):
                if key in mm:
                    mm[key]["cpu_baseline"] = cpu_mm.get(key)
        if rank == 0:
            add_matmul_rooflines(torch, mm, clocks, world)
            line["matmul"] = mm

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


GPT2_LAYERS = ((768, 2304), (768, 768), (768, 3072), (3072, 768))       # (K, N) of one block's four layers


def add_matmul_rooflines(torch, mm, clocks, world):
    """Roofline objects for the matmul entries: the wide call against the
    limb-adjusted int8 rate (11 int8 passes per sf16 product, int8 peak
    measured here with torch._int_mm), the chain kernels against the issue
    rate (their ncu instruction counts)."""
    peak = None
    for key, e in mm.items():
        if key.startswith("wide_") and e:
            n = int(key.split("_")[1])
            peak = peak or int8_peak(torch)
            achieved = 11 * 2 * (n // world) * n * n / (e["ms"] / 1e3) / 1e12
            e["roofline"] = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "int8 TOPS",
                             "frac": achieved / peak, "traffic": None,
                             "kernel": "the wide call (prep x2, tc_gemm, wide_rem, finish)",
                             "peak_kind": "measured in this run: torch._int_mm (cuBLASLt) int8 8192^3",
                             "note": "11 tcgen05 int8 passes per sf16 product; frac = sf16 rate / (int8 rate / 11)"}
    if "chain_512" in mm:
        mm["chain_512"]["roofline"] = issue_roofline(torch, "chain2_kernel (general mode, 512^3)", ["chain2_512"],
                                                     mm["chain_512"]["ms"], clocks)
    for shape, e in mm.get("chain_gpt2_projections", {}).items():
        if isinstance(e, dict):
            e["roofline"] = issue_roofline(torch, f"chain_pk_kernel ({shape})", [f"chain_pk_{shape}"], e["ms"],
                                           clocks)
    g = mm.get("gpt2_small_convert")
    if g:
        keys = [f"chain_pk_4096x{k}x{n}" for k, n in GPT2_LAYERS] * 12 + ["chain_pk_4096x768x50257"]
        rl = issue_roofline(torch, "chain_pk_kernel, the 49 SF layers of one forward", keys, g["ms_per_forward"],
                            clocks)
        if rl:
            rl["note"] = "the chain kernels' instructions over the whole forward's time (float parts included)"
        g["roofline"] = rl


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
    del tA, out
    res[f"wide_{n}_prepared_b"] = bench_wide_prepared(torch, tB, n, rank, world, dist,
                                                      res[f"wide_{n}"].get("codes_sha256"))
    del tB, full
    if rank != 0:
        return res
    # chain 512^3
    A, B = workloads.chain_square(512, 0)
    tA, tB = dev.upload(A), dev.upload(B)
    out = torch.empty(512, 512, dtype=torch.int16, device=dev.torch_device)
    side = torch.cuda.Stream(device=dev.torch_device)
    side.wait_stream(stream)
    with torch.cuda.stream(side):
        for _ in range(3):
            dev.run_device("matmul", fmt, tA, tB, out=out, counts=cnt, stream=side)
    torch.cuda.synchronize()
    # the calls back to back as one CUDA graph (a serving loop's form), so the
    # host's per-call launch path does not gap the 70 us kernels
    reps = 20
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(reps):
            dev.run_device("matmul", fmt, tA, tB, out=out, counts=cnt, stream=torch.cuda.current_stream())
    g.replay()
    torch.cuda.synchronize()
    e0.record(stream)
    g.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    del g
    ms = e0.elapsed_time(e1) / reps
    res["chain_512"] = {"ms": ms, "TOPS": 2 * 512 ** 3 / (ms / 1e3) / 1e12, "unit": "sf16 TOPS (2*M*N*K/s)",
                        "timing": f"{reps} calls captured as one CUDA graph, CUDA events around a replay"}
    return res


def bench_wide_prepared(torch, tB, n, rank, world, dist, want_sha, reps=4):
    """The wide n^3 matmul as a serving loop would run it: B prepared once
    (a replicated, static operand: the reference's prepared weight), calls
    back to back, each call's output rows all-gathered on NCCL's stream while
    the next call computes (two output buffers).  Rows are split evenly over
    the ranks.  ``ms`` = time per call over ``reps`` calls, the last call's
    gather included: CUDA events, max over ranks."""
    import hashlib
    from superfloat.python_b200 import _lib, _shard, workloads
    if n % world:
        return None
    P = n // world
    dev = tB.device
    A, _ = workloads.wide_square(n, n, n, 0)
    tA = torch.from_numpy(A[rank * P:(rank + 1) * P]).to(torch.int16).to(dev)
    del A
    prep = torch.empty(_lib.wide_prepared_b_bytes(16, "v4.9.2", n, n), dtype=torch.uint8, device=dev)
    _lib.wide_prepare_b(16, "v4.9.2", tB, n, n, n, prep)
    ws = torch.empty(_lib.wide_workspace(16, "v4.9.2", 1, P, n, n), dtype=torch.uint8, device=dev)
    loc = torch.empty(2, P, n, dtype=torch.int16, device=dev)
    full = torch.empty(2, n, n, dtype=torch.int16, device=dev)
    cnt = torch.zeros(8, dtype=torch.int64, device=dev)
    stream = torch.cuda.current_stream()

    def calls(k):
        works = []
        for i in range(k):
            b = i & 1
            if len(works) >= 2 and works[-2] is not None:
                works[-2].wait()                  # this buffer's previous gather has finished
            _lib.matmul_wide_prepared(16, "v4.9.2", tA, tB, prep, None, 0, loc[b], None, cnt, 1, P, n, n, n, n,
                                      0, P * n, 0, 0, 0, ws)
            works.append(_shard.gather_piece(full[b], loc[b], 0, dist, world, async_op=True))
        for w in works[-2:]:
            if w is not None:
                w.wait()

    calls(2)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0.record(stream)
    calls(reps)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = _shard.max_over_ranks(e0.elapsed_time(e1) / reps, "cuda", dist, world)
    _lib.check_counts(cnt.cpu().numpy())
    out = {"ms": ms, "TOPS": 2 * n ** 3 / (ms / 1e3) / 1e12, "unit": "sf16 TOPS (2*M*N*K/s)",
           "includes": f"{reps} calls back to back, each with its output rows all-gathered on every rank "
                       "beside the next call's compute (the last gather included); B prepared once, outside",
           "sharding": f"rows of A over {world} GPU(s), {P} rows each, B replicated"}
    if rank == 0:
        sha = hashlib.sha256(full[(reps - 1) & 1].cpu().numpy().astype("<i2").tobytes()).hexdigest()[:16]
        out["codes_sha256"] = sha
        out["codes_equal_unprepared"] = sha == want_sha if want_sha else None
    del tA, prep, ws, loc, full
    return out


def bench_sweep(torch, dist, rank, world, bits=16):
    """Every sf16 code pair through add, sub, mul and div (4 x 65535^2 =
    1.7e10 pairs), the a-rows split evenly over the ranks; each row folds
    into one 32-bit digest on the device.  Device time is the max over
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
    for op, (rd, cnt) in outs.items():
        rows = _shard.gather_rows(rd, cuts, dist, world)
        _shard.sum_counts(cnt, dist, world)
        if rank == 0:
            sha = sweep.digest(sweep.host_rows(rows))
            c = cnt.cpu().numpy()
            ok = ref is not None and sha == ref[op]["sha"] and all(
                int(c[i]) == ref[op][f"n_{e}"] for i, e in enumerate(("overflow", "underflow", "divide", "invalid")))
            match &= ok
            res[op] = {"sha256": sha[:16], "overflow": int(c[0]), "underflow": int(c[1]), "divide": int(c[2])}
    if rank == 0:
        res["digests_match_reference"] = bool(match) if ref is not None else None
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


def bench_gpt2(torch, batch=8, seq=512, reps=5, accumulate="chain"):
    """sft.convert(dtype=sf16) GPT-2-small (12 layers, d_model 768, 12 heads,
    FFN 3072, vocab 50257; random init, seed 0) forward on batch x seq token
    ids, on the GPU, through torch.compile(backend="superfloat") (the timed
    forward; the first compiled call, which traces, is not timed); 49 SF
    layers (chain accumulation, headroom "bound").  The eager forward is
    timed beside it, and the compiled logits must equal the eager ones.
    ``ms_per_forward`` is the median of ``reps`` timed forwards (every one
    is listed: a forward now and then takes up to twice as long on the host
    side, eager and compiled alike)."""
    import warnings
    from transformers import GPT2Config, GPT2LMHeadModel
    import superfloat.python_b200.torch as sft
    torch.manual_seed(0)
    cfg = GPT2Config(n_layer=12, n_embd=768, n_head=12, n_inner=3072, vocab_size=50257, n_positions=1024)
    kw = {"accumulate": "wide", "attention": False} if accumulate == "wide" else {}
    model = sft.convert(GPT2LMHeadModel(cfg).eval(), dtype="sf16", **kw).cuda()
    ids = torch.randint(0, 50257, (batch, seq), generator=torch.Generator().manual_seed(0)).cuda()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    per_rep = {}

    def timed(fn, key):
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(reps + 1)]
        torch.cuda.synchronize()
        evs[0].record()
        for i in range(reps):
            out = fn(ids)
            evs[i + 1].record()
        torch.cuda.synchronize()
        per_rep[key] = [round(evs[i].elapsed_time(evs[i + 1]), 2) for i in range(reps)]
        return statistics.median(per_rep[key]), out

    torch._dynamo.reset()
    with torch.no_grad(), warnings.catch_warnings():
        warnings.simplefilter("ignore")
        eager_logits = model(ids).logits                  # prepares the weights (cached per weight)
        model(ids)
        eager_ms, _ = timed(model, "eager")
        n_rep = len(sft.compile_reports())
        compiled = torch.compile(model, backend="superfloat")
        compiled(ids)                                     # traces and compiles
        compiled(ids)
        ms, out = timed(compiled, "compiled")
    reps_new = sft.compile_reports()[n_rep:]
    same = bool(torch.equal(out.logits, eager_logits))
    torch._dynamo.reset()
    R = batch * seq
    products = R * (768 * 2304 + 768 * 768 + 768 * 3072 + 3072 * 768) * 12 + R * 768 * 50257
    st = sft.last_status(model)
    return {"ms_per_forward": ms, "tokens_per_s": R / (ms / 1e3), "sf_layers": len(st),
            "sf16_TOPS": 2 * products / (ms / 1e3) / 1e12, "saturated": sum(v.saturated or 0 for v in st.values()),
            "eager_ms_per_forward": eager_ms, "compiled_equals_eager": same, "ms_per_rep": per_rep,
            "sf_op_nodes_on_device": sum(len(r.on_device) for r in reps_new),
            "sf_op_nodes_host_emulated": sum(len(r.host_emulated) for r in reps_new), "graphs": len(reps_new),
            "workload": f"GPT-2-small sft.convert(sf16, accumulate={accumulate!r}) forward through "
                        f"torch.compile(backend='superfloat'), {batch} x {seq} tokens, float parts on the GPU"}


if __name__ == "__main__":
    sys.exit(main())
