"""Benchmark of the Loom hot path on B200: effective HBM GB/s per generated
kernel at N = 2^28 fp32 per GPU, 1..8 GPUs (one process per GPU).

One step = one call of each of the seven suite entries (saxpy, relu, dot,
l2_norm_sq, max_value, affine_relu, pipeline_sum), each over N = 2^28
float32 elements per GPU (weak scaling: every GPU owns its own N-element
shards; maps need no communication, each reduction adds one scalar NCCL
collective).  `value` is the whole-job effective bandwidth: algorithmic bytes
(every input read once, every tensor output written once) of all ranks per
step / the step time (max over ranks, CUDA events, inputs resident in HBM).
Every input is 1 GiB, far larger than the 126 MB L2, so no flush is needed
between launches.

`e2e` is the same metric through the reference-facing C-ABI entry (the
synchronous `loom_kernels_<entry>` call) with pinned HOST buffers: every
step copies each entry's inputs host->device, calls the entry, and copies the
result back.

`reference_kernels` (1 GPU) times, on the same inputs and GPU, the CUDA that
the reference's backend generates for the same seven entries, restated by
hand for two of its optimisation profiles (baseline/loom_reference_style.cu):
"none" (no passes: unfused, scalar, tree reductions with a host combine loop)
and "cuda" (its full CUDA set: fused, float4 maps, atomic-output sums).

`--impl reference` times the reference's CPU semantics for the same workload
on this machine's host cores (the C oracle: the reference has no CPU
implementation of this path and its OCaml compiler cannot be built here):
each step is one GPU's workload, the seven entries at the same N, and the
line carries the same `config`.

After the timed region the line's `check` holds the results of the last
step against independent references (sums against fp64 sums all-reduced
over the ranks, max exactly, every rank's reductions bit-identical, a window
of every map bit for bit); a failed check exits non-zero.  Across GPUs
`exchange_wait` reports how long each reduction's peer exchange waited.

Other modes: `--strong` (fixed global sizes sharded over the ranks),
`--single ENTRY` (one entry, for profiler captures), `--pipeline-sweep`,
`--config-sweep`, `--workload-sweep`.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "Effective HBM GB/s & % of B200 peak per kernel, N=2^28 fp32, at 1/2/4/8 GPUs"
ENTRIES = ["saxpy", "relu", "dot", "l2_norm_sq", "max_value", "affine_relu", "pipeline_sum"]
# tensor params per entry, their data source, and algorithmic bytes per element
TENSORS = {
    "saxpy": ("u0", "u1"), "relu": ("nrm",), "dot": ("u0", "u1"), "l2_norm_sq": ("outl",),
    "max_value": ("outl",), "affine_relu": ("u0", "u1"), "pipeline_sum": ("u0", "u1", "u2"),
}
PARAM_NAMES = {
    "saxpy": ("x", "y"), "relu": ("x",), "dot": ("x", "y"), "l2_norm_sq": ("x",),
    "max_value": ("x",), "affine_relu": ("x", "y"), "pipeline_sum": ("x", "y", "w"),
}
SCALARS = {"saxpy": {"a": 2.5}, "affine_relu": {"a": 0.75}, "pipeline_sum": {"a": 0.75}}
MAP_ENTRIES = {"saxpy", "relu", "affine_relu"}
FALLBACK_HBM_GBS = 6650.0
_JSON_OUT = None


def protect_stdout() -> None:
    """Send everything written to fd 1 (NCCL prints its version there on
    rank 0) to stderr, keeping a private copy of stdout for the one JSON
    line."""
    global _JSON_OUT
    if _JSON_OUT is None:
        sys.stdout.flush()
        _JSON_OUT = os.fdopen(os.dup(1), "w")
        os.dup2(2, 1)


def emit(obj) -> None:
    out = _JSON_OUT or sys.stdout
    out.write(json.dumps(obj) + "\n")
    out.flush()


def bytes_per_elem(entry: str) -> int:
    return 4 * (len(TENSORS[entry]) + (1 if entry in MAP_ENTRIES else 0))


def read_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as fh:
            return float(json.load(fh)["hbm_gbs"]), "of measured"
    except (OSError, ValueError, KeyError):
        return FALLBACK_HBM_GBS, "of fallback"


def read_traffic():
    """Per-launch DRAM bytes of each kernel from the committed ncu summary."""
    path = os.path.join(ROOT, "profiles", "dram_traffic.json")
    try:
        with open(path) as fh:
            return json.load(fh)
    except (OSError, ValueError):
        return {}


class ClockSampler:
    """nvidia-smi samples of one GPU every 100 ms, time-stamped on arrival by
    a reader thread; only the samples inside [mark_start, mark_end] count."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.gpu_id = gpu_id
        self.proc = None
        self.lines = []
        self.t0 = self.t1 = None
        self.thread = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.time(), line))

    def start(self):
        import threading
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", self.gpu_id],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def wait_first(self, timeout: float = 10.0):
        end = time.time() + timeout
        while self.proc is not None and not self.lines and time.time() < end:
            time.sleep(0.05)

    def mark_start(self):
        self.t0 = time.time()

    def mark_end(self):
        self.t1 = time.time()

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.15)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=10)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=5)
        t0 = self.t0 if self.t0 is not None else 0.0
        t1 = self.t1 if self.t1 is not None else float("inf")
        rows = [line for t, line in self.lines if t0 <= t <= t1 + 0.1]
        if not rows and self.lines:       # region shorter than one period: nearest sample
            mid = (t0 + t1) / 2 if self.t1 is not None else t0
            rows = [min(self.lines, key=lambda tl: abs(tl[0] - mid))[1]]
        sm, mx, power, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in rows:
            parts = [q.strip() for q in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
                power.append(float(parts[3]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None,
                "power_w_max": max(power) if power else None,
                "samples": len(sm), "reasons": sorted(reasons)}


def setup_dist(args):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(world, value: float) -> float:
    if world == 1:
        return value
    import torch
    import torch.distributed as dist
    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_obj(world, obj):
    if world == 1:
        return [obj]
    import torch.distributed as dist
    out = [None] * world
    dist.all_gather_object(out, obj)
    return out


def make_inputs(n: int, rank: int):
    """Seeded device inputs of the suite (uniform x3, normal, normal+outliers)."""
    import torch
    from loom_b200.workloads import BASE_SEED, INPUT_SEED_STRIDE
    gen = torch.Generator(device="cuda")
    data = {}
    for k, name in enumerate(("u0", "u1", "u2")):
        gen.manual_seed(BASE_SEED + k * INPUT_SEED_STRIDE + rank * 7919)
        t = torch.rand(n, device="cuda", dtype=torch.float32, generator=gen)
        data[name] = t.mul_(2.0).sub_(1.0)
    gen.manual_seed(BASE_SEED + 3 * INPUT_SEED_STRIDE + rank * 7919)
    data["nrm"] = torch.randn(n, device="cuda", dtype=torch.float32, generator=gen)
    gen.manual_seed(BASE_SEED + 4 * INPUT_SEED_STRIDE + rank * 7919)
    outl = torch.randn(n, device="cuda", dtype=torch.float32, generator=gen)
    mask = torch.rand(n, device="cuda", generator=gen) < 0.01   # seeded 1% outliers
    outl[mask] *= 1e3
    data["outl"] = outl
    del mask
    return data


def suite_config(world: int, n_log2: int) -> dict:
    """The workload both arms report: the seven suite entries over N = 2^n_log2
    fp32 elements per GPU."""
    n = 1 << n_log2
    return {
        "workload": ("b200_suite step: saxpy, relu, dot, l2_norm_sq, max_value, "
                     "affine_relu, pipeline_sum, each over N=2^%d fp32 per GPU" % n_log2),
        "n_per_gpu": n,
        "global_n": n * world,
        "entries": ENTRIES,
        "l2": "no flush: every input is %d MiB per GPU (> 126 MB L2)" % (4 * n >> 20),
        "parallelism": f"shard{world} (maps: no communication; reductions: one "
                       "scalar exchange per call)",
    }


def cpu_suite_inputs(n: int):
    """loom_b200.workloads.entry_inputs(e, n) for every suite entry, with the
    arrays shared between entries that draw the same distribution from the
    same seed (the uniform x, y, w of saxpy, dot, affine_relu and
    pipeline_sum; the outlier vector of l2_norm_sq and max_value): five
    arrays of n floats instead of twelve."""
    from loom_b200 import workloads
    cache, out = {}, {}
    for e in ENTRIES:
        tensors, scalars, dist = workloads.ENTRY_SPECS[e]
        inp = {}
        for k, name in enumerate(tensors):
            key = (dist, k)
            if key not in cache:
                cache[key] = workloads.generate(
                    dist, n, workloads.BASE_SEED + k * workloads.INPUT_SEED_STRIDE)
            inp[name] = cache[key]
        inp.update(dict(scalars))
        out[e] = inp
    return out


def launches_per_call(entry: str, world: int, n: int, peer: bool = True) -> int:
    """Kernels of this library one call launches on n elements per GPU: one
    for a map; for a reduction one when its grid is a single CTA or one
    cluster (at most 8 tiles of 256 threads x 4 float4 for one input, x 2
    float4 for more), else the reduction kernel and its finalize.  Across
    GPUs through peer memory the exchange runs inside the finalize CTA, or
    as its own kernel after a one-CTA or one-cluster grid, so a reduction is
    always two kernels; through NCCL the sums add the rank fold (NCCL's own
    kernels are not counted)."""
    if entry in MAP_ENTRIES:
        return 1
    per_tile = 256 * 4 * (4 if len(TENSORS[entry]) == 1 else 2)
    local = 1 if -(-n // per_tile) <= 8 else 2
    if world == 1:
        return local
    if peer:
        return 2
    return local + (1 if entry != "max_value" else 0)


def fmaf_f32(a: float, x, y):
    """Correctly rounded float32 fma(a, x, y) of float32 numpy arrays,
    computed exactly on the host: a*x is exact in float64 (two 24-bit
    significands), s = fl64(a*x + y) comes with its exact error e (Knuth's
    TwoSum), and s rounds to float32 correctly unless it lies exactly
    halfway between two float32 values, where the sign of e decides."""
    import numpy as np
    p = np.float64(np.float32(a)) * x.astype(np.float64)
    yd = y.astype(np.float64)
    s = p + yd
    bb = s - p
    e = (p - (s - bb)) + (yd - bb)
    r = s.astype(np.float32)
    rd = r.astype(np.float64)
    other = np.where(rd < s, np.nextafter(r, np.float32(np.inf)),
                     np.nextafter(r, np.float32(-np.inf)))
    tie = (rd != s) & ((rd + other.astype(np.float64)) * 0.5 == s) & (e != 0)
    hi, lo = np.maximum(r, other), np.minimum(r, other)
    return np.where(tie & (e > 0), hi, np.where(tie & (e < 0), lo, r))


REDUCTIONS = ["dot", "l2_norm_sq", "max_value", "pipeline_sum"]
CHECK_SLICE = 1 << 16


def _sum_values(entry: str, data, lo: int, hi: int):
    """The fp32 per-element values a suite sum folds, for [lo, hi) of this
    rank's inputs (pipeline_sum's fmaf is formed in fp64 and rounded once
    more to fp32; a double rounding there moves a value by one fp32 ulp at
    most, far below the sum's bar)."""
    if entry == "dot":
        return data["u0"][lo:hi] * data["u1"][lo:hi]
    if entry == "l2_norm_sq":
        v = data["outl"][lo:hi]
        return v * v
    z = (0.75 * data["u0"][lo:hi].double() + data["u1"][lo:hi].double()).float()
    return z.clamp_min(0.0) * data["u2"][lo:hi]


def check_results(data, outs, n: int, world: int, rank: int, device: str = "cuda"):
    """After the timed region: the results of the last step against
    independent references.  Sums: the ranks' fp64 sums of the fp32
    per-element values, all-reduced, with the bar |got - ref| <= 1e-6 *
    log2(N) * |ref| over the global N; max: exact against a MAX all-reduce
    of torch.max; every rank's reduction outputs bit-identical to rank 0's;
    maps: a 2^16-element window of every rank's outputs bit for bit against
    the host (fmaf formed exactly, relu as x > 0 ? x : 0)."""
    import numpy as np
    import torch
    local = torch.zeros(3, dtype=torch.float64, device=device)
    chunk = 1 << 26
    for i, e in enumerate(["dot", "l2_norm_sq", "pipeline_sum"]):
        for lo in range(0, n, chunk):
            local[i] += _sum_values(e, data, lo, min(n, lo + chunk)).double().sum()
    mx = data["outl"].max().reshape(1)
    if world > 1:
        import torch.distributed as dist
        dist.all_reduce(local, op=dist.ReduceOp.SUM)
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
    refs = local.tolist()
    got = {e: float(outs[e][0].item()) for e in REDUCTIONS}
    bits = {e: int(outs[e].view(torch.int32)[0].item()) for e in REDUCTIONS}
    all_bits = gather_obj(world, bits)
    identical = all(b == all_bits[0] for b in all_bits)
    n_global = n * world
    bar = 1e-6 * max(1.0, math.log2(n_global))
    result = {"ranks": world, "global_n": n_global,
              "reductions_identical_on_every_rank": identical}
    ok = identical
    for e, ref in zip(["dot", "l2_norm_sq", "pipeline_sum"], refs):
        rel = abs(got[e] - ref) / abs(ref) if ref != 0 else abs(got[e])
        passed = rel <= bar
        ok &= passed
        result[e] = {"got": got[e], "ref_fp64": ref, "rel_err": rel, "bar": bar,
                     "passed": passed}
    max_ok = got["max_value"] == float(mx.item())
    ok &= max_ok
    result["max_value"] = {"got": got["max_value"], "ref": float(mx.item()), "passed": max_ok}
    L = min(n, CHECK_SLICE)
    lo = (rank * 7919 * 4096) % max(1, n - L + 1)
    x = data["u0"][lo:lo + L].cpu().numpy()
    y = data["u1"][lo:lo + L].cpu().numpy()
    r = data["nrm"][lo:lo + L].cpu().numpy()
    want = {"saxpy": fmaf_f32(2.5, x, y),
            "relu": np.where(r > 0, r, np.float32(0.0)).astype(np.float32)}
    z = fmaf_f32(0.75, x, y)
    want["affine_relu"] = np.where(z > 0, z, np.float32(0.0)).astype(np.float32)
    maps_ok = {}
    for e, w in want.items():
        g = outs[e][lo:lo + L].cpu().numpy()
        maps_ok[e] = bool(np.array_equal(g.view(np.uint32), w.view(np.uint32)))
    all_maps = gather_obj(world, maps_ok)
    maps = {e: all(m[e] for m in all_maps) for e in want}
    ok &= all(maps.values())
    result["maps_bit_exact"] = maps
    result["map_elems_checked_per_rank"] = L
    result["passed"] = bool(ok)
    return result


def run_ours(args) -> None:
    import ctypes

    import torch
    from loom_b200.build import load_suite

    world, rank, local = setup_dist(args)
    pkg = load_suite()
    n = 1 << args.n_log2
    peak, peak_src = read_peak()
    data = make_inputs(n, rank)
    outs = {e: torch.empty(n if e in MAP_ENTRIES else 1, device="cuda") for e in ENTRIES}
    comm = pkg.comm_from_process_group() if world > 1 else None
    if comm is not None and args.exchange == "nccl":
        comm.set_peer_exchange(False)
    stream = torch.cuda.current_stream()

    # Pre-bind every call (no Python tensor work inside the timed loop).
    calls = []
    for e in ENTRIES:
        ent = pkg[e]
        args_c = []
        tens = dict(zip(PARAM_NAMES[e], TENSORS[e]))
        for p in ent.params:
            if p["kind"] == "scalar-f32":
                args_c.append(ctypes.c_float(SCALARS[e][p["name"]]))
            else:
                args_c.append(ctypes.c_void_p(data[tens[p["name"]]].data_ptr()))
        if world > 1:
            ws = ent.workspace(n, dist=True)
            tail = [ctypes.c_int64(n), ctypes.c_void_p(outs[e].data_ptr()),
                    ctypes.c_void_p(ws.data_ptr()) if ws is not None else None,
                    ctypes.c_size_t(ws.numel() if ws is not None else 0),
                    ctypes.c_void_p(comm.handle), ctypes.c_void_p(stream.cuda_stream)]
            fn = ent.dist_fn
        else:
            ws = ent.workspace(n)
            tail = [ctypes.c_int64(n), ctypes.c_void_p(outs[e].data_ptr()),
                    ctypes.c_void_p(ws.data_ptr()) if ws is not None else None,
                    ctypes.c_size_t(ws.numel() if ws is not None else 0),
                    ctypes.c_void_p(stream.cuda_stream)]
            fn = ent.stream_fn
        calls.append((e, fn, args_c + tail))

    def step(events=None):
        for i, (e, fn, a) in enumerate(calls):
            if events is not None:
                events[i][0].record(stream)
            st = fn(*a)
            if st != 0:
                raise RuntimeError(f"{e} returned status {st}")
            if events is not None:
                events[i][1].record(stream)

    props = torch.cuda.get_device_properties(local)
    sampler = ClockSampler(f"GPU-{props.uuid}" if hasattr(props, "uuid") else str(local))
    sampler.start()
    sampler.wait_first()
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()

    per_kernel = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                   for _ in calls] for _ in range(args.steps)]
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    if comm is not None:
        comm.exchange_stats(reset=True)
    barrier(world)
    torch.cuda.synchronize()
    sampler.mark_start()
    start.record(stream)
    for s in range(args.steps):
        step(per_kernel[s])
    end.record(stream)
    torch.cuda.synchronize()
    sampler.mark_end()
    barrier(world)
    clocks = sampler.stop()
    wait = comm.exchange_stats() if comm is not None else None
    elapsed_ms = start.elapsed_time(end)
    kernel_ms = {e: sum(per_kernel[s][i][0].elapsed_time(per_kernel[s][i][1])
                        for s in range(args.steps)) / args.steps
                 for i, (e, _, _) in enumerate(calls)}
    elapsed_ms = max_over_ranks(world, elapsed_ms)
    ms_per_step = elapsed_ms / args.steps
    step_bytes = sum(bytes_per_elem(e) for e in ENTRIES) * n
    value = step_bytes * world / (ms_per_step * 1e-3) / 1e9

    # e2e through the reference-facing synchronous entry with pinned host buffers
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(pkg, data, outs, n, args, world, comm)
    ref_kernels = None
    if world == 1 and args.ref_kernel_steps > 0:
        ref_kernels = run_reference_kernels(data, outs, n, args)
    check = check_results(data, outs, n, world, rank)
    all_clocks = gather_obj(world, clocks)
    all_kernels = gather_obj(world, kernel_ms)
    all_wait = gather_obj(world, wait)

    if rank == 0:
        traffic = read_traffic()
        kernels = {}
        for e in ENTRIES:
            ms = max(k[e] for k in all_kernels)
            gbs = bytes_per_elem(e) * n / (ms * 1e-3) / 1e9
            kernels[e] = {"us_per_call": round(ms * 1e3, 2), "gbs": round(gbs, 1),
                          "frac": round(gbs / peak, 4), "bytes_per_elem": bytes_per_elem(e)}
        dom = max(ENTRIES, key=lambda e: kernels[e]["us_per_call"])
        dom_bytes = bytes_per_elem(dom) * n
        # ncu's DRAM bytes of one launch at 2^26, scaled to this N: the reads
        # are the algorithmic bytes exactly, so traffic grows in proportion
        measured = traffic.get(dom, {}).get("dram_bytes_per_launch_at_2^26")
        dom_traffic = int(measured * n / (1 << 26)) if measured else None
        line = {
            "metric": METRIC,
            "value": round(value, 1),
            "unit": "GB/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_per_step, 4),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "f32",
            "data": "synthetic (seeded U(-1,1), N(0,1), N(0,1) with 1% x1e3 outliers)",
            "pct_of_peak": round(100 * value / (peak * world), 2),
            "config": suite_config(world, args.n_log2),
            "exchange": (None if comm is None else
                         ("peer memory (NVLink P2P stores)" if comm.peer_exchange
                          else "NCCL all-gather / all-reduce")),
            "kernels": kernels,
            "roofline": {
                "bound": "hbm",
                "kernel": dom,
                "achieved": round(dom_bytes / (kernels[dom]["us_per_call"] * 1e-6) / 1e9, 1),
                "peak": peak,
                "peak_source": peak_src,
                "unit": "GB/s",
                "frac": round(dom_bytes / (kernels[dom]["us_per_call"] * 1e-6) / 1e9 / peak, 4),
                "traffic": dom_traffic,
                "algorithmic_bytes_per_launch": dom_bytes,
            },
            "clocks": {
                "sm_mhz": all_clocks[0]["sm_mhz"],
                "sm_max_mhz": all_clocks[0]["sm_max_mhz"],
                "reasons": sorted({r for c in all_clocks for r in c["reasons"]}),
                "per_rank_sm_mhz": [c["sm_mhz"] for c in all_clocks],
            },
            "gpu_launches": args.steps * sum(
                launches_per_call(e, world, n, comm is not None and comm.peer_exchange)
                for e in ENTRIES),
            "e2e": e2e,
            "check": check,
        }
        if comm is not None and comm.peer_exchange:
            line["exchange_wait"] = {
                "what": "per rank, over the timed steps: time from sending its value to "
                        "holding every rank's, in each reduction's peer exchange "
                        "(%globaltimer stamps in the exchange)",
                "exchanges_per_rank": all_wait[0]["exchanges"],
                "mean_us_per_exchange": [round(w["total_us"] / max(1, w["exchanges"]), 2)
                                         for w in all_wait],
                "max_us": [round(w["max_us"], 2) for w in all_wait],
            }
        if ref_kernels is not None:
            ref_kernels["product_over_profile"] = {
                p: round(value / v["value"], 3) for p, v in ref_kernels["profiles"].items()}
            line["reference_kernels"] = ref_kernels
        if world == 1 and not args.no_cpu:
            line["cpu_baseline"] = cpu_baseline(args.cpu_log2, args.cpu_seconds)
        emit(line)
    if comm is not None:
        comm.check()
        comm.destroy()
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    if not check["passed"]:
        sys.exit(1)


def run_e2e(pkg, data, outs, n, args, world, comm):
    """Host-buffer end to end: every step copies each entry's inputs from
    pinned host memory to the GPU, runs it and copies the result back.

    `value` goes through the public host-buffer call (`Entry.call_host`,
    which pipelines a map's chunks so that input and output copies overlap
    and uses the `_dist` entry for reductions across GPUs); `sync_abi` is
    the same loop through the plain synchronous reference entry with one
    whole-array copy in and out."""
    import ctypes

    import torch
    host = {k: torch.empty(n, dtype=torch.float32, pin_memory=True) for k in data}
    for k, v in data.items():
        host[k].copy_(v)
    host_out = {e: torch.empty(n if e in MAP_ENTRIES else 1, dtype=torch.float32,
                               pin_memory=True) for e in ENTRIES}
    stream = torch.cuda.current_stream()
    h2d = sum(4 * n * len(TENSORS[e]) for e in ENTRIES)
    d2h = sum(4 * (n if e in MAP_ENTRIES else 1) for e in ENTRIES)
    step_bytes = sum(bytes_per_elem(e) for e in ENTRIES) * n

    def pipelined_step():
        for e in ENTRIES:
            ent = pkg[e]
            kw = {p: host[t] for p, t in zip(PARAM_NAMES[e], TENSORS[e])}
            kw.update(SCALARS.get(e, {}))
            ent.call_host(out=host_out[e], comm=comm if world > 1 else None, **kw)

    def sync_abi_step():
        for e in ENTRIES:
            ent = pkg[e]
            for k in set(TENSORS[e]):
                data[k].copy_(host[k], non_blocking=True)
            args_c = []
            tens = dict(zip(PARAM_NAMES[e], TENSORS[e]))
            for p in ent.params:
                if p["kind"] == "scalar-f32":
                    args_c.append(ctypes.c_float(SCALARS[e][p["name"]]))
                else:
                    args_c.append(ctypes.c_void_p(data[tens[p["name"]]].data_ptr()))
            ws = ent.workspace(n, dist=world > 1)
            tail = [ctypes.c_int64(n), ctypes.c_void_p(outs[e].data_ptr()),
                    ctypes.c_void_p(ws.data_ptr()) if ws is not None else None,
                    ctypes.c_size_t(ws.numel() if ws is not None else 0)]
            if world > 1:
                st = ent.dist_fn(*args_c, *tail, ctypes.c_void_p(comm.handle),
                                 ctypes.c_void_p(stream.cuda_stream))
            else:
                st = ent.fn(*args_c, *tail)
            if st != 0:
                raise RuntimeError(f"{e} returned status {st}")
            host_out[e].copy_(outs[e], non_blocking=True)
        stream.synchronize()

    def timed(step):
        steps = max(1, args.e2e_steps)
        step()
        torch.cuda.synchronize()
        barrier(world)
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(steps):
            step()            # returns only after its copies and kernels completed
        end.record(stream)
        torch.cuda.synchronize()
        return max_over_ranks(world, start.elapsed_time(end)) / steps

    ms = timed(pipelined_step)
    ms_sync = timed(sync_abi_step)
    return {"value": round(step_bytes * world / (ms * 1e-3) / 1e9, 2), "unit": "GB/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": max(1, args.e2e_steps),
            "ms_per_step": round(ms, 3),
            "path": "Entry.call_host (public host-buffer call: chunked map pipeline, "
                    + ("_stream entries" if world == 1 else "_dist entries for reductions")
                    + "), pinned host buffers, CUDA events around whole synchronised steps",
            "sync_abi": {"value": round(step_bytes * world / (ms_sync * 1e-3) / 1e9, 2),
                         "ms_per_step": round(ms_sync, 3),
                         "path": ("loom_kernels_<entry> (synchronous reference ABI)"
                                  if world == 1 else "loom_kernels_<entry>_dist")
                                 + ", one whole-array copy in and out"}}


def run_reference_kernels(data, outs, n, args):
    """The reference's generated CUDA for the same seven entries, restated by
    hand (baseline/loom_reference_style.cu) under its "none" and "cuda"
    profiles, timed on this GPU like the product: CUDA events around every
    call on the launching stream, the same inputs, steps of the seven calls.
    Each profile's outputs are checked against the product's first."""
    import torch
    from baseline import reference_style as rs
    lib = rs.ReferenceStyle()
    stream = torch.cuda.current_stream()
    step_bytes = sum(bytes_per_elem(e) for e in ENTRIES) * n
    result = {"source": "baseline/loom_reference_style.cu (nvcc -O3, sm_100a)",
              "steps": args.ref_kernel_steps, "profiles": {}}
    for profile in rs.PROFILES:
        calls, bufs = [], []
        for e in ENTRIES:
            kw = {p: data[t] for p, t in zip(PARAM_NAMES[e], TENSORS[e])}
            kw.update(SCALARS.get(e, {}))
            out = torch.empty_like(outs[e])
            size = lib.workspace_size(profile, e, n)
            ws = torch.empty(size, dtype=torch.uint8, device="cuda") if size else None
            bufs.append((out, ws))
            calls.append((e, out, lib.bind(profile, e, n, out, ws, **kw)))

        def step(events=None):
            for i, (e, _, fn) in enumerate(calls):
                if events is not None:
                    events[i][0].record(stream)
                st = fn()
                if st != 0:
                    raise RuntimeError(f"reference-style {profile} {e} returned status {st}")
                if events is not None:
                    events[i][1].record(stream)

        for _ in range(3):
            step()
        torch.cuda.synchronize()
        agrees = {}
        for e, out, _ in calls:
            if e in MAP_ENTRIES or e == "max_value":
                agrees[e] = bool(torch.equal(out.view(torch.int32), outs[e].view(torch.int32)))
            else:
                a, b = float(out[0]), float(outs[e][0])
                agrees[e] = abs(a - b) <= 1e-4 * (abs(b) + math.sqrt(n))
        ev = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in calls] for _ in range(args.ref_kernel_steps)]
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        start.record(stream)
        for s in range(args.ref_kernel_steps):
            step(ev[s])
        end.record(stream)
        torch.cuda.synchronize()
        ms = start.elapsed_time(end) / args.ref_kernel_steps
        kernels = {}
        for i, (e, _, _) in enumerate(calls):
            k_ms = sum(ev[s][i][0].elapsed_time(ev[s][i][1])
                       for s in range(args.ref_kernel_steps)) / args.ref_kernel_steps
            kernels[e] = {"us_per_call": round(k_ms * 1e3, 2),
                          "gbs": round(bytes_per_elem(e) * n / (k_ms * 1e-3) / 1e9, 1)}
        result["profiles"][profile] = {
            "value": round(step_bytes / (ms * 1e-3) / 1e9, 1), "unit": "GB/s",
            "ms_per_step": round(ms, 4),
            "gpu_launches_per_step": sum(rs.LAUNCHES_2P28[profile].values()),
            "kernels": kernels, "agrees_with_product": agrees}
        del calls, bufs
        torch.cuda.empty_cache()
    return result


def cpu_baseline(log2n: int, seconds: float, threads: int = 0, single_log2n: int = 24):
    """The C oracle (the reference's per-element semantics, OpenMP) on the
    host cores, on the GPU arm's per-GPU workload (N=2^log2n per entry) for
    about `seconds`; reports effective GB/s.  The one-core figure is taken on
    N=2^single_log2n per entry, to keep it to a few seconds."""
    from oracle.loom_oracle import Oracle, load_programs
    threads = threads or len(os.sched_getaffinity(0))
    oracle = Oracle(load_programs(os.path.join(ROOT, "oracle",
                                               "suite_kernels.tensor_ir.json")), name="b200_suite")
    n = 1 << log2n
    inputs = cpu_suite_inputs(n)
    for e in ENTRIES:
        oracle.run(e, inputs[e], threads=threads)
    reps, total = 0, 0.0
    t0 = time.perf_counter()
    while True:
        for e in ENTRIES:
            oracle.run(e, inputs[e], threads=threads)
        reps += 1
        total = time.perf_counter() - t0
        if total >= seconds:
            break
    step_bytes = sum(bytes_per_elem(e) for e in ENTRIES) * n
    del inputs
    n1 = 1 << single_log2n
    inputs1 = cpu_suite_inputs(n1)
    reps1 = 0
    t0 = time.perf_counter()
    while True:
        for e in ENTRIES:
            oracle.run(e, inputs1[e], threads=1)
        reps1 += 1
        total1 = time.perf_counter() - t0
        if total1 >= seconds / 4:
            break
    step_bytes1 = sum(bytes_per_elem(e) for e in ENTRIES) * n1
    return {"value": round(step_bytes * reps / total / 1e9, 2), "unit": "GB/s",
            "cores": threads, "kind": "port",
            "sample": f"the 7 suite entries at N=2^{log2n} each (the GPU arm's per-GPU "
                      f"workload), {reps} steps in {total:.1f} s",
            "seconds": round(total, 2),
            "single_thread": {"value": round(step_bytes1 * reps1 / total1 / 1e9, 2),
                              "unit": "GB/s", "cores": 1,
                              "sample": f"N=2^{single_log2n} per entry, {reps1} steps in "
                                        f"{total1:.1f} s"}}


def run_reference(args) -> None:
    """The reference arm: the CPU restatement of the reference's semantics for
    this path (the C oracle; the reference has no CPU implementation of it
    and its OCaml compiler cannot be built here) on all host cores, timing
    exactly --steps steps after --warmup.  A step is the GPU arm's per-GPU
    workload, the seven entries at N=2^--n-log2 each; with N GPUs the GPU
    arm's step is N such shards, which the host cores would process one
    after another at the same rate, so the line reports the same metric on
    the GPU arm's config.  Under torchrun only rank 0 runs."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    from oracle.loom_oracle import Oracle, load_programs
    threads = len(os.sched_getaffinity(0))
    oracle = Oracle(load_programs(os.path.join(ROOT, "oracle",
                                               "suite_kernels.tensor_ir.json")), name="b200_suite")
    n = 1 << args.n_log2
    inputs = cpu_suite_inputs(n)
    for _ in range(args.warmup):
        for e in ENTRIES:
            oracle.run(e, inputs[e], threads=threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        for e in ENTRIES:
            oracle.run(e, inputs[e], threads=threads)
    total = time.perf_counter() - t0
    step_bytes = sum(bytes_per_elem(e) for e in ENTRIES) * n
    value = step_bytes * args.steps / total / 1e9
    sample = (f"one GPU's shard of the workload per step: the 7 suite entries at "
              f"N=2^{args.n_log2} each" + (f" (of {world} shards)" if world > 1 else ""))
    emit({
        "impl": "reference",
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(total / args.steps * 1e3, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded U(-1,1), N(0,1), N(0,1) with 1% x1e3 outliers)",
        "config": suite_config(world, args.n_log2),
        "cpu_baseline": {"value": round(value, 2), "unit": "GB/s", "cores": threads,
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 2), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    })


def _median_us(call, reps: int, flush, stream) -> float:
    """Median device time of `call` in us: CUDA events on the launching
    stream around each call, after 3 untimed calls.  `flush` is None or a
    pair of buffers larger than L2: before every timed call the first is
    rewritten (so no input is served from L2) and the second is read, which
    writes the dirty lines of the first back before the timed call starts
    rather than during it."""
    import torch
    for _ in range(3):
        call()
    times = []
    for _ in range(reps):
        if flush is not None:
            flush[0].fill_(1.0)
            flush[1].sum()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        call()
        b.record(stream)
        b.synchronize()
        times.append(a.elapsed_time(b) * 1e3)
    return statistics.median(times)


def _median_wall_us(call, reps: int, flush) -> float:
    """Median host wall time of `call` in us, the way the reference harness
    times a kernel (experiments/source/harness/run.py:1154-1166): device
    synchronise, perf_counter, the call, device synchronise, perf_counter;
    with the same L2 flush as _median_us before each call."""
    import torch
    for _ in range(3):
        call()
    torch.cuda.synchronize()
    times = []
    for _ in range(reps):
        if flush is not None:
            flush[0].fill_(1.0)
            flush[1].sum()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        call()
        torch.cuda.synchronize()
        times.append((time.perf_counter() - t0) * 1e6)
    return statistics.median(times)


def _graph_us(entry_obj, kw, out, calls: int = 20, replays: int = 20) -> float:
    """Per-call device time of `calls` back-to-back calls captured in one CUDA
    graph on a side stream and replayed `replays` times (no flush: the
    launch-bound regime this is meant for)."""
    import torch
    side = torch.cuda.Stream()
    call, _ = entry_obj.bind(out=out, stream=side, **kw)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        for _ in range(calls):
            call()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    cur = torch.cuda.current_stream()
    a.record(cur)
    for _ in range(replays):
        graph.replay()
    b.record(cur)
    b.synchronize()
    us = a.elapsed_time(b) * 1e3 / (calls * replays)
    del graph
    return us


def _reference_calls(lib, entry, n, out, kw):
    """Bound reference-style calls of both profiles, with their workspaces."""
    import torch
    calls = {}
    for profile in ("cuda", "none"):
        size = lib.workspace_size(profile, entry, n)
        ws = torch.empty(size, dtype=torch.uint8, device="cuda") if size else None
        fn = lib.bind(profile, entry, n, out, ws, **kw)

        def call(fn=fn, profile=profile):
            st = fn()
            if st != 0:
                raise RuntimeError(f"reference-style {profile} {entry} returned status {st}")
        calls[profile] = (call, ws)
    return calls


def _timed_row(row, entry, nbytes, product_call, ref_calls, reps, flush, stream, peak):
    us = _median_us(product_call, reps, flush, stream)
    row[entry + "_us"] = round(us, 2)
    row[entry + "_gbs"] = round(nbytes / (us * 1e-6) / 1e9, 1)
    row[entry + "_frac"] = round(nbytes / (us * 1e-6) / 1e9 / peak, 4)
    row[entry + "_wall_us"] = round(_median_wall_us(product_call, reps, flush), 2)
    for profile, (call, _) in ref_calls.items():
        r_us = _median_us(call, reps, flush, stream)
        row[f"{entry}_ref_{profile}_us"] = round(r_us, 2)
        row[f"{entry}_ref_{profile}_gbs"] = round(nbytes / (r_us * 1e-6) / 1e9, 1)
        row[f"{entry}_ref_{profile}_wall_us"] = round(_median_wall_us(call, reps, flush), 2)


def run_pipeline_sweep(args) -> None:
    """The fused-pipeline configuration swept over N (1 GPU): device time per
    call of affine_relu (z = relu(a*x + y)) and pipeline_sum (sum(z*w)),
    median of CUDA-event-timed calls, for the product and for the
    reference-style kernels of both profiles on the same inputs.  A 512 MiB
    buffer is rewritten (then another read) before every timed call, so
    that no input is served from L2 and the kernels' cache hints cannot
    favour one side through lines left over from the previous call.  Every
    call is bound once, so the per-call host work is the same for both.  Up
    to 2^26 the product is also timed as 20 back-to-back calls replayed from
    one CUDA graph (`*_graph_us`, per call, no flush).  Prints one JSON
    line."""
    import torch
    from baseline.reference_style import ReferenceStyle
    from loom_b200.build import load_suite
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    pkg = load_suite()
    lib = ReferenceStyle()
    peak, peak_src = read_peak()
    stream = torch.cuda.current_stream()
    flush_buf = (torch.empty(128 << 20, dtype=torch.float32, device="cuda"),
                 torch.ones(128 << 20, dtype=torch.float32, device="cuda"))
    points = []
    gen = torch.Generator(device="cuda")
    for log2n in args.sweep:
        n = 1 << log2n
        gen.manual_seed(20260417 + log2n)
        x = torch.rand(n, device="cuda", generator=gen).mul_(2).sub_(1)
        y = torch.rand(n, device="cuda", generator=gen).mul_(2).sub_(1)
        w = torch.rand(n, device="cuda", generator=gen).mul_(2).sub_(1)
        z = torch.empty(n, device="cuda")
        s = torch.empty(1, device="cuda")
        reps = 200 if n <= (1 << 22) else (20 if n <= (1 << 28) else 5)
        flush = flush_buf
        row = {"n": n, "log2n": log2n, "l2_flush": True}
        kz = {"a": 0.75, "x": x, "y": y}
        ks = {"a": 0.75, "x": x, "y": y, "w": w}
        refs = _reference_calls(lib, "affine_relu", n, z, kz)
        call, _ = pkg["affine_relu"].bind(out=z, stream=stream, **kz)
        _timed_row(row, "affine_relu", 12 * n, call, refs, reps, flush, stream, peak)
        del refs
        refs = _reference_calls(lib, "pipeline_sum", n, s, ks)
        call, _ = pkg["pipeline_sum"].bind(out=s, stream=stream, **ks)
        _timed_row(row, "pipeline_sum", 12 * n, call, refs, reps, flush, stream, peak)
        del refs
        if n <= (1 << 26):
            row["affine_relu_graph_us"] = round(_graph_us(pkg["affine_relu"], kz, z), 2)
            row["pipeline_sum_graph_us"] = round(_graph_us(pkg["pipeline_sum"], ks, s), 2)
        points.append(row)
        del x, y, w, z
        torch.cuda.empty_cache()
    emit({"mode": "pipeline_sweep", "metric": METRIC, "unit": "GB/s", "peak": peak,
          "peak_source": peak_src,
          "config": {"workload": "fused pipeline: affine_relu z = relu(0.75*x + y) "
                                 "and pipeline_sum s = sum(z*w), x, y, w ~ U(-1,1)"},
          "points": points})


# The four single-entry workload configurations, each at its own size.
CONFIG_POINTS = [("saxpy", 24), ("relu", 26), ("dot", 28), ("l2_norm_sq", 30), ("max_value", 30)]


def run_config_sweep(args) -> None:
    """Each workload configuration at its own N (saxpy 2^24, relu 2^26, dot
    2^28, l2_norm_sq and max_value 2^30; 1 GPU): median device time per call
    of the product and of the reference-style kernels of both profiles, on
    the configuration's seeded inputs.  A 512 MiB buffer is rewritten (then
    another read) before every timed call.  Prints one JSON line."""
    import torch
    from baseline.reference_style import ReferenceStyle
    from loom_b200.build import load_suite
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    pkg = load_suite()
    lib = ReferenceStyle()
    peak, peak_src = read_peak()
    stream = torch.cuda.current_stream()
    flush_buf = (torch.empty(128 << 20, dtype=torch.float32, device="cuda"),
                 torch.ones(128 << 20, dtype=torch.float32, device="cuda"))
    points = []
    for entry, log2n in CONFIG_POINTS:
        n = 1 << log2n
        data = make_inputs(n, 0)
        kw = {p: data[t] for p, t in zip(PARAM_NAMES[entry], TENSORS[entry])}
        kw.update(SCALARS.get(entry, {}))
        for k in list(data):
            if k not in TENSORS[entry]:
                del data[k]
        torch.cuda.empty_cache()
        out = torch.empty(n if entry in MAP_ENTRIES else 1, device="cuda")
        nbytes = bytes_per_elem(entry) * n
        flush = flush_buf
        reps = 50 if n <= (1 << 26) else 20
        row = {"entry": entry, "n": n, "log2n": log2n, "l2_flush": True,
               "bytes_per_call": nbytes}
        refs = _reference_calls(lib, entry, n, out, kw)
        call, _ = pkg[entry].bind(out=out, stream=stream, **kw)
        _timed_row(row, entry, nbytes, call, refs, reps, flush, stream, peak)
        points.append(row)
        del refs, data, kw, out
        torch.cuda.empty_cache()
    emit({"mode": "config_sweep", "metric": METRIC, "unit": "GB/s", "peak": peak,
          "peak_source": peak_src, "points": points})


def run_workload_sweep(args) -> None:
    """The reference harness's 33 supported kernels (packaged from the
    FrontIR fixtures in tests/golden/sources/workloads) at N = 2^log2 for
    each --sweep size (1 GPU): median device time per call (bound calls,
    CUDA events, 20 calls after 3 warm-up, a write-then-read 512 MiB L2
    flush before each), inputs N(0,1) and the harness's scalar arguments.
    GB/s = 4 bytes x (tensor inputs + 1 for a tensor result) x N / time.
    --workload-package picks the build: the default flags ("workloads"),
    the fusion and body-rendering flags ("workloads_flags"), or the flag set
    of the reference harness's tuned CUDA profile ("workloads_cuda_fixed").
    Prints one JSON line."""
    import torch
    from loom_b200.build import BUILT_DIR
    from loom_b200.loader import Package
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    table_path = os.path.join(ROOT, "tests", "golden", "sources", "workloads", "workloads.json")
    with open(table_path) as fh:
        table = json.load(fh)
    pkg = Package(os.path.join(BUILT_DIR, args.workload_package))
    peak, peak_src = read_peak()
    stream = torch.cuda.current_stream()
    flush = (torch.empty(128 << 20, dtype=torch.float32, device="cuda"),
             torch.ones(128 << 20, dtype=torch.float32, device="cuda"))
    gen = torch.Generator(device="cuda")
    points = []
    for log2n in args.sweep:
        n = 1 << log2n
        for k, w in enumerate(table):
            gen.manual_seed(20260417 + 104729 * k + log2n)
            kw = {t: torch.randn(n, device="cuda", generator=gen) for t in w["tensor_inputs"]}
            kw.update({name: float(v) for name, v in w["scalar_args"].items()})
            tensor_out = w["result_kind"] == "tensor"
            out = torch.empty(n if tensor_out else 1, device="cuda")
            call, _ = pkg[w["entry"]].bind(out=out, stream=stream, **kw)
            us = _median_us(call, 20, flush, stream)
            nbytes = 4 * n * (len(w["tensor_inputs"]) + (1 if tensor_out else 0))
            points.append({"workload": w["name"], "log2n": log2n, "us": round(us, 2),
                           "gbs": round(nbytes / (us * 1e-6) / 1e9, 1),
                           "frac": round(nbytes / (us * 1e-6) / 1e9 / peak, 4),
                           "bytes_per_call": nbytes})
            del kw, out, call
        torch.cuda.empty_cache()
    emit({"mode": "workload_sweep", "metric": METRIC, "unit": "GB/s", "peak": peak,
          "peak_source": peak_src, "package": args.workload_package, "points": points})


# Fixed global sizes for the strong-scaling mode: (config, entries, log2 of the
# global N, input distribution); the pipeline at every --strong-sizes size.
STRONG_L2_MAX = ("l2_norm_sq_max", ("l2_norm_sq", "max_value"), 30, "normal_outliers")


def global_slice(kind: str, seed: int, start: int, stop: int, chunk: int = 1 << 24,
                 device: str = "cuda"):
    """Elements [start, stop) of a seeded global input that does not depend
    on how it is sharded: the global array is cut into fixed chunks, each
    drawn on the device from its own seed, and a rank draws only the chunks
    its shard overlaps."""
    import torch
    out = torch.empty(stop - start, device=device)
    gen = torch.Generator(device=device)
    c = start // chunk
    while c * chunk < stop:
        lo = c * chunk
        gen.manual_seed(seed * 1000003 + c)
        if kind == "uniform":
            v = torch.rand(chunk, device=device, generator=gen).mul_(2.0).sub_(1.0)
        else:
            v = torch.randn(chunk, device=device, generator=gen)
            v[torch.rand(chunk, device=device, generator=gen) < 0.01] *= 1e3
        s0, s1 = max(start, lo), min(stop, lo + chunk)
        out[s0 - start:s1 - start] = v[s0 - lo:s1 - lo]
        c += 1
    return out


def _bound_entry(pkg, entry, tensors, n_local, out, world, comm, stream):
    """A pre-converted call of `entry` on this rank's shard: the `_dist`
    entry across GPUs, the stream entry on one."""
    import ctypes
    ent = pkg[entry]
    args_c = []
    for p in ent.params:
        if p["kind"] == "scalar-f32":
            args_c.append(ctypes.c_float(SCALARS[entry][p["name"]]))
        else:
            args_c.append(ctypes.c_void_p(tensors[p["name"]].data_ptr()))
    ws = ent.workspace(max(1, n_local), dist=world > 1)
    tail = [ctypes.c_int64(n_local), ctypes.c_void_p(out.data_ptr()),
            ctypes.c_void_p(ws.data_ptr()) if ws is not None else None,
            ctypes.c_size_t(ws.numel() if ws is not None else 0)]
    if world > 1:
        fn, tail = ent.dist_fn, tail + [ctypes.c_void_p(comm.handle)]
    else:
        fn = ent.stream_fn
    tail.append(ctypes.c_void_p(stream.cuda_stream))

    def call():
        st = fn(*args_c, *tail)
        if st != 0:
            raise RuntimeError(f"{entry} returned status {st}")
    return call, ws


def run_strong(args) -> None:
    """Strong scaling: fixed global sizes sharded over the N ranks with
    loom_b200.shard (l2_norm_sq and max_value at N = 2^30; the fused
    pipeline, affine_relu and pipeline_sum, at every --strong-sizes size).
    Per call: a write-then-read 512 MiB L2 flush, a one-element all-reduce
    that lines the ranks up on the device, then CUDA events around the call
    on every rank; a call's time is the max over ranks, and the point's time
    the median over the calls.  For reductions across GPUs the
    peer exchange's wait (from sending this rank's value to holding every
    rank's) is read from the exchange buffer's statistics.  Each point's
    results are checked: sums against the ranks' fp64 sums of the fp32
    values (bar 1e-6 * log2(N) * |ref|), max exactly, maps bit for bit on a
    2^16 window per rank.  Prints one JSON line."""
    import numpy as np
    import torch
    from loom_b200.build import load_suite
    from loom_b200.shard import shard_bounds
    world, rank, local = setup_dist(args)
    pkg = load_suite()
    comm = pkg.comm_from_process_group() if world > 1 else None
    stream = torch.cuda.current_stream()
    peak, peak_src = read_peak()
    flush = (torch.empty(128 << 20, dtype=torch.float32, device="cuda"),
             torch.ones(128 << 20, dtype=torch.float32, device="cuda"))
    align = torch.zeros(1, device="cuda")
    configs = [STRONG_L2_MAX] + [("pipeline", ("affine_relu", "pipeline_sum"), k, "uniform")
                                 for k in args.strong_sizes]
    points = []
    all_ok = True
    for name, entries, log2n, kind in configs:
        n = 1 << log2n
        start, stop = shard_bounds(n, world)[rank]
        n_local = stop - start
        names = ("x",) if kind != "uniform" else ("x", "y", "w")
        tens = {t: global_slice(kind, 20260417 + 104729 * k + log2n, start, stop)
                for k, t in enumerate(names)}
        reps = 50 if n <= (1 << 26) else (10 if n <= (1 << 30) else 5)
        for entry in entries:
            is_map = entry in MAP_ENTRIES
            out = torch.empty(max(1, n_local) if is_map else 1, device="cuda")
            call, ws = _bound_entry(pkg, entry, tens, n_local, out, world, comm, stream)
            for _ in range(3):
                call()
            torch.cuda.synchronize()
            if comm is not None:
                comm.exchange_stats(reset=True)
            barrier(world)
            times = []
            for _ in range(reps):
                flush[0].fill_(1.0)
                flush[1].sum()
                if world > 1:
                    # line the ranks up on the device: the start events below
                    # follow a collective that ends on every GPU at once, so a
                    # rank's flush does not count as the others' exchange wait
                    import torch.distributed as dist
                    dist.all_reduce(align)
                a = torch.cuda.Event(enable_timing=True)
                b = torch.cuda.Event(enable_timing=True)
                a.record(stream)
                call()
                b.record(stream)
                b.synchronize()
                times.append(a.elapsed_time(b) * 1e3)
            wait = comm.exchange_stats() if comm is not None else None
            all_times = gather_obj(world, times)
            per_call = [max(t[i] for t in all_times) for i in range(reps)]
            us = statistics.median(per_call)
            if is_map:
                L = min(n_local, CHECK_SLICE)
                lo = (rank * 7919 * 4096) % max(1, n_local - L + 1)
                x = tens["x"][lo:lo + L].cpu().numpy()
                y = tens["y"][lo:lo + L].cpu().numpy()
                z = fmaf_f32(0.75, x, y)
                want = np.where(z > 0, z, np.float32(0.0)).astype(np.float32)
                got = out[lo:lo + L].cpu().numpy()
                ok = bool(np.array_equal(got.view(np.uint32), want.view(np.uint32)))
                ok = all(gather_obj(world, ok))
                detail = {"maps_bit_exact": ok}
            else:
                got = float(out[0].item())
                if entry == "max_value":
                    ref = tens["x"].max().reshape(1)
                    if world > 1:
                        import torch.distributed as dist
                        dist.all_reduce(ref, op=dist.ReduceOp.MAX)
                    ok = got == float(ref.item())
                    detail = {"got": got, "ref": float(ref.item())}
                else:
                    acc = torch.zeros(1, dtype=torch.float64, device="cuda")
                    for lo in range(0, n_local, 1 << 26):
                        hi = min(n_local, lo + (1 << 26))
                        if entry == "l2_norm_sq":
                            v = tens["x"][lo:hi] * tens["x"][lo:hi]
                        else:
                            zz = (0.75 * tens["x"][lo:hi].double()
                                  + tens["y"][lo:hi].double()).float()
                            v = zz.clamp_min(0.0) * tens["w"][lo:hi]
                        acc += v.double().sum()
                    if world > 1:
                        import torch.distributed as dist
                        dist.all_reduce(acc, op=dist.ReduceOp.SUM)
                    ref = float(acc.item())
                    rel = abs(got - ref) / abs(ref)
                    ok = rel <= 1e-6 * max(1.0, math.log2(n))
                    detail = {"got": got, "ref_fp64": ref, "rel_err": rel}
                bits = gather_obj(world, float(np.float32(got)))
                ok = bool(ok) and all(b == bits[0] for b in bits)
            all_ok &= bool(ok)
            nbytes = bytes_per_elem(entry) * n
            row = {"config": name, "entry": entry, "global_n": n, "log2n": log2n,
                   "n_per_rank_max": max(b - a for a, b in shard_bounds(n, world)),
                   "us_per_call": round(us, 2), "gbs": round(nbytes / (us * 1e-6) / 1e9, 1),
                   "frac_of_world_peak": round(nbytes / (us * 1e-6) / 1e9 / (peak * world), 4),
                   "reps": reps, "check": dict(detail, passed=bool(ok))}
            if wait is not None and not is_map:
                waits = gather_obj(world, wait)
                row["exchange_wait_us_mean"] = [round(w["total_us"] / max(1, w["exchanges"]), 2)
                                                for w in waits]
                row["exchange_wait_us_max"] = [round(w["max_us"], 2) for w in waits]
            points.append(row)
            del out, ws, call
        del tens
        torch.cuda.empty_cache()
    if rank == 0:
        emit({"mode": "strong", "metric": METRIC, "unit": "GB/s", "n_gpus": world,
              "scaling": "strong", "peak": peak, "peak_source": peak_src,
              "exchange": (None if comm is None else
                           ("peer memory (NVLink P2P stores)" if comm.peer_exchange
                            else "NCCL all-gather / all-reduce")),
              "config": {"workload": "fixed global N sharded over the ranks: l2_norm_sq and "
                                     "max_value at 2^30 (N(0,1), 1 percent x1e3 outliers); "
                                     "affine_relu and pipeline_sum at 2^"
                                     + ", 2^".join(str(k) for k in args.strong_sizes)
                                     + " (U(-1,1))",
                         "l2": "write-then-read 512 MiB flush before every timed call"},
              "checks_passed": bool(all_ok), "points": points})
    if comm is not None:
        comm.check()
        comm.destroy()
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    if not all_ok:
        sys.exit(1)


def run_single(args) -> None:
    """One suite entry at N=2^--n-log2 on one GPU, --steps bound calls after
    --warmup on the suite's seeded inputs: the small, bounded command that
    an ncu capture of one kernel runs.  Prints one JSON line with the median
    device time per call (CUDA events; no L2 flush)."""
    import torch
    from loom_b200.build import load_suite
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    pkg = load_suite()
    entry = args.single
    n = 1 << args.n_log2
    data = make_inputs(n, 0)
    kw = {p: data[t] for p, t in zip(PARAM_NAMES[entry], TENSORS[entry])}
    kw.update(SCALARS.get(entry, {}))
    for k in list(data):
        if k not in TENSORS[entry]:
            del data[k]
    out = torch.empty(n if entry in MAP_ENTRIES else 1, device="cuda")
    stream = torch.cuda.current_stream()
    call, _ = pkg[entry].bind(out=out, stream=stream, **kw)
    for _ in range(args.warmup):
        call()
    torch.cuda.synchronize()
    times = []
    for _ in range(args.steps):
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        call()
        b.record(stream)
        b.synchronize()
        times.append(a.elapsed_time(b) * 1e3)
    us = statistics.median(times)
    emit({"mode": "single", "entry": entry, "n": n, "calls": args.steps,
          "us_per_call": round(us, 2),
          "gbs": round(bytes_per_elem(entry) * n / (us * 1e-6) / 1e9, 1)})


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--n-log2", type=int, default=28)
    ap.add_argument("--e2e-steps", type=int, default=2)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--exchange", choices=["peer", "nccl"], default="peer",
                    help="scalar exchange of the reductions across GPUs: peer memory "
                         "(where every GPU reaches the others) or NCCL")
    ap.add_argument("--ref-kernel-steps", type=int, default=30,
                    help="steps of the reference-style GPU kernels (1 GPU; 0 skips them)")
    ap.add_argument("--cpu-log2", type=int, default=28,
                    help="N=2^k per entry of the CPU baseline's sample (default: the GPU "
                         "arm's per-GPU N)")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--pipeline-sweep", action="store_true",
                    help="time the fused pipeline over --sweep sizes instead of the suite step")
    ap.add_argument("--sweep", type=int, nargs="*", default=[10, 14, 18, 22, 26, 30, 32])
    ap.add_argument("--config-sweep", action="store_true",
                    help="time each single-entry configuration at its own N instead of the step")
    ap.add_argument("--single", choices=ENTRIES,
                    help="time one entry at N=2^--n-log2 (--steps calls after --warmup)")
    ap.add_argument("--strong", action="store_true",
                    help="strong scaling: fixed global sizes sharded over the ranks")
    ap.add_argument("--strong-sizes", type=int, nargs="*", default=[18, 22, 26, 30, 32],
                    help="log2 of the pipeline's global N in --strong mode")
    ap.add_argument("--workload-sweep", action="store_true",
                    help="time the reference harness's 33 kernels at the --sweep sizes")
    ap.add_argument("--workload-package", default="workloads",
                    choices=["workloads", "workloads_flags", "workloads_cuda_fixed"],
                    help="which build of the harness's kernels --workload-sweep times")
    args = ap.parse_args()
    protect_stdout()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.single:
        run_single(args)
        return
    if args.strong:
        run_strong(args)
        return
    if args.config_sweep:
        run_config_sweep(args)
        return
    if args.workload_sweep:
        run_workload_sweep(args)
        return
    if args.pipeline_sweep:
        run_pipeline_sweep(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
