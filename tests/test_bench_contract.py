"""bench.py's output contract: one JSON line on stdout with the keys the
benchmark driver reads, for the reference arm (CPU, here) and the product
arm (GPU, small N); the non-zero ranks of the reference arm print nothing;
the clock summary keeps only samples inside the timed region and reports the
throttle reasons seen there."""

import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402

BASE_KEYS = {"metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
             "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config"}


def _run(args, env=None, timeout=600):
    proc = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py")] + args,
                          capture_output=True, text=True, timeout=timeout,
                          env=dict(os.environ, **(env or {})))
    return proc


def test_reference_arm_prints_one_json_line():
    proc = _run(["--impl", "reference", "--steps", "2", "--warmup", "3", "--n-log2", "12"])
    assert proc.returncode == 0, proc.stderr
    lines = [line for line in proc.stdout.splitlines() if line.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert BASE_KEYS <= set(d)
    assert d["impl"] == "reference" and d["steps"] == 2 and d["warmup"] == 3
    assert d["value"] > 0 and d["unit"] == "GB/s" and d["higher_is_better"] is True
    assert {"value", "unit", "cores", "kind", "sample"} <= set(d["cpu_baseline"])
    assert d["cpu_baseline"]["kind"] == "port"
    assert d["e2e"] == {"value": d["value"], "unit": "GB/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}
    # the same workload description as the GPU arm's line
    assert d["config"] == bench.suite_config(1, 12)


def test_reference_arm_other_ranks_print_nothing():
    proc = _run(["--impl", "reference", "--steps", "1", "--warmup", "3", "--n-log2", "10"],
                env={"RANK": "1", "WORLD_SIZE": "2"})
    assert proc.returncode == 0, proc.stderr
    assert proc.stdout.strip() == ""


def test_warmup_below_three_is_refused():
    proc = _run(["--impl", "reference", "--steps", "1", "--warmup", "2"])
    assert proc.returncode != 0


def test_launch_counts():
    n = 1 << 28
    assert [bench.launches_per_call(e, 1, n) for e in bench.ENTRIES] == [1, 1, 2, 2, 2, 1, 2]
    assert [bench.launches_per_call(e, 4, n, peer=False) for e in bench.ENTRIES] == \
        [1, 1, 3, 3, 2, 1, 3]
    assert [bench.launches_per_call(e, 4, n, peer=True) for e in bench.ENTRIES] == \
        [1, 1, 2, 2, 2, 1, 2]
    assert all(bench.launches_per_call(e, 1, 4096) == 1 for e in bench.ENTRIES)


def test_fmaf_f32_is_correctly_rounded():
    # against exact rational arithmetic, on random operands and on operands
    # built so that a*x + y falls next to the midpoint of two float32 values
    from fractions import Fraction

    import numpy as np

    def round32(q):
        f = np.float32(float(q))
        cands = [f, np.nextafter(f, np.float32(np.inf)), np.nextafter(f, np.float32(-np.inf))]
        return min(cands, key=lambda c: (abs(Fraction(float(c)) - q),
                                         int(np.array(c).view(np.uint32)) & 1))

    rng = np.random.default_rng(5)
    x = list(rng.uniform(-1, 1, 300).astype(np.float32))
    y = list(rng.uniform(-1, 1, 300).astype(np.float32))
    for k in range(1, 60):
        for sh in (24, 25, 26):
            x.append(np.float32(1 + k * 2.0 ** -23))
            y.append(np.float32(3 * 2.0 ** -sh) * (1 if k % 2 else -1))
    x, y = np.array(x, np.float32), np.array(y, np.float32)
    for a in (2.5, 0.75, 1.0, 3.0):
        got = bench.fmaf_f32(a, x, y)
        for i in range(len(x)):
            q = Fraction(float(np.float32(a))) * Fraction(float(x[i])) + Fraction(float(y[i]))
            want = round32(q)
            assert np.array(got[i]).view(np.uint32) == np.array(want).view(np.uint32), (a, i)


def test_cpu_inputs_are_the_entries_inputs():
    import numpy as np

    from loom_b200 import workloads
    shared = bench.cpu_suite_inputs(1000)
    for e in bench.ENTRIES:
        want = workloads.entry_inputs(e, 1000)
        assert set(shared[e]) == set(want)
        for k, v in want.items():
            if isinstance(v, np.ndarray):
                assert np.array_equal(shared[e][k], v), (e, k)
            else:
                assert shared[e][k] == v


@pytest.mark.parametrize("kind", ["uniform", "normal_outliers"])
def test_strong_inputs_do_not_depend_on_the_sharding(kind):
    # the strong-scaling mode draws the global input in fixed chunks, so the
    # ranks' shards concatenate to the same array for every world size
    import torch

    from loom_b200.shard import shard_bounds
    n, chunk = 10007, 1000
    whole = bench.global_slice(kind, 5, 0, n, chunk=chunk, device="cpu")
    for world in (1, 2, 3, 4, 8):
        parts = [bench.global_slice(kind, 5, a, b, chunk=chunk, device="cpu")
                 for a, b in shard_bounds(n, world)]
        assert torch.equal(torch.cat(parts), whole), world
    if kind == "normal_outliers":
        assert (whole.abs() > 50).sum() > 0          # the 1% of outliers are there


class _FakeProc:
    def terminate(self):
        pass

    def wait(self, timeout=None):
        return 0


def test_clock_summary_keeps_only_the_timed_region():
    s = bench.ClockSampler("0")
    s.proc = _FakeProc()
    row = "0, {sm}, 1965, 700.0, 0x0, {hw}, Not Active, Not Active, {cap}\n"
    s.lines = [(1.0, row.format(sm=900, hw="Active", cap="Not Active")),     # before
               (10.0, row.format(sm=1800, hw="Not Active", cap="Active")),
               (11.0, row.format(sm=1850, hw="Not Active", cap="Not Active")),
               (12.0, row.format(sm=1900, hw="Not Active", cap="Active")),
               (30.0, row.format(sm=800, hw="Active", cap="Not Active"))]    # after
    s.t0, s.t1 = 9.5, 12.5
    c = s.stop()
    assert c["sm_mhz"] == 1850 and c["sm_max_mhz"] == 1965 and c["samples"] == 3
    assert c["reasons"] == ["sw_power_cap"]


@pytest.mark.gpu
def test_product_arm_prints_one_json_line():
    proc = _run(["--steps", "5", "--warmup", "3", "--n-log2", "20", "--no-cpu",
                 "--e2e-steps", "1", "--ref-kernel-steps", "2"])
    assert proc.returncode == 0, proc.stderr[-2000:]
    lines = [line for line in proc.stdout.splitlines() if line.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert BASE_KEYS <= set(d)
    assert d["n_gpus"] == 1 and d["scaling"] == "weak" and d["dtype"] == "f32"
    assert {"bound", "achieved", "peak", "unit", "frac", "traffic"} <= set(d["roofline"])
    assert {"sm_mhz", "sm_max_mhz", "reasons"} <= set(d["clocks"])
    assert d["gpu_launches"] == 5 * sum(bench.launches_per_call(e, 1, 1 << 20)
                                        for e in bench.ENTRIES)
    assert {"value", "unit", "h2d_bytes_per_step", "d2h_bytes_per_step"} <= set(d["e2e"])
    assert d["e2e"]["h2d_bytes_per_step"] > 0
    assert d["check"]["passed"], d["check"]
    assert d["config"] == bench.suite_config(1, 20)
    for profile in ("none", "cuda"):
        ref = d["reference_kernels"]["profiles"][profile]
        assert all(ref["agrees_with_product"].values()), (profile, ref["agrees_with_product"])
