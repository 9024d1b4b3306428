"""The workload configurations at their full sizes.

Up to N = 2^30 the CUDA results are compared with the oracle on the seeded
inputs (same bar as test_gpu_parity).  At N = 2^30 and 2^32 for the pipeline
entries (inputs of 4 and 16 GiB each) the check is size-independent: inputs
built on the device from constants plus a few spikes placed across the 2^31
and 2^32 index boundaries, whose exact results are known in closed form --
this exercises 64-bit indexing and the ragged tail at the largest sizes.
"""

import math

import numpy as np
import pytest
import torch

from loom_b200 import workloads

from test_gpu_parity import MAPS, assert_bits, check_sum

pytestmark = pytest.mark.gpu


def _device_inputs(inp):
    return {k: (torch.from_numpy(v).cuda() if isinstance(v, np.ndarray) else v)
            for k, v in inp.items()}


@pytest.mark.parametrize("config", [c for c in workloads.CONFIGS], ids=lambda c: c.name)
def test_config_full_size(suite_pkg, oracle, config):
    n = config.n
    for entry in config.entries:
        inp = workloads.entry_inputs(entry, n)
        ref = oracle.run(entry, inp)
        dev = _device_inputs(inp)
        got = suite_pkg[entry](**dev)
        torch.cuda.synchronize()
        if entry in MAPS:
            assert_bits(got.cpu().numpy(), ref)
        elif entry == "max_value":
            assert float(got.cpu()[0]) == float(np.float32(ref))
        else:
            check_sum(entry, float(got.cpu()[0]), ref, inp, n)
        del dev, got


@pytest.mark.parametrize("n", [1 << 26, 1 << 28])
def test_pipeline_sweep_vs_oracle(suite_pkg, oracle, n):
    inp = workloads.entry_inputs("pipeline_sum", n, seed_offset=n)
    dev = _device_inputs(inp)
    z = suite_pkg["affine_relu"](x=dev["x"], y=dev["y"], a=0.75)
    s = suite_pkg["pipeline_sum"](**dev)
    torch.cuda.synchronize()
    assert_bits(z.cpu().numpy(), oracle.run("affine_relu", {k: inp[k] for k in ("a", "x", "y")}))
    check_sum("pipeline_sum", float(s.cpu()[0]), oracle.run("pipeline_sum", inp), inp, n)


@pytest.mark.parametrize("n", [(1 << 30) + 7, 1 << 32])
def test_pipeline_huge_closed_form(suite_pkg, n):
    spikes = [0, 1, (1 << 31) - 1, 1 << 31, (1 << 31) + 3, n - 5, n - 1]
    spikes = sorted({k for k in spikes if k < n})
    x = torch.ones(n, dtype=torch.float32, device="cuda")
    y = torch.full((n,), -0.5, dtype=torch.float32, device="cuda")
    w = torch.ones(n, dtype=torch.float32, device="cuda")
    idx = torch.tensor(spikes, dtype=torch.int64, device="cuda")
    x[idx] = 3.0  # z = relu(0.75*3 - 0.5) = 1.75 there, 0.25 elsewhere
    z = suite_pkg["affine_relu"](x=x, y=y, a=0.75)
    s = suite_pkg["pipeline_sum"](x=x, y=y, w=w, a=0.75)
    torch.cuda.synchronize()
    assert int((z == 0.25).sum().item()) == n - len(spikes)
    assert torch.all(z[idx] == 1.75).item()
    exact = 0.25 * (n - len(spikes)) + 1.75 * len(spikes)
    assert float(s.item()) == float(np.float32(exact))
    del z
    mx = suite_pkg["max_value"](x=y.index_fill_(0, idx[-1:], 9.0))
    torch.cuda.synchronize()
    assert float(mx.item()) == 9.0
    sq = suite_pkg["l2_norm_sq"](x=w.fill_(0.5))
    torch.cuda.synchronize()
    assert float(sq.item()) == float(np.float32(0.25 * n))
