"""Entry.call_host: the public host-buffer call (pinned or pageable host
inputs, host result).  Maps are streamed in chunks through two device slots
on two streams, so the test uses small chunks to cycle the slots many times
and a ragged last chunk; results must match the oracle with the bar of
test_gpu_parity."""

import numpy as np
import pytest
import torch

from loom_b200 import workloads

from test_gpu_parity import MAPS, assert_bits, check_sum

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("entry", ["saxpy", "relu", "affine_relu", "dot", "max_value",
                                   "pipeline_sum"])
@pytest.mark.parametrize("pinned", [True, False])
def test_call_host_matches_oracle(suite_pkg, oracle, entry, pinned):
    n = 5 * 65536 + 13
    inp = workloads.entry_inputs(entry, n, seed_offset=77)
    ref = oracle.run(entry, inp)
    host = {}
    for k, v in inp.items():
        if isinstance(v, np.ndarray):
            t = torch.from_numpy(v)
            host[k] = t.pin_memory() if pinned else t
        else:
            host[k] = v
    got = suite_pkg[entry].call_host(chunk_elems=65536, **host).numpy()
    if entry in MAPS:
        assert_bits(got, ref)
    elif entry == "max_value":
        assert float(got[0]) == float(np.float32(ref))
    else:
        check_sum(entry, float(got[0]), ref, inp, n)


def test_call_host_repeated_and_resized(suite_pkg, oracle):
    e = suite_pkg["saxpy"]
    for n in (1 << 20, 1000, (1 << 20) + 7):
        inp = workloads.entry_inputs("saxpy", n, seed_offset=n)
        got = e.call_host(chunk_elems=1 << 18, **{k: (torch.from_numpy(v) if isinstance(
            v, np.ndarray) else v) for k, v in inp.items()}).numpy()
        assert_bits(got, oracle.run("saxpy", inp))
