"""The stream entries under CUDA graph capture and on concurrent streams.

* Graph capture: every suite entry, bound once (`Entry.bind`) to a side
  stream, is captured into one CUDA graph -- programmatic dependent launches,
  cluster launches and finalize kernels included -- and the replayed graph
  must give the same bits as the eager calls.
* Concurrency: the entries hold no state between calls, and the loader keeps
  one cached workspace per stream, so the same entries launched through one
  Package on several streams at once must give the same bits as one after
  another.
"""

import numpy as np
import pytest
import torch

from loom_b200 import workloads
from loom_b200.build import load_suite

from test_gpu_parity import to_device

pytestmark = pytest.mark.gpu

ENTRIES = ["saxpy", "relu", "dot", "l2_norm_sq", "max_value", "affine_relu", "pipeline_sum"]


def _inputs(n, seed):
    return {e: {k: (to_device(v) if isinstance(v, np.ndarray) else v)
                for k, v in workloads.entry_inputs(e, n, seed_offset=seed).items()}
            for e in ENTRIES}


@pytest.mark.parametrize("n", [3, 5000, (1 << 18) + 5])
def test_graph_replay_matches_eager(n):
    pkg = load_suite()
    inputs = _inputs(n, seed=n)
    eager = {e: pkg[e](**inputs[e]).cpu().numpy() for e in ENTRIES}
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    bound = {e: pkg[e].bind(stream=side, **inputs[e]) for e in ENTRIES}
    graph = torch.cuda.CUDAGraph()
    torch.cuda.synchronize()
    with torch.cuda.graph(graph, stream=side):
        for e in ENTRIES:
            bound[e][0]()
    for out in (o for _, o in bound.values()):
        out.zero_()
    torch.cuda.synchronize()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    for e in ENTRIES:
        got = bound[e][1].cpu().numpy()
        assert np.array_equal(got.view(np.uint32), eager[e].view(np.uint32)), (e, n)


def test_concurrent_streams_match_serial():
    pkg = load_suite()
    n = (1 << 20) + 7
    streams = [torch.cuda.Stream() for _ in range(4)]
    sets = [_inputs(n, seed=100 + i) for i in range(len(streams))]
    serial = [{e: pkg[e](**s[e]).cpu().numpy() for e in ENTRIES} for s in sets]
    torch.cuda.synchronize()
    # one Package for all streams: its cached workspaces are per stream
    calls = [[pkg[e].bind(stream=s, **ins[e]) for e in ENTRIES]
             for s, ins in zip(streams, sets)]
    torch.cuda.synchronize()
    for _ in range(3):
        for per_stream in calls:
            for call, _ in per_stream:
                call()
    torch.cuda.synchronize()
    for i, per_stream in enumerate(calls):
        for e, (_, out) in zip(ENTRIES, per_stream):
            got = out.cpu().numpy()
            assert np.array_equal(got.view(np.uint32), serial[i][e].view(np.uint32)), (i, e)
