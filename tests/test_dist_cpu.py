"""Multi-rank host logic on CPU (gloo, world size 2): shard planning, the
rendezvous of the communicator id, and the rank-ordered fold of per-rank
fp64 partials that the `_dist` / `_multi` entries perform on the GPU.
The per-shard values come from the oracle; no GPU is involved."""

import math
import multiprocessing as mp
import os
import socket

import numpy as np
import pytest

from loom_b200 import workloads
from loom_b200.shard import shard_bounds

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SUITE_IR = os.path.join(ROOT, "oracle", "suite_kernels.tensor_ir.json")
N = 100_003


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, queue):
    import torch.distributed as dist

    from oracle.loom_oracle import Oracle, load_programs
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        oracle = Oracle(load_programs(SUITE_IR), name="b200_suite")
        # rendezvous of an opaque communicator id, as Package.comm_from_process_group does
        box = [bytes(range(128)) if rank == 0 else None]
        dist.broadcast_object_list(box, src=0)
        assert box[0] == bytes(range(128))
        result = {}
        for entry in ("dot", "l2_norm_sq", "pipeline_sum", "max_value", "saxpy"):
            full = workloads.entry_inputs(entry, N)
            start, stop = shard_bounds(N, world)[rank]
            mine = {k: (v[start:stop] if isinstance(v, np.ndarray) else v) for k, v in full.items()}
            if stop > start:
                local = oracle.run(entry, mine)
            else:
                local = -math.inf if entry == "max_value" else 0.0
            gathered = [None] * world
            dist.all_gather_object(gathered, local)
            if entry == "saxpy":
                result[entry] = np.concatenate(gathered)
            elif entry == "max_value":
                result[entry] = max(gathered)
            else:
                acc = 0.0
                for v in gathered:          # rank order, as rank_combine_kernel folds
                    acc += v
                result[entry] = acc
        if rank == 0:
            queue.put(result)
    finally:
        dist.destroy_process_group()


def test_two_rank_shard_and_fold(oracle):
    world = 2
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    result = queue.get(timeout=240)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for entry in ("dot", "l2_norm_sq", "pipeline_sum"):
        ref = oracle.run(entry, workloads.entry_inputs(entry, N))
        assert result[entry] == pytest.approx(ref, rel=1e-12)
    ref_max = oracle.run("max_value", workloads.entry_inputs("max_value", N))
    assert result["max_value"] == ref_max
    ref_map = oracle.run("saxpy", workloads.entry_inputs("saxpy", N))
    assert np.array_equal(result["saxpy"].view(np.uint32), ref_map.view(np.uint32))


@pytest.mark.parametrize("n", [0, 1, 3, 4, 5, 17, 4099, 1 << 20, (1 << 28) + 3])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shard_bounds_cover_and_align(n, world):
    b = shard_bounds(n, world)
    assert len(b) == world and b[0][0] == 0 and b[-1][1] == n
    assert all(b[i][1] == b[i + 1][0] for i in range(world - 1))
    assert all(start % 4 == 0 for start, stop in b if stop > start)
    sizes = [stop - start for start, stop in b]
    assert max(sizes) - min(sizes) <= 7  # one 4-element unit, plus a partial last unit
