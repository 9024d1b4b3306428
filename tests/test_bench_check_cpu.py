"""bench.py's results check across ranks (check_results), on 2 gloo ranks on
the CPU: outputs computed independently (maps with an exact fmaf, sums in
fp64 all-reduced) pass; a map element one ulp off on one rank, a sum off by
far more than the bar, and ranks that disagree on a reduction each fail it."""

import multiprocessing as mp
import os
import socket
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, plant, q):
    import datetime

    import torch
    import torch.distributed as dist
    sys.path.insert(0, ROOT)
    import bench
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        n = 5000
        g = torch.Generator().manual_seed(100 + rank)
        data = {k: torch.rand(n, generator=g) * 2 - 1 for k in ("u0", "u1", "u2")}
        data["nrm"] = torch.randn(n, generator=g)
        outl = torch.randn(n, generator=g)
        outl[::97] *= 1e3
        data["outl"] = outl
        x, y = data["u0"].numpy(), data["u1"].numpy()
        outs = {"saxpy": torch.from_numpy(bench.fmaf_f32(2.5, x, y)),
                "relu": torch.where(data["nrm"] > 0, data["nrm"], torch.zeros(n))}
        z = bench.fmaf_f32(0.75, x, y)
        outs["affine_relu"] = torch.from_numpy(np.where(z > 0, z, np.float32(0.0)))
        sums = torch.stack([bench._sum_values(e, data, 0, n).double().sum()
                            for e in ("dot", "l2_norm_sq", "pipeline_sum")])
        dist.all_reduce(sums)
        mx = data["outl"].max().reshape(1)
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        for e, v in zip(("dot", "l2_norm_sq", "pipeline_sum"), sums.tolist()):
            outs[e] = torch.tensor([v], dtype=torch.float32)
        outs["max_value"] = mx.clone()
        if plant == "map_ulp" and rank == 1:
            outs["saxpy"][123] = torch.from_numpy(np.nextafter(outs["saxpy"][123:124].numpy(),
                                                               np.float32(np.inf)))
        if plant == "sum_off":
            outs["dot"] *= 1.001
        if plant == "ranks_disagree" and rank == 1:
            outs["l2_norm_sq"] = torch.from_numpy(np.nextafter(outs["l2_norm_sq"].numpy(),
                                                               np.float32(np.inf)))
        res = bench.check_results(data, outs, n, world, rank, device="cpu")
        if rank == 0:
            q.put(res)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("plant", [None, "map_ulp", "sum_off", "ranks_disagree"])
def test_check_leg_on_two_ranks(plant):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, plant, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        res = q.get(timeout=120)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert all(p.exitcode == 0 for p in procs)
    if plant is None:
        assert res["passed"], res
    else:
        assert not res["passed"], (plant, res)
    if plant == "map_ulp":
        assert res["maps_bit_exact"] == {"saxpy": False, "relu": True, "affine_relu": True}
    if plant == "sum_off":
        assert not res["dot"]["passed"] and res["l2_norm_sq"]["passed"]
    if plant == "ranks_disagree":
        assert not res["reductions_identical_on_every_rank"]
