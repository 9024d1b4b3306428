"""Multi-GPU entries against the oracle on the full (unsharded) input.

* `_multi`: one process drives every visible GPU (up to 8), one contiguous
  shard per device (`loom_b200.shard.shard_bounds`); reductions exchange
  their scalar through peer memory or, switched, one grouped NCCL
  collective.
* `_dist`: one process per GPU (2 ranks), the communicator's id rendezvoused
  over a gloo process group; every reduction runs through both exchange
  paths, which must give the same bits.
* A bounded wait: a reduction launched on one rank only must give up after
  its time limit, report it through `Comm.check`, and return NaN, leaving
  the GPU usable.

Maps must reproduce the oracle bit for bit once the shards are concatenated;
reductions must give the same bits on every device, max exactly and sums to
the bar of test_gpu_parity.  Skipped with fewer than 2 GPUs.
"""

import math
import multiprocessing as mp
import os
import socket

import numpy as np
import pytest
import torch

from loom_b200 import workloads
from loom_b200.shard import shard_bounds

from test_gpu_parity import MAPS, check_sum

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")]

ENTRIES = ["saxpy", "relu", "affine_relu", "dot", "l2_norm_sq", "max_value", "pipeline_sum"]


def _check(entry, results, ref, full, n):
    if entry in MAPS:
        got = np.concatenate(results)
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), entry
        return
    bits = {np.float32(r).view(np.uint32).item() for r in results}
    assert len(bits) == 1, (entry, results)       # every device holds the same value
    got = float(results[0])
    if entry == "max_value":
        assert got == float(np.float32(ref))
    else:
        check_sum(entry, got, ref, full, n)


@pytest.mark.parametrize("exchange", ["peer", "nccl"])
@pytest.mark.parametrize("n", [(1 << 22) + 3, 37, 3])
def test_multi_one_process(suite_pkg, oracle, n, exchange):
    devs = list(range(min(torch.cuda.device_count(), 8)))
    comms = suite_pkg.comm_init_all(devs)
    try:
        assert all(c.peer_exchange for c in comms)    # NVLink: every pair reaches the others
        for c in comms:
            c.set_peer_exchange(exchange == "peer")
        bounds = shard_bounds(n, len(devs))
        for entry in ENTRIES:
            full = workloads.entry_inputs(entry, n, seed_offset=len(devs))
            shards = [{k: (torch.from_numpy(np.ascontiguousarray(v[s:e])).to(f"cuda:{d}")
                           if isinstance(v, np.ndarray) else v) for k, v in full.items()}
                      for d, (s, e) in zip(devs, bounds)]
            outs, host = suite_pkg[entry].multi(comms, shards)
            for d in devs:
                torch.cuda.synchronize(d)
            results = [o.cpu().numpy() if entry in MAPS else float(o.cpu()[0]) for o in outs]
            _check(entry, results, oracle.run(entry, full), full, n)
            if entry not in MAPS:
                assert host == results[0]
        for c in comms:
            c.check()
            stats = c.exchange_stats(reset=True)
            # every reduction exchanged once per device on the peer path
            assert stats["exchanges"] == (4 if exchange == "peer" else 0), stats
            assert stats["max_us"] >= stats["total_us"] / max(1, stats["exchanges"])
    finally:
        for c in comms:
            c.destroy()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _dist_rank(rank, world, port, n, queue):
    import datetime

    import torch.distributed as dist

    from loom_b200.build import load_suite
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    comm = None
    try:
        pkg = load_suite()
        comm = pkg.comm_from_process_group()
        assert comm.peer_exchange
        start, stop = shard_bounds(n, world)[rank]
        for entry in ENTRIES:
            full = workloads.entry_inputs(entry, n, seed_offset=world + 100)
            mine = {k: (torch.from_numpy(np.ascontiguousarray(v[start:stop])).cuda()
                        if isinstance(v, np.ndarray) else v) for k, v in full.items()}
            runs = []
            for peer in (True, False, True):
                comm.set_peer_exchange(peer)
                out = pkg[entry].dist(comm, **mine)
                torch.cuda.synchronize()
                runs.append(out.cpu().numpy())
            comm.check()
            # the same bits through peer memory, NCCL, and peer memory again
            assert all(np.array_equal(r.view(np.uint32), runs[0].view(np.uint32))
                       for r in runs), entry
            res = runs[0] if entry in MAPS else float(runs[0][0])
            gathered = [None] * world
            dist.all_gather_object(gathered, res)
            if rank == 0:
                queue.put((entry, gathered))
    finally:
        if comm is not None:
            comm.destroy()
        dist.destroy_process_group()


def test_dist_one_process_per_gpu(oracle):
    world, n = 2, (1 << 21) + 5
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dist_rank, args=(r, world, port, n, queue)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        got = dict(queue.get(timeout=300) for _ in ENTRIES)
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    assert all(p.exitcode == 0 for p in procs)
    for entry in ENTRIES:
        full = workloads.entry_inputs(entry, n, seed_offset=world + 100)
        _check(entry, got[entry], oracle.run(entry, full), full, n)


@pytest.mark.parametrize("n", [4096, 1 << 20])
def test_exchange_wait_is_bounded(suite_pkg, n):
    # Only device 0 takes part: its exchange waits for a value that nobody
    # sends, gives up after its time limit (1 s here), records the failure
    # and returns NaN.  The device stays usable.  n = 4096 is a one-cluster
    # grid followed by the exchange kernel; n = 2^20 is a grid of 512 CTAs
    # followed by the finalize CTA that runs the exchange.
    comms = suite_pkg.comm_init_all([0, 1])
    try:
        assert comms[0].peer_exchange
        comms[0].set_timeout_ms(1000)
        x = torch.ones(n, device="cuda:0")
        with torch.cuda.device(0):
            out = suite_pkg["dot"].dist(comms[0], x=x, y=x)
            torch.cuda.synchronize()
        assert np.isnan(float(out.cpu()[0]))
        with pytest.raises(Exception) as info:
            comms[0].check()
        assert info.value.status == 4          # LOOM_STATUS_COMM_ERROR
        assert float(suite_pkg["dot"](x=x, y=x).cpu()[0]) == float(n)
    finally:
        for c in comms:
            c.destroy()
