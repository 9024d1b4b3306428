"""Reductions over grids of every shape, and the caller's workspace.

A reduction of more than 8 CTAs writes one partial per CTA into the caller's
workspace and a finalize CTA folds them.  Against the CPU oracle (max
bit-exact, sums within 1e-6 * max(1, log2 n) * |ref|):

* grid sizes 9 (the smallest two-launch grid), 255-257, 4097, and 32768 and
  more tiles (the partial-slot cap, where CTAs take several tiles), aligned
  and with a 3-element head;
* 889-3553 tiles, where a grid of one to three waves of resident CTAs runs
  as one wave with several tiles per CTA (on a B200, 888 resident CTAs of
  the two- and three-input kernels, 1184 of the one-input ones), around
  both ends of that range; and the number of partials such a call writes;
* workspaces filled beforehand with zeros, ones, 0xff bytes and random
  bytes: nothing in a workspace has to start at any value;
* one workspace reused by calls of different sizes and entries: a call
  reads only the partials it wrote;
* determinism: the same inputs give the same bits.
"""

import ctypes
import math

import numpy as np
import pytest
import torch

from loom_b200 import workloads
from test_gpu_parity import check_sum, to_device

pytestmark = pytest.mark.gpu


def tile_of(entry):
    return 4096 if entry in ("l2_norm_sq", "max_value") else 2048


def check(entry, got, ref, inp, n):
    if entry == "max_value":
        assert got == float(np.float32(ref)), (entry, n, got, ref)
    else:
        check_sum(entry, got, ref, inp, n)


def call_with_workspace(pkg, entry, dev, ws):
    """The synchronous reference entry through the C ABI with the caller's
    workspace `ws` (a uint8 device tensor)."""
    e = pkg[entry]
    out = torch.full((1,), float("nan"), device="cuda")
    args = []
    for p in e.params:
        v = dev[p["name"]]
        args.append(ctypes.c_float(v) if p["kind"] == "scalar-f32"
                    else ctypes.c_void_p(v.data_ptr()))
    n = next(v.shape[0] for v in dev.values() if isinstance(v, torch.Tensor))
    st = e.call_raw(*args, ctypes.c_int64(n), ctypes.c_void_p(out.data_ptr()),
                    ctypes.c_void_p(ws.data_ptr()), ctypes.c_size_t(ws.numel()))
    assert st == 0, (entry, n, st)
    return float(out.cpu()[0])


@pytest.mark.parametrize("entry", ["dot", "l2_norm_sq", "max_value", "pipeline_sum"])
def test_grid_sizes(suite_pkg, oracle, entry):
    tile = tile_of(entry)
    sizes = [(9, 0), (9, 5), (255, 1), (256, 0), (256, 1), (257, 0), (4097, 3),
             (889, 0), (1185, 3), (1777, 0), (2048, 1), (2665, 0), (3552, 0), (3553, 2)]
    if entry in ("dot", "l2_norm_sq"):
        sizes += [(32768, 0), (32769, 0), (3 * 32768 + 5, 7)]
    for g, d in sizes:
        n = g * tile + d
        for offset in (0, 3):
            inp = workloads.entry_inputs(entry, n, seed_offset=g + d + offset)
            ref = oracle.run(entry, inp)
            dev = {k: (to_device(v, offset) if isinstance(v, np.ndarray) else v)
                   for k, v in inp.items()}
            got = float(suite_pkg[entry](**dev).cpu()[0])
            check(entry, got, ref, inp, n)


def balanced_grid(tiles, wave):
    """The launcher's grid for a reduction of `tiles` tiles on a device that
    holds `wave` of its CTAs at once (loom_b200_launch.cuh)."""
    if tiles <= wave or tiles > 3 * wave:
        return tiles
    per_cta = -(-tiles // wave)
    return -(-tiles // per_cta)


def test_mid_grids_run_as_one_wave(suite_pkg, oracle):
    # The stage writes one partial per CTA (fp64 for sums, fp32 for max) at
    # the start of the workspace (its first 256-byte boundary); in a workspace
    # of 0xff bytes the slots it wrote are the ones that changed, and they
    # must be the grid's prefix.
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    for entry, tiles in (("dot", 2048), ("pipeline_sum", 2048), ("l2_norm_sq", 2000),
                         ("max_value", 3000)):
        n = tiles * tile_of(entry) + 1
        inp = workloads.entry_inputs(entry, n, seed_offset=tiles)
        dev = {k: (to_device(v) if isinstance(v, np.ndarray) else v) for k, v in inp.items()}
        ws = _workspace(suite_pkg, entry, n, "ff")
        check(entry, call_with_workspace(suite_pkg, entry, dev, ws), oracle.run(entry, inp),
              inp, n)
        base = (-ws.data_ptr()) % 256
        slot = np.uint32 if entry == "max_value" else np.uint64
        raw = ws.cpu().numpy()[base:]
        slots = raw[:len(raw) // slot().itemsize * slot().itemsize].view(slot)
        written = np.flatnonzero(slots != np.iinfo(slot).max)
        grid = len(written)
        assert np.array_equal(written, np.arange(grid)), (entry, grid)
        # `tiles` whole tiles (the one extra element is the scalar tail), two
        # or three per CTA
        assert grid < tiles, (entry, grid)
        assert grid in {balanced_grid(tiles, sms * k) for k in range(1, 9)}, (entry, grid)


def _workspace(pkg, entry, n, fill):
    size = pkg[entry].workspace_size(n)
    ws = torch.empty(size, dtype=torch.uint8, device="cuda")
    if fill == "zeros":
        ws.zero_()
    elif fill == "ones":
        ws.fill_(1)
    elif fill == "ff":
        ws.fill_(255)
    elif fill == "random":
        g = torch.Generator(device="cuda")
        g.manual_seed(12345)
        ws.copy_(torch.randint(0, 256, (size,), dtype=torch.uint8, device="cuda", generator=g))
    return ws


@pytest.mark.parametrize("fill", ["zeros", "ones", "ff", "random"])
def test_any_prior_workspace_contents(suite_pkg, oracle, fill):
    n = 1000 * 2048 + 7            # 1001 tiles of a two-input reduction
    inp = workloads.entry_inputs("dot", n, seed_offset=77)
    ref = oracle.run("dot", inp)
    dev = {k: to_device(v) for k, v in inp.items()}
    ws = _workspace(suite_pkg, "dot", n, fill)
    for _ in range(3):
        check("dot", call_with_workspace(suite_pkg, "dot", dev, ws), ref, inp, n)


def test_reused_workspace(suite_pkg, oracle):
    # one workspace, calls that alternate between grids and entries: each call
    # must read only the partials it wrote, never one left by an earlier call
    big = 4096 * 2048 - 5
    ws = _workspace(suite_pkg, "dot", big, "random")
    cases = []
    for k, n in enumerate([big, 300 * 2048, 9 * 2048 + 1, 4000 * 2048, 17 * 2048]):
        entry = "dot" if k % 2 == 0 else "pipeline_sum"
        inp = workloads.entry_inputs(entry, n, seed_offset=500 + k)
        cases.append((entry, n, inp, oracle.run(entry, inp),
                      {kk: (to_device(v) if isinstance(v, np.ndarray) else v)
                       for kk, v in inp.items()}))
    for _ in range(2):
        for entry, n, inp, ref, dev in cases:
            assert suite_pkg[entry].workspace_size(n) <= ws.numel()
            check(entry, call_with_workspace(suite_pkg, entry, dev, ws), ref, inp, n)


def test_reductions_are_deterministic_over_grids(suite_pkg):
    for entry, n in (("dot", 2047 * 2048 + 3), ("l2_norm_sq", 1500 * 4096 + 1),
                     ("pipeline_sum", 3000 * 2048)):
        inp = workloads.entry_inputs(entry, n, seed_offset=11)
        dev = {k: (to_device(v, 1) if isinstance(v, np.ndarray) else v) for k, v in inp.items()}
        a = suite_pkg[entry](**dev).cpu().numpy()
        b = suite_pkg[entry](**dev).cpu().numpy()
        assert a.view(np.uint32)[0] == b.view(np.uint32)[0]
        assert not math.isnan(float(a[0]))
