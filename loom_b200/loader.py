"""Thin ctypes / PyTorch host loader over a generated package's C ABI.

Mirrors the reference harness's CUDA runner
(``experiments/source/harness/run.py:1795-1895``): read ``manifest.json``,
``ctypes.CDLL`` the artefact, bind each entry from its manifest ``params``,
size and cache the workspace with ``<symbol>_workspace_size``, and call with
device pointers.  A non-zero status raises ``LoomError``.

There is no CPU fallback: if the library cannot be loaded, or a tensor is not
a contiguous float32 CUDA tensor, the call fails.
"""

from __future__ import annotations

import ctypes
import json
import os
from typing import Dict, List, Optional, Sequence

STATUS_NAMES = {0: "OK", 1: "INVALID_ARGUMENT", 2: "WORKSPACE_TOO_SMALL", 3: "CUDA_ERROR",
                4: "COMM_ERROR"}


class LoomError(RuntimeError):
    def __init__(self, symbol: str, status: int):
        super().__init__(f"{symbol} returned {status} ({STATUS_NAMES.get(status, '?')})")
        self.status = status


def _torch():
    import torch
    return torch


class Entry:
    """One exported entry of a package."""

    def __init__(self, lib: ctypes.CDLL, meta: dict, package: "Package"):
        self.lib = lib
        self.meta = meta
        self.package = package
        self.name = meta["entry_name"]
        self.symbol = meta["symbol_name"]
        self.params = meta["params"]
        self.result_kind = meta["result_kind"]
        self.tensor_params = [p["name"] for p in self.params if p["kind"] == "tensor1-f32"]
        self.scalar_params = [p["name"] for p in self.params if p["kind"] == "scalar-f32"]
        ptypes = [ctypes.c_float if p["kind"] == "scalar-f32" else ctypes.c_void_p
                  for p in self.params]
        self.fn = getattr(lib, self.symbol)
        self.fn.argtypes = ptypes + [ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p,
                                     ctypes.c_size_t]
        self.fn.restype = ctypes.c_int
        self.ws_fn = getattr(lib, meta["workspace_symbol"])
        self.ws_fn.argtypes = [ctypes.c_int64]
        self.ws_fn.restype = ctypes.c_size_t
        self.stream_fn = getattr(lib, meta.get("stream_symbol", self.symbol + "_stream"))
        self.stream_fn.argtypes = list(self.fn.argtypes) + [ctypes.c_void_p]
        self.stream_fn.restype = ctypes.c_int
        self.noworkspace_fn = None
        if meta.get("no_workspace_symbol"):
            self.noworkspace_fn = getattr(lib, meta["no_workspace_symbol"])
            self.noworkspace_fn.argtypes = ptypes + [ctypes.c_int64, ctypes.c_void_p]
            self.noworkspace_fn.restype = ctypes.c_int
        self.dist_fn = None
        if meta.get("dist_symbol"):
            self.dist_fn = getattr(lib, meta["dist_symbol"])
            self.dist_fn.argtypes = ptypes + [ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p,
                                              ctypes.c_size_t, ctypes.c_void_p, ctypes.c_void_p]
            self.dist_fn.restype = ctypes.c_int
            self.dist_ws_fn = getattr(lib, meta["dist_workspace_symbol"])
            self.dist_ws_fn.argtypes = [ctypes.c_int64]
            self.dist_ws_fn.restype = ctypes.c_size_t
        self.multi_fn = None
        if meta.get("multi_symbol"):
            self.multi_fn = getattr(lib, meta["multi_symbol"])
            mtypes = [ctypes.c_float if p["kind"] == "scalar-f32" else ctypes.c_void_p
                      for p in self.params]
            self.multi_fn.argtypes = [ctypes.c_int, ctypes.c_void_p] + mtypes + [
                ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                ctypes.c_void_p]
            self.multi_fn.restype = ctypes.c_int
        self._ws: Dict[tuple, object] = {}

    # -- helpers ------------------------------------------------------------
    def workspace_size(self, n: int) -> int:
        return int(self.ws_fn(int(n)))

    def workspace(self, n: int, device=None, dist: bool = False, stream=None):
        """Cached device workspace for n elements (None when not needed).
        One workspace per (device, stream, size): calls on one stream are
        ordered by that stream, and calls on different streams, which may
        run at the same time, never share one."""
        torch = _torch()
        size = int(self.dist_ws_fn(n)) if dist else self.workspace_size(n)
        if size <= 0:
            return None
        device = torch.device(device if device is not None else "cuda")
        handle = int(getattr(stream, "cuda_stream", stream) or 0)
        key = (str(device), handle, size)
        ws = self._ws.get(key)
        if ws is None:
            ws = torch.empty(size, dtype=torch.uint8, device=device)
            self._ws[key] = ws
        return ws

    def _args(self, inputs: Dict[str, object], n: Optional[int] = None) -> List[object]:
        torch = _torch()
        args: List[object] = []
        for p in self.params:
            v = inputs[p["name"]]
            if p["kind"] == "scalar-f32":
                args.append(ctypes.c_float(float(v)))
            else:
                if not (isinstance(v, torch.Tensor) and v.is_cuda and v.dtype == torch.float32
                        and v.is_contiguous()):
                    raise TypeError(f"{self.name}: {p['name']} must be a contiguous float32 "
                                    "CUDA tensor")
                if n is not None and v.numel() != n:
                    raise ValueError(f"{self.name}: {p['name']} has {v.numel()} elements, "
                                     f"expected {n}")
                args.append(ctypes.c_void_p(v.data_ptr()))
        return args

    def _n(self, inputs: Dict[str, object]) -> int:
        return int(inputs[self.tensor_params[0]].numel())

    def _device(self, inputs: Dict[str, object]):
        """The one CUDA device that holds every tensor input."""
        devs = {inputs[t].device for t in self.tensor_params if hasattr(inputs[t], "device")}
        if len(devs) != 1:
            raise ValueError(f"{self.name}: tensor inputs must be on one CUDA device, got "
                             f"{sorted(str(d) for d in devs)}")
        return devs.pop()

    def _check_out(self, out, n: int, device) -> None:
        """The output must hold the whole result on the inputs' device: the
        kernels write n floats (1 for a scalar result) through it."""
        torch = _torch()
        need = n if self.result_kind == "tensor" else 1
        if not (isinstance(out, torch.Tensor) and out.is_cuda and out.dtype == torch.float32
                and out.is_contiguous()):
            raise TypeError(f"{self.name}: out must be a contiguous float32 CUDA tensor")
        if out.device != device:
            raise ValueError(f"{self.name}: out is on {out.device}, inputs on {device}")
        if out.numel() < need:
            raise ValueError(f"{self.name}: out has {out.numel()} elements, needs {need}")

    def new_output(self, n: int, device):
        torch = _torch()
        if self.result_kind == "tensor":
            return torch.empty(n, dtype=torch.float32, device=device)
        return torch.empty(1, dtype=torch.float32, device=device)

    # -- calls ----------------------------------------------------------------
    def __call__(self, out=None, stream=None, **inputs):
        """Run on device tensors; returns the output tensor (n floats, or 1
        float for a scalar result).  With `stream` (a torch.cuda.Stream or a
        raw handle) the call is asynchronous on that stream."""
        torch = _torch()
        n = self._n(inputs)
        args = self._args(inputs, n)
        device = self._device(inputs)
        if out is None:
            out = self.new_output(n, device)
        self._check_out(out, n, device)
        with torch.cuda.device(device):
            ws = self.workspace(n, device, stream=stream)
            wsp = ctypes.c_void_p(ws.data_ptr()) if ws is not None else None
            wss = ctypes.c_size_t(ws.numel() if ws is not None else 0)
            tail = [ctypes.c_int64(n), ctypes.c_void_p(out.data_ptr()), wsp, wss]
            if stream is None:
                status = self.fn(*args, *tail)
            else:
                handle = getattr(stream, "cuda_stream", stream)
                status = self.stream_fn(*args, *tail, ctypes.c_void_p(handle))
        if status != 0:
            raise LoomError(self.symbol, status)
        return out

    def bind(self, out=None, stream=None, **inputs):
        """The same call with every argument converted once: returns
        `(call, out)`, where `call()` launches on `stream` (the legacy
        default stream when None) and raises LoomError on a bad status.
        For launch loops where the per-call Python work would show, and for
        stream capture.  The tensors must stay alive while `call` is used."""
        n = self._n(inputs)
        args = self._args(inputs, n)
        device = self._device(inputs)
        if device.index != _torch().cuda.current_device():
            raise ValueError(f"{self.name}: bind with the inputs' device ({device}) current; "
                             "the bound call launches on the current device")
        if out is None:
            out = self.new_output(n, device)
        self._check_out(out, n, device)
        ws = self.workspace(n, device, stream=stream)
        wsp = ctypes.c_void_p(ws.data_ptr()) if ws is not None else None
        wss = ctypes.c_size_t(ws.numel() if ws is not None else 0)
        handle = getattr(stream, "cuda_stream", stream) if stream is not None else 0
        full = args + [ctypes.c_int64(n), ctypes.c_void_p(out.data_ptr()), wsp, wss,
                       ctypes.c_void_p(handle)]
        fn, symbol = self.stream_fn, self.symbol

        def call():
            status = fn(*full)
            if status != 0:
                raise LoomError(symbol, status)
        return call, out

    def call_raw(self, *args) -> int:
        return int(self.fn(*args))

    def dist(self, comm: "Comm", out=None, stream=None, **inputs):
        """This rank's shard of a multi-GPU call (one process per GPU)."""
        if self.dist_fn is None:
            raise RuntimeError(f"{self.package.name} was built without multi-GPU entries")
        n = self._n(inputs)
        args = self._args(inputs, n)
        device = self._device(inputs)
        if out is None:
            out = self.new_output(n, device)
        self._check_out(out, n, device)
        ws = self.workspace(n, device, dist=True, stream=stream)
        wsp = ctypes.c_void_p(ws.data_ptr()) if ws is not None else None
        wss = ctypes.c_size_t(ws.numel() if ws is not None else 0)
        handle = getattr(stream, "cuda_stream", stream) if stream is not None else None
        status = self.dist_fn(*args, ctypes.c_int64(n), ctypes.c_void_p(out.data_ptr()), wsp,
                              wss, ctypes.c_void_p(comm.handle), ctypes.c_void_p(handle))
        if status != 0:
            raise LoomError(self.symbol + "_dist", status)
        return out


    def call_host(self, out=None, comm: Optional["Comm"] = None, chunk_elems: int = 1 << 23,
                  **inputs):
        """Run on HOST inputs (CPU torch tensors, ideally pinned, or numpy
        arrays) and return a CPU tensor.  The current CUDA device runs it.

        Maps stream in chunks through two device slots per tensor: chunk c+1
        is copied in (and computed) on one stream while chunk c is copied
        out on another, so the host->device and device->host PCIe directions
        run at the same time.  Reductions copy each input to the device once
        and call the entry (the `_dist` entry when `comm` is given, so every
        rank gets the global result).  Host memory must not be touched until
        the call returns; it synchronises before returning."""
        torch = _torch()
        host = {}
        for p in self.params:
            v = inputs[p["name"]]
            if p["kind"] == "tensor1-f32":
                if not isinstance(v, torch.Tensor):
                    v = torch.from_numpy(v)
                if v.is_cuda or v.dtype != torch.float32 or not v.is_contiguous():
                    raise TypeError(f"{self.name}: {p['name']} must be a contiguous float32 "
                                    "host tensor")
            host[p["name"]] = v
        n = int(host[self.tensor_params[0]].numel())
        for t in self.tensor_params:
            if host[t].numel() != n:
                raise ValueError(f"{self.name}: tensor inputs must share one length")
        dev = torch.device("cuda", torch.cuda.current_device())
        if out is None:
            out = torch.empty(n if self.result_kind == "tensor" else 1, dtype=torch.float32,
                              pin_memory=True)
        st = self._host_state(dev, chunk_elems if self.result_kind == "tensor" else n)
        s_in, s_out = st["streams"]
        cur = torch.cuda.current_stream(dev)
        s_in.wait_stream(cur)
        if self.result_kind == "scalar":
            with torch.cuda.stream(s_in):
                dev_in = {t: st["slots"][t][0][:n] for t in self.tensor_params}
                for t in self.tensor_params:
                    dev_in[t].copy_(host[t], non_blocking=True)
                args = {**{k: v for k, v in host.items() if k not in dev_in}, **dev_in}
                res = st["out"][0]
                if comm is not None:
                    self.dist(comm, out=res, stream=s_in, **args)
                else:
                    self(out=res, stream=s_in, **args)
                out.copy_(res, non_blocking=True)
            s_in.synchronize()
            return out
        chunk = st["chunk"]
        for c, off in enumerate(range(0, n, chunk)):
            ln = min(chunk, n - off)
            slot = c % 2
            if c >= 2:
                s_in.wait_event(st["drained"][slot])
            with torch.cuda.stream(s_in):
                dev_in = {t: st["slots"][t][slot][:ln] for t in self.tensor_params}
                for t in self.tensor_params:
                    dev_in[t].copy_(host[t][off:off + ln], non_blocking=True)
                args = {**{k: v for k, v in host.items() if k not in dev_in}, **dev_in}
                res = st["out"][slot][:ln]
                self(out=res, stream=s_in, **args)
                st["computed"][slot].record(s_in)
            s_out.wait_event(st["computed"][slot])
            with torch.cuda.stream(s_out):
                out[off:off + ln].copy_(res, non_blocking=True)
                st["drained"][slot].record(s_out)
        s_out.synchronize()
        s_in.synchronize()
        return out

    def _host_state(self, dev, chunk: int):
        """Per-device streams, events and device slots of call_host (cached,
        grown on demand)."""
        torch = _torch()
        key = str(dev)
        st = self._ws.get(("host", key))
        chunk = max(1, int(chunk))
        if st is None or st["chunk"] < chunk:
            nslots = 2 if self.result_kind == "tensor" else 1
            st = {
                "chunk": chunk,
                "streams": (torch.cuda.Stream(dev), torch.cuda.Stream(dev)),
                "slots": {t: [torch.empty(chunk, dtype=torch.float32, device=dev)
                              for _ in range(nslots)] for t in self.tensor_params},
                "out": [torch.empty(chunk if self.result_kind == "tensor" else 1,
                                    dtype=torch.float32, device=dev) for _ in range(nslots)],
                "computed": [torch.cuda.Event() for _ in range(2)],
                "drained": [torch.cuda.Event() for _ in range(2)],
            }
            self._ws[("host", key)] = st
        return st

    def multi(self, comms: Sequence["Comm"], shards: Sequence[Dict[str, object]], outs=None):
        """One process, one shard per device: ``shards[d]`` holds the tensor
        inputs on ``comms[d]``'s device (scalars are taken from ``shards[0]``).
        Returns (per-device outputs, host scalar or None)."""
        if self.multi_fn is None:
            raise RuntimeError(f"{self.package.name} was built without multi-GPU entries")
        torch = _torch()
        nd = len(comms)
        if nd != len(shards) or nd == 0:
            raise ValueError("one shard per communicator")
        ns = [self._n(sh) for sh in shards]
        if outs is None:
            outs = [self.new_output(ns[d], shards[d][self.tensor_params[0]].device)
                    for d in range(nd)]
        for d in range(nd):
            self._check_out(outs[d], ns[d], self._device(shards[d]))
        keep = []
        args = [ctypes.c_int(nd), (ctypes.c_void_p * nd)(*[c.handle for c in comms])]
        for p in self.params:
            if p["kind"] == "scalar-f32":
                args.append(ctypes.c_float(float(shards[0][p["name"]])))
            else:
                for sh, n in zip(shards, ns):
                    self._args({q["name"]: sh[q["name"]] for q in self.params}, n)
                arr = (ctypes.c_void_p * nd)(*[sh[p["name"]].data_ptr() for sh in shards])
                keep.append(arr)
                args.append(ctypes.cast(arr, ctypes.c_void_p))
        shard_n = (ctypes.c_int64 * nd)(*ns)
        out_arr = (ctypes.c_void_p * nd)(*[o.data_ptr() for o in outs])
        wss = [self.workspace(ns[d], outs[d].device, dist=True) for d in range(nd)]
        ws_arr = (ctypes.c_void_p * nd)(*[w.data_ptr() if w is not None else 0 for w in wss])
        ws_sz = (ctypes.c_size_t * nd)(*[w.numel() if w is not None else 0 for w in wss])
        host = ctypes.c_float(float("nan"))
        status = self.multi_fn(*args, shard_n, out_arr, ws_arr, ws_sz,
                               ctypes.byref(host) if self.result_kind == "scalar" else None)
        if status != 0:
            raise LoomError(self.symbol + "_multi", status)
        return outs, (float(host.value) if self.result_kind == "scalar" else None)


class Comm:
    """A communicator owned by a package (one rank of one process): NCCL,
    plus the peer-memory scalar exchange where every GPU reaches the
    others' memory."""

    def __init__(self, package: "Package", handle: int, nranks: int, rank: int):
        self.package = package
        self.handle = handle
        self.nranks = nranks
        self.rank = rank

    @property
    def peer_exchange(self) -> bool:
        """Whether reductions exchange their scalar through peer memory."""
        return bool(self.package._comm_peer_exchange(ctypes.c_void_p(self.handle)))

    def set_peer_exchange(self, enable: bool) -> None:
        """Switch between the peer-memory exchange and NCCL.  Every rank
        must make the same choice before its next reduction."""
        st = self.package._comm_set_peer_exchange(ctypes.c_void_p(self.handle), int(enable))
        if st != 0:
            raise LoomError(f"loom_{self.package.name}_comm_set_peer_exchange", st)

    def set_timeout_ms(self, ms: int) -> None:
        """How long a peer exchange waits for the other ranks before it gives
        up (its result is then NaN and `check` raises)."""
        st = self.package._comm_set_timeout_ms(ctypes.c_void_p(self.handle), int(ms))
        if st != 0:
            raise LoomError(f"loom_{self.package.name}_comm_set_timeout_ms", st)

    def check(self) -> None:
        """Wait for this rank's device; raise if a peer exchange gave up
        waiting for another rank (its result was NaN)."""
        st = self.package._comm_check(ctypes.c_void_p(self.handle))
        if st != 0:
            raise LoomError(f"loom_{self.package.name}_comm_check", st)

    def exchange_stats(self, reset: bool = False) -> dict:
        """This rank's peer-exchange wait statistics since the communicator
        was created or last reset (after waiting for its device): total and
        largest time from sending its value to holding every rank's, in
        microseconds, and the number of exchanges timed; zeroed afterwards
        with `reset`.  All zero on the NCCL path."""
        out = (ctypes.c_uint64 * 3)()
        if self.package._comm_exchange_stats is None:
            raise RuntimeError(f"{self.package.name} was built without exchange statistics")
        st = self.package._comm_exchange_stats(ctypes.c_void_p(self.handle), out, int(reset))
        if st != 0:
            raise LoomError(f"loom_{self.package.name}_comm_exchange_stats", st)
        return {"total_us": out[0] / 1e3, "max_us": out[1] / 1e3, "exchanges": int(out[2])}

    def destroy(self) -> None:
        if self.handle:
            self.package._comm_destroy(ctypes.c_void_p(self.handle))
            self.handle = 0


class Package:
    """A built package: ``Package(out_dir)`` or ``Package(manifest_path)``."""

    def __init__(self, path: str):
        manifest = path if path.endswith(".json") else os.path.join(path, "manifest.json")
        with open(manifest, "r", encoding="utf-8") as fh:
            self.manifest = json.load(fh)
        self.name = self.manifest["package_name"]
        artifact = self.manifest["artifact_path"]
        if not os.path.exists(artifact):
            artifact = os.path.join(os.path.dirname(manifest), os.path.basename(artifact))
        self.path = artifact
        self.lib = ctypes.CDLL(artifact)
        self.entries = {e["entry_name"]: Entry(self.lib, e, self)
                        for e in self.manifest["entries"]}
        prefix = f"loom_{self.name}_comm"
        self._has_comm = hasattr(self.lib, prefix + "_unique_id")
        if self._has_comm:
            self._comm_id_size = getattr(self.lib, prefix + "_id_size")
            self._comm_id_size.restype = ctypes.c_int
            self._comm_unique_id = getattr(self.lib, prefix + "_unique_id")
            self._comm_unique_id.argtypes = [ctypes.c_void_p, ctypes.c_size_t]
            self._comm_init_rank = getattr(self.lib, prefix + "_init_rank")
            self._comm_init_rank.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_int,
                                             ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t]
            self._comm_init_all = getattr(self.lib, prefix + "_init_all")
            self._comm_init_all.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_int,
                                            ctypes.POINTER(ctypes.c_int)]
            self._comm_destroy = getattr(self.lib, prefix + "_destroy")
            self._comm_destroy.argtypes = [ctypes.c_void_p]
            self._comm_set_peer_exchange = getattr(self.lib, prefix + "_set_peer_exchange")
            self._comm_set_peer_exchange.argtypes = [ctypes.c_void_p, ctypes.c_int]
            self._comm_set_timeout_ms = getattr(self.lib, prefix + "_set_timeout_ms")
            self._comm_set_timeout_ms.argtypes = [ctypes.c_void_p, ctypes.c_int64]
            self._comm_peer_exchange = getattr(self.lib, prefix + "_peer_exchange")
            self._comm_peer_exchange.argtypes = [ctypes.c_void_p]
            self._comm_check = getattr(self.lib, prefix + "_check")
            self._comm_check.argtypes = [ctypes.c_void_p]
            # packages built before the exchange statistics lack the symbol
            self._comm_exchange_stats = getattr(self.lib, prefix + "_exchange_stats", None)
            if self._comm_exchange_stats is not None:
                self._comm_exchange_stats.argtypes = [ctypes.c_void_p,
                                                      ctypes.POINTER(ctypes.c_uint64),
                                                      ctypes.c_int]

    def __getitem__(self, entry: str) -> Entry:
        return self.entries[entry]

    def __getattr__(self, entry: str) -> Entry:
        entries = self.__dict__.get("entries", {})
        if entry in entries:
            return entries[entry]
        raise AttributeError(entry)

    # -- communicators ------------------------------------------------------
    def comm_unique_id(self) -> bytes:
        size = int(self._comm_id_size())
        buf = ctypes.create_string_buffer(size)
        status = self._comm_unique_id(buf, size)
        if status != 0:
            raise LoomError("comm_unique_id", status)
        return buf.raw

    def comm_init_rank(self, nranks: int, rank: int, uid: bytes) -> Comm:
        """One rank of a communicator on the current CUDA device (collective)."""
        handle = ctypes.c_void_p(0)
        buf = ctypes.create_string_buffer(uid, len(uid))
        status = self._comm_init_rank(ctypes.byref(handle), nranks, rank, buf, len(uid))
        if status != 0:
            raise LoomError("comm_init_rank", status)
        return Comm(self, handle.value, nranks, rank)

    def comm_from_process_group(self, group=None) -> Comm:
        """Rendezvous a communicator over an initialised torch.distributed group."""
        import torch.distributed as dist
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        box = [self.comm_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(box, src=0, group=group)
        return self.comm_init_rank(world, rank, box[0])

    def comm_init_all(self, devices: Sequence[int]) -> List[Comm]:
        n = len(devices)
        handles = (ctypes.c_void_p * n)()
        devs = (ctypes.c_int * n)(*devices)
        status = self._comm_init_all(handles, n, devs)
        if status != 0:
            raise LoomError("comm_init_all", status)
        return [Comm(self, handles[i], n, i) for i in range(n)]
