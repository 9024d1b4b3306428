"""Build and load the reference-style GPU baseline.

`loom_reference_style.cu` restates, by hand, the CUDA that the reference's
backend (src/loom_backend_cuda/cuda_backend.ml) generates for the seven suite
entries under two of its optimisation profiles: "none" (loom_none_fixed) and
"cuda" (loom_cuda_fixed).  It is built with the reference's nvcc flags for
sm_100a into `baseline/_ref/` and timed beside the product on the same GPU.
Benchmark and test infrastructure only.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "loom_reference_style.cu")
OUT_DIR = os.path.join(HERE, "_ref")
LIB = os.path.join(OUT_DIR, "libloom_reference_style.so")

PROFILES = ("none", "cuda")
# parameters of each entry in the reference's argument order ("a" is the
# scalar, the rest are tensors), as in the suite's C ABI
PARAMS = {
    "saxpy": ("a", "x", "y"), "relu": ("x",), "dot": ("x", "y"), "l2_norm_sq": ("x",),
    "max_value": ("x",), "affine_relu": ("a", "x", "y"), "pipeline_sum": ("a", "x", "y", "w"),
}
MAPS = {"saxpy", "relu", "affine_relu"}
# kernel launches per call, by profile (maps, then reductions at n = 2^28:
# a first kernel, the combine launches down to one value, and the cuda
# profile's memset for atomic outputs is not a kernel)
LAUNCHES_2P28 = {
    "none": {"saxpy": 1, "relu": 1, "affine_relu": 1, "dot": 4, "l2_norm_sq": 4,
             "max_value": 3, "pipeline_sum": 5},
    "cuda": {"saxpy": 1, "relu": 1, "affine_relu": 1, "dot": 1, "l2_norm_sq": 1,
             "max_value": 3, "pipeline_sum": 1},
}


def nvcc_command(nvcc: str = "nvcc"):
    # the reference's build line (cuda_backend.ml:2625-2645), for sm_100a
    return [nvcc, "-std=c++17", "-O3", "-shared", "-Xcompiler", "-fPIC",
            "-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-o", LIB, SRC]


def build(force: bool = False) -> str:
    if (not force and os.path.exists(LIB)
            and os.path.getmtime(LIB) >= os.path.getmtime(SRC)):
        return LIB
    os.makedirs(OUT_DIR, exist_ok=True)
    subprocess.run(nvcc_command(), check=True)
    return LIB


class ReferenceStyle:
    """ctypes binding of `loomref_<profile>_<entry>` and its workspace
    function."""

    def __init__(self, path: str = LIB):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} is not built (baseline.reference_style.build())")
        self.lib = ctypes.CDLL(path)
        self.fns = {}
        for profile in PROFILES:
            for entry, params in PARAMS.items():
                fn = getattr(self.lib, f"loomref_{profile}_{entry}")
                fn.restype = ctypes.c_int
                fn.argtypes = ([ctypes.c_float if p == "a" else ctypes.c_void_p for p in params]
                               + [ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p,
                                  ctypes.c_size_t])
                ws = getattr(self.lib, f"loomref_{profile}_{entry}_workspace_size")
                ws.restype = ctypes.c_size_t
                ws.argtypes = [ctypes.c_int64]
                self.fns[(profile, entry)] = (fn, ws)

    def workspace_size(self, profile: str, entry: str, n: int) -> int:
        return int(self.fns[(profile, entry)][1](n))

    def bind(self, profile: str, entry: str, n: int, out, workspace, **inputs):
        """The call with its arguments fixed: a zero-argument callable that
        returns the entry's status.  `inputs` maps parameter names to device
        tensors or (for "a") a float; `workspace` is a device tensor of at
        least workspace_size bytes, or None."""
        fn = self.fns[(profile, entry)][0]
        args = []
        for p in PARAMS[entry]:
            v = inputs[p]
            args.append(ctypes.c_float(v) if p == "a" else ctypes.c_void_p(v.data_ptr()))
        ws_ptr = ctypes.c_void_p(workspace.data_ptr()) if workspace is not None else None
        ws_len = workspace.numel() * workspace.element_size() if workspace is not None else 0
        args += [ctypes.c_int64(n), ctypes.c_void_p(out.data_ptr()), ws_ptr,
                 ctypes.c_size_t(ws_len)]
        return lambda: fn(*args)
