"""loom_b200: a B200-native (sm_100a) CUDA backend and runtime for the Loom
tensor compiler's data-parallel hot path -- ``Tensor1.map / map2 /
reduce_sum / reduce_max`` over 1D float32 tensors and their fused
map-then-reduce chains -- behind the reference's ``loomc compile/package
--target cuda`` artefact layout and C ABI.

Layers:
  tensor_ir   TensorIR model and JSON (the input boundary)
  plan        fused B200 plan per entry (one streaming kernel per entry)
  render      scalar-body rendering with the reference's emission rules
  codegen     generated CUDA (body functors + C ABI wrappers) and header
  artifact    package/compile drivers, nvcc (sm_100a), manifest and report
  loader      thin ctypes/PyTorch host loader over the C ABI
  csrc/       hand-written sm_100a kernels and launchers
"""

__version__ = "0.1.0"
