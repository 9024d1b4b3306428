"""Which generated reduction bodies are marked non-negative (kNonNegative).

A sum whose values can never be negative may add up to 16 values per tile in
fp32 before converting (Chunking in loom_b200_device.cuh): with no
cancellation the error stays within a few fp32 units of the total.  Every
other sum adds each value in fp64.  Only the square families qualify: a
value multiplied by itself (norm-square, x*x) or a difference multiplied by
itself (delta-square, (a-b)*(a-b)); a signed product, a weighted square or a
select must not.
"""

import json
import os

from loom_b200 import tensor_ir as TI
from loom_b200.codegen import render_body_struct
from loom_b200.plan import plan_entry

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def _marked(prog):
    src = render_body_struct(plan_entry(prog, "kernels"))
    assert src.count("kNonNegative") == 1
    return "static constexpr bool kNonNegative = true;" in src


def test_suite_bodies():
    progs = [TI.program_from_json(o) for o in
             json.load(open(os.path.join(ROOT, "oracle", "suite_kernels.tensor_ir.json")))]
    marked = {p.entry_name: _marked(p) for p in progs}
    assert marked == {"saxpy": False, "relu": False, "dot": False, "l2_norm_sq": True,
                      "max_value": False, "affine_relu": False, "pipeline_sum": False}


def test_harness_kernel_bodies():
    from test_workloads import _programs
    marked = {name: _marked(p) for name, p in _programs().items()}
    # l2_norm_sq is x*x; mse_sum and inventory_penalty_sum are (a-b)*(a-b)
    assert sorted(k for k, v in marked.items() if v) == \
        ["inventory_penalty_sum", "l2_norm_sq", "mse_sum"]
