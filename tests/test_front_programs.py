"""Seeded random entries over the structured forms of the entry language
(tests/golden/sources/front_programs, make_front_programs.py there): local
helpers with one or two parameters, helpers ending in if/else, helpers
calling helpers or passed to maps, tuple and annotated lets, qualified
primitives, select, unary plus, equality tests and tensor-level helpers.

* FrontIR: equal to what the reference's Python frontend printed for every
  entry (tests/golden/front_programs_front_ir.json).
* Lowering: every entry lowers to valid TensorIR except two that the
  reference's normalize rejects as well.  It binds a helper's arguments in
  the helper's own closure, not in the caller's environment
  (src/loom_normalize/normalize.ml:96-113), so an argument that names the
  caller's parameter is left unbound (f000: ``h0(select(a > v, v, u))``
  inside ``h1(u, v)``), and a helper applied to a call of itself does not
  see itself (f020: ``h0(h0(u, s), ...)``).  The messages are tensorize's
  (src/loom_tensorize/tensorize.ml:47, :95).
* Passes: with every restated pass flag, and with the flag set of the
  reference harness's tuned CUDA profile, each program evaluates in float64
  to what it evaluates to without flags, up to rounding.
"""

import json
import os

import numpy as np
import pytest

from loom_b200 import tensor_ir as TI
from loom_b200.build import CUDA_FIXED_FLAGS
from loom_b200.frontend import FrontendError, front_ir, program_from_front_ir

from test_pass_equivalence import ALL_PASSES, evaluate

HERE = os.path.dirname(os.path.abspath(__file__))
SOURCE = os.path.join(HERE, "golden", "sources", "front_programs", "front_programs.py")
GOLDEN = json.load(open(os.path.join(HERE, "golden", "front_programs_front_ir.json")))
REJECTED = {"f000": "unbound scalar variable v",
            "f020": "unknown function call inside scalar lambda: h0"}


def test_front_ir_matches_the_reference_frontend():
    with open(SOURCE, encoding="utf-8") as fh:
        src = fh.read()
    assert len(GOLDEN) == 30
    for entry, want in GOLDEN.items():
        assert front_ir(src, entry) == want, entry


def test_rejections_follow_the_reference_normalize():
    for entry, message in REJECTED.items():
        with pytest.raises(FrontendError) as info:
            program_from_front_ir(GOLDEN[entry])
        assert str(info.value) == message, entry


@pytest.mark.parametrize("flags", [ALL_PASSES, tuple(CUDA_FIXED_FLAGS)],
                         ids=["all_passes", "cuda_fixed"])
def test_lowering_and_passes_preserve_values(flags):
    n = 500
    for entry, front in sorted(GOLDEN.items()):
        if entry in REJECTED:
            continue
        plain = program_from_front_ir(front)
        rewritten = program_from_front_ir(front, flags)
        TI.validate(plain)
        TI.validate(rewritten)
        rng = np.random.default_rng(int(entry[1:]))
        inp = {"x": rng.standard_normal(n), "y": rng.standard_normal(n), "a": 0.75}
        want, mag = evaluate(plain, inp, n)
        got, _ = evaluate(rewritten, inp, n)
        tol = 1e-9 * (np.asarray(mag) + 1.0)
        assert np.all(np.abs(np.asarray(got) - np.asarray(want)) <= tol), entry
