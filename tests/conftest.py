import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

SUITE_IR = os.path.join(ROOT, "oracle", "suite_kernels.tensor_ir.json")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device")


@pytest.fixture(scope="session")
def suite_programs():
    from oracle.loom_oracle import load_programs
    return load_programs(SUITE_IR)


@pytest.fixture(scope="session")
def oracle(suite_programs):
    from oracle.loom_oracle import Oracle
    return Oracle(suite_programs, name="b200_suite")


@pytest.fixture(scope="session")
def suite_pkg():
    """The built suite package; GPU tests only (fails loudly if unbuilt)."""
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test collected without a CUDA device")
    from loom_b200.build import load_suite
    return load_suite()
