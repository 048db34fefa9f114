import json
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "multigpu: needs two or more GPUs")


@pytest.fixture(scope="session")
def golden():
    with open(os.path.join(ROOT, "tests", "golden", "reference_fixtures.json")) as fh:
        return {c["id"]: c for c in json.load(fh)["cases"]}


@pytest.fixture(scope="session")
def oracle():
    from oracle import host_ref
    host_ref.build()
    return host_ref


@pytest.fixture(scope="session")
def device():
    """The CUDA device.  GPU tests fail (never skip) when it cannot be opened,
    so a GPU run cannot pass on a silent fallback."""
    from hephaestus_b200 import CudaDevice
    return CudaDevice(0)
