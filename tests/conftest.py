import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU")


def pytest_collection_modifyitems(config, items):
    # GPU tests need a device; fail loudly rather than pass on a CPU fallback
    pass


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import Oracle, build

    build()
    return Oracle()


@pytest.fixture(scope="session")
def ref_sampler():
    from oracle.oracle import RefSampler

    if not RefSampler.available():
        pytest.skip("oracle/_ref not built (reference sources absent)")
    return RefSampler()


@pytest.fixture(scope="session")
def cuda():
    import torch

    assert torch.cuda.is_available(), "GPU test run without a CUDA device"
    cap = torch.cuda.get_device_capability()
    assert cap[0] == 10, f"needs sm_100, got sm_{cap[0]}{cap[1]}"
    from noel_b200 import build

    build.build()
    return torch.device("cuda:0")
