import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "triattention-ggml_b200")
ORACLE = os.path.join(REPO, "oracle")
GOLDEN = os.path.join(REPO, "tests", "golden")
for p in (PKG, ORACLE):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def oracle():
    import oracle_py
    if not os.path.exists(oracle_py.ORACLE_SO):
        oracle_py.build(ref=True)
    return oracle_py.Oracle()


@pytest.fixture(scope="session")
def reflib():
    import oracle_py
    if not oracle_py.RefLib.available():
        oracle_py.build(ref=True)
    if not oracle_py.RefLib.available():
        pytest.skip("compiled reference (oracle/_ref) not available")
    return oracle_py.RefLib()


@pytest.fixture(scope="session")
def synth_stats_path():
    return os.path.join(GOLDEN, "synth_l2h8kv4.tria")


@pytest.fixture(scope="session")
def torch_dev():
    """cuda:0 with the library built; GPU tests fail (not skip) without a GPU."""
    import torch
    import tria_b200
    if not torch.cuda.is_available():
        pytest.fail("no CUDA device: the GPU tests need a B200")
    if not os.path.exists(tria_b200.LIB_PATH):
        tria_b200.build()
    return torch.device("cuda:0")
