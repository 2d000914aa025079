import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the sm_100a kernels)")


@pytest.fixture(scope="session")
def irx():
    import irptx_b200
    irptx_b200._lib()          # loud failure when libirx.so is not built
    return irptx_b200


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("a gpu-marked test ran without a CUDA device")
    torch.cuda.init()
    return torch


@pytest.fixture(autouse=True)
def _reference_core_for_gpu_tests(request):
    """Every GPU test may compare against the reference core's PTX (oracle/_ref/irptx, built by
    __graft_entry__.build() and carried with the tree). Under the gpu marker a missing core is a
    failure, not a silently skipped comparison."""
    if request.node.get_closest_marker("gpu") is None:
        return
    from oracle import refptx
    if not refptx.core_available():
        pytest.fail("the reference core oracle/_ref/irptx is missing: build it (make -C oracle) before the GPU tests")
