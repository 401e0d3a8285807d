import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "multigpu: needs two or more CUDA devices")


@pytest.fixture(autouse=True)
def _skip_gpu_without_cuda(request):
    if request.node.get_closest_marker("gpu") is not None:
        import torch

        if not torch.cuda.is_available():
            pytest.skip("needs a CUDA device")
