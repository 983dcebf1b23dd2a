import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (sm_100a) and the built grappa_b200._cuda extension")
    config.addinivalue_line("markers", "multigpu: needs two or more GPUs")


def pytest_collection_modifyitems(config, items):
    import torch

    n = torch.cuda.device_count() if torch.cuda.is_available() else 0
    skip_gpu = pytest.mark.skip(reason="no CUDA device")
    skip_multi = pytest.mark.skip(reason="needs two or more GPUs")
    for item in items:
        if "gpu" in item.keywords and n == 0:
            item.add_marker(skip_gpu)
        elif "multigpu" in item.keywords and n < 2:
            item.add_marker(skip_multi)
