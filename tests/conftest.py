import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "kvq-decode_b200"), os.path.join(ROOT, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "multigpu: needs >= 2 CUDA GPUs")


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        have_cuda = torch.cuda.is_available()
        n = torch.cuda.device_count() if have_cuda else 0
    except Exception:  # pragma: no cover
        have_cuda, n = False, 0
    skip_gpu = pytest.mark.skip(reason="needs a CUDA GPU")
    skip_multi = pytest.mark.skip(reason="needs >= 2 CUDA GPUs")
    for item in items:
        if "gpu" in item.keywords and not have_cuda:
            item.add_marker(skip_gpu)
        if "multigpu" in item.keywords and n < 2:
            item.add_marker(skip_multi)
