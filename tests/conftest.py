"""pytest configuration: the `gpu` marker and repository paths."""
import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (REPO, os.path.join(REPO, "opure-voxelengine_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def pytest_collection_modifyitems(config, items):
    # A GPU test on a machine without a GPU is skipped, not failed, so that
    # `pytest -m "not gpu"` and a plain `pytest` both work here.
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:  # torch absent or broken: no GPU path either
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)
