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


@pytest.fixture(scope="session")
def smollm_dirs(tmp_path_factory):
    """BASELINE config 0's model (SmolLM-135M shape, N(0, 0.02) seed 0, fp16) and config 3's
    draft (the same weights + N(0, 0.004) noise, noise seed 6), written once per session."""
    from voxelengine import engine as ve
    root = tmp_path_factory.mktemp("smollm")
    target = ve.synth_model(str(root / "target"), seed=0)
    draft = ve.synth_model(str(root / "draft"), seed=0, noise_seed=6, noise_std=0.004)
    return target, draft
