"""Shared test setup: import paths, the `gpu` marker and common fixtures."""
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
PKG = REPO / "tessera-inference_b200"
ORACLE = REPO / "oracle"
GOLDEN = Path(__file__).resolve().parent / "golden"
for p in (PKG, ORACLE):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        have_gpu = torch.cuda.is_available()
    except Exception:
        have_gpu = False
    if have_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


@pytest.fixture(scope="session")
def weights_path(tmp_path_factory):
    """Seed-0 Xavier-uniform Large weights (zero biases), as the benchmark uses."""
    import synth
    return synth.make_weights(tmp_path_factory.mktemp("w") / "student_large_seed0.tcw", seed=0)


@pytest.fixture(scope="session")
def weights_perturbed_path(tmp_path_factory):
    """Seed-0 weights with non-zero biases and LayerNorm affine parameters."""
    import synth
    return synth.make_weights(tmp_path_factory.mktemp("wp") / "student_large_seed0_p.tcw", seed=0, perturb=0.05)
