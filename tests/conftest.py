import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT / "prefix-head_b200"))
sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: minutes-long case (full 270M geometry)")


def has_gpu() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def model_dir(tmp_path_factory):
    d = os.environ.get("GEM_TEST_CACHE")
    return Path(d) if d else tmp_path_factory.mktemp("models")


@pytest.fixture(scope="session")
def small(model_dir):
    from gem_b200 import synth
    return synth.ensure("small", classes=64, directory=model_dir)


@pytest.fixture(scope="session")
def threads():
    return max(1, min(16, os.cpu_count() or 1))
