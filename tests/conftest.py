import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "llama98-zh_b200")
for p in (ROOT, PKG, os.path.join(ROOT, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)

MODEL_ROOT = os.environ.get("LZ98_MODEL_DIR", "/tmp/lz98_models")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def model_dir(name: str) -> str:
    """Directory holding the synthetic model `name` (written on first use)."""
    import lz98_synth
    d = os.path.join(MODEL_ROOT, name)
    lz98_synth.write_model(lz98_synth.CONFIGS[name], d)
    return d


@pytest.fixture(scope="session")
def tiny_dir():
    return model_dir("tiny")


@pytest.fixture(scope="session")
def mini_dir():
    return model_dir("mini")
