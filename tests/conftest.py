import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT / "oracle", ROOT / "qwen3.cpp_b200", ROOT / "tests", ROOT / "tests" / "golden"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: takes more than a few seconds on CPU")


@pytest.fixture(scope="session")
def full_weights():
    """Seed-0 random-init Qwen3-0.6B in Qwen3.bin layout (generated once, cached in /tmp)."""
    import gen_weights
    return gen_weights.cached_model(0)


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    d = ROOT / "tests" / "golden"
    return {p.stem: dict(np.load(p)) for p in d.glob("*.npz")}


@pytest.fixture(scope="session")
def q3lib():
    """The CUDA library, built if needed; GPU tests fail loudly if it cannot be loaded."""
    import build
    build.build()
    import q3b200
    return q3b200
