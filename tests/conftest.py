import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parents[1]
GOLDEN = REPO / "tests" / "golden"
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built libq4gpu.so")


class _Npz:
    """Lazy view of a fixture archive; ``kat['name/field']``."""

    def __init__(self, path: Path):
        self._d = np.load(path)

    def __getitem__(self, key):
        return self._d[key]

    def group(self, prefix: str) -> dict:
        p = prefix + "/"
        return {k[len(p):]: self._d[k] for k in self._d.files if k.startswith(p)}

    def keys(self):
        return self._d.files


@pytest.fixture(scope="session")
def kat():
    return _Npz(GOLDEN / "kat_vectors.npz")


@pytest.fixture(scope="session")
def refh():
    return _Npz(GOLDEN / "ref_helpers.npz")


@pytest.fixture(scope="session")
def refmodel():
    p = GOLDEN / "ref_model_seed0.npz"
    if not p.exists():
        pytest.skip("whole-model golden not generated")
    return _Npz(p)
