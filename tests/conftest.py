"""Test configuration: import paths and the ``gpu`` marker.

``-m "not gpu"`` runs on any CPU machine: the oracle against the golden
vectors, the facade contract against a fake backend, host-side logic and the
C-ABI library's exports. ``-m gpu`` runs the CUDA parity tests on a B200.
"""
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
for path in (ROOT / "fast-audiovae_b200", ROOT):
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU and the built CUDA library")


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    def load(name):
        with np.load(GOLDEN / name, allow_pickle=False) as archive:
            return {k: archive[k] for k in archive.files}
    return load
