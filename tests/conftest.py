"""Shared pytest configuration.

Tests marked ``gpu`` need a CUDA device (a B200); everything else runs on a
CPU-only host.  The repository root is put on ``sys.path`` so that the
package, the oracle and ``bench.py`` import without installation.
"""

from __future__ import annotations

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    path = os.path.join(ROOT, "tests", "golden", "w4a4_golden.npz")
    with np.load(path) as data:
        return {k: data[k] for k in data.files}
