"""Shared fixtures.

Markers: ``gpu`` tests need a CUDA device (run with ``-m gpu`` on a B200);
everything else runs on CPU.
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent
GOLDEN = REPO / "tests" / "golden"
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device")


def pytest_collection_modifyitems(config, items):
    try:
        import torch

        has_gpu = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def manifest():
    return json.loads((GOLDEN / "MANIFEST.json").read_text())


@pytest.fixture(scope="session")
def enc_golden():
    return np.load(GOLDEN / "encoder_golden.npz")


@pytest.fixture(scope="session")
def fwd_golden():
    return np.load(GOLDEN / "forward_golden.npz")


@pytest.fixture(scope="session")
def fmt_golden():
    return np.load(GOLDEN / "format_golden.npz")


@pytest.fixture(scope="session")
def float_golden():
    return np.load(GOLDEN / "float_golden.npz")


@pytest.fixture(scope="session")
def ldlq_golden():
    return np.load(GOLDEN / "ldlq_golden.npz")


@pytest.fixture(scope="session")
def golden_dir():
    return GOLDEN


@pytest.fixture(scope="session")
def module_golden_arrays():
    return np.load(GOLDEN / "module_golden.npz")


@pytest.fixture(scope="session")
def storage_golden():
    path = GOLDEN / "storage_golden.npz"
    if not path.exists():
        pytest.skip("storage golden not generated")
    return np.load(path)
