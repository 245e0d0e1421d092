"""Shared pytest set-up: import paths, the ``gpu`` marker and golden loaders."""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parents[1]
PACKAGE_DIR = REPO / "cuda-nvfp4-decoder-attention_b200"
GOLDEN = REPO / "tests" / "golden"
for p in (str(REPO), str(PACKAGE_DIR)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def load_golden(name: str) -> dict:
    with np.load(GOLDEN / f"{name}.npz") as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def golden_format():
    return load_golden("format")


@pytest.fixture(scope="session")
def golden_stages():
    return load_golden("stages")


@pytest.fixture(scope="session")
def golden_forward():
    return load_golden("forward")


@pytest.fixture(scope="session")
def golden_canonical():
    return load_golden("canonical")
