"""Shared pytest setup: the ``gpu`` marker, import paths and golden fixtures."""

from __future__ import annotations

import json
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden", "sbda_golden.npz")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); parity tests through the C ABI")


PATH_GOLDEN = os.path.join(ROOT, "tests", "golden", "path_golden.npz")
BLOCK_GOLDEN = os.path.join(ROOT, "tests", "golden", "block_golden.npz")
LM_GOLDEN = os.path.join(ROOT, "tests", "golden", "lm_golden.npz")


class Golden:
    """Reference-generated vectors (see tests/golden/make_golden.py)."""

    def __init__(self, path: str) -> None:
        self._data = np.load(path)
        meta = json.loads(bytes(self._data["manifest"]).decode())
        self.cases = meta["cases"]
        self.schedules = meta.get("schedules", {})
        self.total_layers = meta.get("total_layers", 12)

    def get(self, case: str, key: str):
        import torch

        return torch.from_numpy(np.array(self._data[f"{case}/{key}"]))


@pytest.fixture(scope="session")
def golden() -> Golden:
    return Golden(GOLDEN)


@pytest.fixture(scope="session")
def path_golden() -> Golden:
    return Golden(PATH_GOLDEN)


@pytest.fixture(scope="session")
def block_golden() -> Golden:
    return Golden(BLOCK_GOLDEN)


@pytest.fixture(scope="session")
def lm_golden() -> Golden:
    return Golden(LM_GOLDEN)
