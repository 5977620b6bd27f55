"""Shared test setup: import paths, the `gpu` marker, golden fixture loaders."""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
PACKAGE_ROOT = ROOT / "elastic-kv-vmm_b200"
GOLDEN = Path(__file__).resolve().parent / "golden"
for path in (str(PACKAGE_ROOT), str(ROOT)):
    if path not in sys.path:
        sys.path.insert(0, path)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def load_npz_cases(name):
    """{case: {key: array}} from a fixture written as ``case__key`` entries."""
    cases = {}
    with np.load(GOLDEN / name) as data:
        for key in data.files:
            case, field = key.split("__", 1)
            cases.setdefault(case, {})[field] = data[key]
    return cases


def load_json(name):
    return json.loads((GOLDEN / name).read_text())


@pytest.fixture(scope="session")
def library_path():
    """Path of libekv_b200.so, building it first if it is missing."""
    from ekv_b200 import build

    if not build.LIBRARY.exists():
        build.build()
    return build.LIBRARY


@pytest.fixture(scope="session")
def cuda_device(library_path):
    import torch

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch.device("cuda:0")
