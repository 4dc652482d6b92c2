"""Shared pytest configuration: the ``gpu`` marker and golden-fixture helpers."""

import json
import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (sm_100a) device")


def load_golden(name):
    return np.load(GOLDEN / f"{name}.npz")


def golden_json(arr):
    return json.loads(bytes(np.asarray(arr, np.uint8)).decode())


@pytest.fixture(scope="session")
def golden():
    return {k: load_golden(k) for k in ("masks", "segmented", "tiled", "numerics")}


def cuda_available():
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False
