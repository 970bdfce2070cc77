"""Shared pytest setup: repo root on sys.path and the ``gpu`` marker.

Tests marked ``gpu`` need a CUDA device (a B200); everything else runs on CPU.
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def load_json(name: str):
    return json.loads((GOLDEN / name).read_text())


def load_npz(name: str) -> dict[str, np.ndarray]:
    with np.load(GOLDEN / name) as data:
        return {k: data[k] for k in data.files}


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("gpu test needs a CUDA device")
    return torch.device("cuda", 0)
