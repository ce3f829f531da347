"""Shared test set-up: the ``gpu`` marker, the golden fixtures and the oracle."""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = Path(__file__).resolve().parent / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


def golden_names() -> list[str]:
    """The MSDA golden cases (deformable aggregation: da_*.npz, FlashSCA: fsca_*.npz)."""
    return sorted(p.stem for p in GOLDEN.glob("*.npz") if not p.stem.startswith(("da_", "fsca_")))


def load_golden(name: str) -> dict[str, np.ndarray]:
    with np.load(GOLDEN / f"{name}.npz") as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("this test needs a CUDA device; run it on the GPU box (-m gpu)")
    return torch.device("cuda", 0)
