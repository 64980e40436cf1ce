"""Test configuration: import paths and the ``gpu`` marker.

``-m "not gpu"`` runs on any host: the oracle against the reference's golden
vectors, the host validation and the C-ABI library's exported symbols.
``-m gpu`` runs the CUDA parity tests (a B200 is required).
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
for p in (ROOT, ROOT / "tests" / "golden", ROOT / "cid-engine_b200"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "fuzz: property-based differential tests")
    config.addinivalue_line("markers", "precision: decision-boundary and precision tests")


def cuda_ready() -> bool:
    import torch

    return torch.cuda.is_available()
