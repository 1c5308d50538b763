"""Test markers and shared helpers. `gpu`: needs a B200 (sm_100a) and the built CUDA library; everything else runs
on the CPU (`python -m pytest tests/ -m "not gpu"`)."""

from __future__ import annotations

import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
GOLDEN = ROOT / "tests" / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs an NVIDIA B200 (sm_100a) and the built libjeffb200.so")
    config.addinivalue_line("markers", "slow: a long CPU oracle run")


def pytest_collection_modifyitems(config: pytest.Config, items: list[pytest.Item]) -> None:
    import torch

    if torch.cuda.is_available() or os.environ.get("JEFF_B200_FORCE_GPU_TESTS"):
        return
    skip = pytest.mark.skip(reason="needs a CUDA GPU (torch.cuda.is_available() is False)")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)
