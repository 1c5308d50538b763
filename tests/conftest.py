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

# The reference's client and runtime packages, where a checkout exists (the development machine; never the GPU box):
# on the path before anything imports jeff_b200, so jeff_b200.errors binds the reference's own result and error
# classes and the engine tests run against them. JEFF_B200_LOCAL_TYPES=1 keeps them off the path (the stand-in types
# are then tested, as on a machine without the reference).
REFERENCE = Path(os.environ.get("JEFF_REFERENCE", "/root/reference"))
REFERENCE_PACKAGES = [REFERENCE / "packages" / "python" / "src", REFERENCE / "runtime" / "python" / "src"]
if not os.environ.get("JEFF_B200_LOCAL_TYPES") and all(p.is_dir() for p in REFERENCE_PACKAGES):
    for package_dir in REFERENCE_PACKAGES:
        if str(package_dir) not in sys.path:
            sys.path.append(str(package_dir))


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
