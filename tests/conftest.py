"""Shared pytest setup: the `gpu` marker, import paths and GPU fixtures."""

from __future__ import annotations

import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

REFERENCE = Path(os.environ.get("PHEW_REFERENCE", "/root/reference"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def has_gpu() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:  # noqa: BLE001
        return False


def pytest_collection_modifyitems(config, items):
    if has_gpu():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def mx():
    """The product namespace on cuda:0 (fails loudly if the library is missing)."""
    import phew_b200.mx as bmx

    bmx.core.device()
    return bmx


@pytest.fixture(scope="session")
def oracle():
    from oracle import mlx_cpu

    return mlx_cpu


def reference_importable() -> bool:
    return (REFERENCE / "phew" / "__init__.py").exists()
