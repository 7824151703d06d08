"""Shared pytest setup: the `gpu` marker, import paths and GPU fixtures."""

from __future__ import annotations

import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

def _reference_root() -> Path | None:
    """The phew reference checkout: $PHEW_REFERENCE, else wherever an
    importable ``phew`` package lives; None when neither exists (the tests
    that drive the reference's own code are then skipped)."""
    env = os.environ.get("PHEW_REFERENCE")
    if env:
        return Path(env)
    import importlib.util

    spec = importlib.util.find_spec("phew")
    if spec is not None and spec.origin:
        return Path(spec.origin).resolve().parent.parent
    return None


REFERENCE = _reference_root()


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
    return REFERENCE is not None and (REFERENCE / "phew" / "__init__.py").exists()
