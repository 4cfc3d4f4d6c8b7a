"""Shared pytest setup: the ``gpu`` marker, the repo root on ``sys.path`` and the package loader."""

from __future__ import annotations

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (a B200) and the built native library")


def _cuda_available() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:  # pragma: no cover - torch import failure
        return False


def pytest_collection_modifyitems(config, items):
    if _cuda_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def pkg():
    """The ``rf-detr-jax_b200`` package, imported as ``rfdetr_jax_b200``."""
    import __graft_entry__

    return __graft_entry__.load_package()


@pytest.fixture
def tuning(pkg):
    """``tuning(name, value)`` sets one of the library's process-wide tuning knobs
    (``rfdetr_set_tuning``) for the test; every knob it touched returns to its default after."""
    touched = []

    def set_knob(name, value):
        touched.append(name)
        pkg._native.set_tuning(name, value)

    yield set_knob
    for name in touched:
        pkg._native.set_tuning(name, None)
