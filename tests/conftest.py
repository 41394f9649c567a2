"""Test configuration: repository root on sys.path, the ``gpu`` marker, package helpers.

The package folder is ``0709_b200`` (not a valid identifier), so tests import
modules through ``importlib``: ``mod("runtime.store")``.
"""

from __future__ import annotations

import importlib
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REPO = ROOT
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

PKG = "0709_b200"


def mod(name: str):
    return importlib.import_module(f"{PKG}.{name}" if name else PKG)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU and the compiled CUDA extension")


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)
