"""Test configuration: import paths for the package and the (test-only) oracle, the ``gpu``
marker, and shared helpers."""

import os
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
PKG = REPO / "bdh-gpu-fast_b200"
ORACLE = REPO / "oracle"
GOLDEN = Path(__file__).resolve().parent / "golden"

for p in (str(PKG), str(ORACLE)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an NVIDIA B200 (sm_100a) GPU")


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this environment")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(autouse=True)
def _clean_env(monkeypatch):
    for k in ("BDH_ATTN_IMPL", "BDH_ATTN_AUTOGRAD", "BDH_ATTN_AUTO", "BDH_ATTN_AUTO_THRESHOLD",
              "BDH_ATTN_AUTO_COLD_THRESHOLD", "BDH_ROPE_IMPL"):
        monkeypatch.delenv(k, raising=False)
    yield


def golden(name: str):
    import numpy as np

    return np.load(GOLDEN / f"golden_{name}.npz")
