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


def config2_case():
    """The config-2-width case of golden_config2_bf16.npz (tests/golden/config2_case.py)."""
    if str(GOLDEN) not in sys.path:
        sys.path.insert(0, str(GOLDEN))
    import config2_case

    return config2_case


def reference_bf16_floor(g) -> float:
    """The reference's own execution-to-execution spread of its config-2-width bf16 logits
    (golden_config2_bf16.npz): the same autocast run with one CPU thread and with ATen's GEMMs
    instead of oneDNN's, each against the stored run. Only fp32 accumulation orders differ."""
    import numpy as np

    ref = g["logits_bf16_cuda_policy"].astype(np.float64)

    def rel(a):
        return float(np.linalg.norm(a.astype(np.float64) - ref) / np.linalg.norm(ref))

    return max(rel(g["logits_bf16_cuda_policy_1thread"]), rel(g["logits_bf16_cuda_policy_aten_gemm"]))
