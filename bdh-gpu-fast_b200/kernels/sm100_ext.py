"""Loader of ``bdh_sm100_ext``: the PyTorch extension that binds libbdh_sm100.so under the names
of the reference's native module ``bdh_cuda_ext`` (csrc/tril_attn_bind.cpp:25-40:
``tril_score_v``, ``tril_decode``, ``has_cuda``), plus ``tril_score_v_bwd``, ``rope_rotate``,
``rope_tril_score_v``, ``rope_tril_decode`` and the fused layer's ``latent_encode``,
``latent_gate_dec``, ``layer_norm`` and ``residual_layer_norm``.

The extension is a C++ module built in-tree next to the library
(``python bdh-gpu-fast_b200/build_lib.py --ext``; ``__graft_entry__.build()`` does it). It calls
the same C-ABI entry points as the ctypes binding of ``kernels.sm100_attn`` (one library
instance in the process: the extension finds it by its soname), without the per-call ctypes
argument marshalling.
"""

from __future__ import annotations

import importlib.util
import sys
from pathlib import Path
from types import ModuleType
from typing import Optional

import torch  # noqa: F401 - the extension links against torch's shared libraries

from . import sm100_attn

EXT_PATH = Path(__file__).resolve().parent.parent / "bdh_sm100_ext.so"

_ext: Optional[ModuleType] = None
_ext_error: Optional[BaseException] = None


def load_ext() -> ModuleType:
    """Import (once) and return ``bdh_sm100_ext``; raises ImportError when it is not built or
    does not match the library's ABI."""
    global _ext, _ext_error
    if _ext is not None:
        return _ext
    try:
        if not EXT_PATH.exists():
            raise ImportError(f"{EXT_PATH} is not built (python bdh-gpu-fast_b200/build_lib.py --ext)")
        sm100_attn.load_library()  # the library first: the extension then binds this instance
        spec = importlib.util.spec_from_file_location("bdh_sm100_ext", EXT_PATH)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        if mod.abi_version() != sm100_attn.ABI_VERSION:
            raise ImportError(f"{EXT_PATH}: library ABI {mod.abi_version()}, expected "
                              f"{sm100_attn.ABI_VERSION}")
    except BaseException as exc:  # noqa: BLE001 - remembered for ext_status()
        _ext_error = exc
        raise
    sys.modules.setdefault("bdh_sm100_ext", mod)
    _ext = mod
    return mod


def try_load_ext() -> Optional[ModuleType]:
    """The extension, or None when it is not built or failed to load (remembered: not retried)."""
    if _ext is None and _ext_error is not None:
        return None
    try:
        return load_ext()
    except BaseException:  # noqa: BLE001
        return None


def ext_error() -> Optional[BaseException]:
    return _ext_error


def model_ops() -> ModuleType:
    """The fused layer's library entries (``latent_encode``, ``tril_score_v``, ``layer_norm``,
    ``latent_gate_dec``, ``residual_layer_norm``, same signatures): from the extension when it is
    built and ``BDH_SM100_EXT`` is not ``0``, else the ctypes binding. Both call the same C-ABI
    entries with the same arguments (the same bits); the extension costs less host time per
    call, which is what an eager step of the model spends between its kernels."""
    import os

    if os.environ.get("BDH_SM100_EXT", "1") != "0":
        ext = try_load_ext()
        if ext is not None:
            return ext
    return sm100_attn
