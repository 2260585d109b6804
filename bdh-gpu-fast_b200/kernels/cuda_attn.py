"""``kernels.cuda_attn`` of the reference, served by the sm_100a library.

Same public names as the reference module (``kernels/cuda_attn.py``: ``tril_score_v`` :391-414,
``tril_decode`` :490-502, the eager references :293-310 / :417-448, ``has_cuda_ext`` /
``has_cuda_kernel`` / ``ext_status`` :91-100, :505-513, the tile pickers :134-290), so callers
written against it import this module unchanged. Differences on purpose:

* ``tril_score_v`` / ``tril_decode`` run the B200 kernels through ``bdh_sm100_ext`` (the
  PyTorch extension with the reference module's names, ``kernels.sm100_ext``) as the reference
  calls ``bdh_cuda_ext`` (``import bdh_cuda_ext as _ext``, :85), or through the ctypes binding
  of the same library (``kernels.sm100_attn``) when the extension is not built. They never fall
  back: CPU tensors or a missing library raise instead of silently returning the reference's
  CPU result (``cuda_attn.py:401-409``). Shapes are checked first, with the reference's
  ValueError messages (:103-131);
* the ``*_tiled_ref`` CPU mirrors of the reference's CUDA tiling compute the same values as the
  plain references and are kept as aliases;
* the tile pickers describe this library's fixed tcgen05 tiles (128-row query blocks, 128/256-key
  blocks; 16..128 cached rows per decode CTA) and exist for API compatibility only.
"""

from __future__ import annotations

import torch

from . import sm100_attn as _sm
from . import sm100_ext as _sx

CUDA_TILE_M = 128
CUDA_TILE_N = 128
CUDA_TILE_D = 256
CUDA_TILE_M_MAX = 256
CUDA_TILE_N_MAX = 256
CUDA_DECODE_TILE_N = 16
CUDA_DECODE_TILE_N_MAX = 128


def has_cuda_ext() -> bool:
    """True if the native path imports (the extension, else the library through ctypes)."""
    return _sx.try_load_ext() is not None or _sm.has_cuda_ext()


def has_cuda_kernel() -> bool:
    return has_cuda_ext() and torch.cuda.is_available()


def ext_status() -> str:
    ext = _sx.try_load_ext()
    binding = "bdh_sm100_ext" if ext is not None else f"ctypes (bdh_sm100_ext: {_sx.ext_error()!r})"
    return f"{_sm.ext_status()} binding={binding}"


def pick_cuda_cold_tiles(T: int, Dk: int, *args, **kwargs):
    """(query-tile rows, key-tile cols) of the forward: the tcgen05 tiles (API compatibility)."""
    return CUDA_TILE_M, CUDA_TILE_N


def pick_cuda_decode_tile_n(S: int, *args, **kwargs) -> int:
    """Cached rows per decode CTA at most (the split plan picks 16..128; API compatibility)."""
    return CUDA_DECODE_TILE_N_MAX


def tril_score_v_ref(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """Eager reference ``(q @ k.mT).tril(-1) @ v`` (V heads broadcast), any device."""
    _sm._check_cold_shapes(q, k, v)
    return (q @ k.transpose(-2, -1)).tril(diagonal=-1) @ v


def tril_score_v_tiled_ref(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *,
                           tile_m: int | None = None, tile_n: int | None = None) -> torch.Tensor:
    """Same values as ``tril_score_v_ref`` (the reference's CPU mirror of its CUDA tiling)."""
    return tril_score_v_ref(q, k, v)


def tril_score_v(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """``(q @ k.mT).tril(-1) @ v`` on the sm_100a tensor cores (CUDA tensors only)."""
    _sm._check_cold_shapes(q, k, v)
    ext = _sx.try_load_ext()
    if ext is not None:
        return ext.tril_score_v(q, k, v)
    return _sm.tril_score_v(q, k, v)


def tril_decode_ref(q: torch.Tensor, k_past: torch.Tensor, v_past: torch.Tensor) -> torch.Tensor:
    """Eager reference ``(q @ k_past.mT) @ v_past`` (S = 0 gives zeros), any device."""
    B, H, Tq, S, D = _sm._check_decode_shapes(q, k_past, v_past)
    if S == 0:
        return q.new_zeros(B, H, Tq, D)
    return (q @ k_past.transpose(-2, -1)) @ v_past


def tril_decode_tiled_ref(q: torch.Tensor, k_past: torch.Tensor, v_past: torch.Tensor, *,
                          tile_n: int | None = None) -> torch.Tensor:
    """Same values as ``tril_decode_ref``."""
    return tril_decode_ref(q, k_past, v_past)


def tril_decode(q: torch.Tensor, k_past: torch.Tensor, v_past: torch.Tensor) -> torch.Tensor:
    """``(q @ k_past.mT) @ v_past`` streaming the cache on the GPU (CUDA tensors only)."""
    _sm._check_decode_shapes(q, k_past, v_past)
    ext = _sx.try_load_ext()
    if ext is not None:
        return ext.tril_decode(q, k_past, v_past)
    return _sm.tril_decode(q, k_past, v_past)
