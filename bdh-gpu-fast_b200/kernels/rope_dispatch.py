"""Env-gated RoPE dispatch (``BDH_ROPE_IMPL``), same surface as the reference
``kernels/rope_dispatch.py:32-99``.

    export BDH_ROPE_IMPL=eager   # default — table-driven pair rotation (bit-identical math)
    export BDH_ROPE_IMPL=fused   # with BDH_ATTN_IMPL=cuda_sm100 the model fuses RoPE into the
                                 # attention entry (in-register cos/sin, no tables)

``bdh_rope_rotate`` / ``bdh_rope_rotate_paired`` receive precomputed (cos, sin) tables and
apply them with the eager pair math under both settings; the table-free B200 kernel is reached
through ``kernels.attention_dispatch.bdh_rope_attn`` / ``bdh_rope_attn_decode`` (and
``kernels.sm100_attn.rope_rotate``), which take the model's ``freqs`` buffer instead.
"""

from __future__ import annotations

import os
from typing import Literal, Optional

import torch

from .rope import eager_rope_rotate, rope_rotate_paired, rope_rotate_t1

ImplName = Literal["eager", "fused"]
_VALID = ("eager", "fused")

_ROPE_IMPL_ENV: object = object()
_ROPE_IMPL_RESOLVED: ImplName = "eager"


def resolve_rope_impl(requested: str | None = None) -> ImplName:
    """Resolve ``BDH_ROPE_IMPL`` (or an explicit request) to ``eager`` or ``fused``."""
    global _ROPE_IMPL_ENV, _ROPE_IMPL_RESOLVED

    def _norm(raw: str) -> ImplName:
        raw = (raw or "eager").strip().lower()
        if raw not in _VALID:
            raise ValueError(f"BDH_ROPE_IMPL must be {'|'.join(_VALID)}, got {raw!r}")
        return raw  # type: ignore[return-value]

    if requested is not None:
        return _norm(requested)
    env = os.environ.get("BDH_ROPE_IMPL", "eager")
    if env == _ROPE_IMPL_ENV:
        return _ROPE_IMPL_RESOLVED
    resolved = _norm(env)
    _ROPE_IMPL_ENV = env
    _ROPE_IMPL_RESOLVED = resolved
    return resolved


def bdh_rope_rotate(v: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                    out: Optional[torch.Tensor] = None, *, impl: str | None = None) -> torch.Tensor:
    """Apply (cos, sin) tables to ``v`` (``impl`` validated; both settings use the pair math)."""
    resolve_rope_impl(impl)
    if v.dim() >= 2 and v.shape[-2] == 1:
        return rope_rotate_t1(v, cos, sin, out=out)
    return eager_rope_rotate(v, cos, sin, out=out)


def bdh_rope_rotate_paired(v: torch.Tensor, cos_p: torch.Tensor, sin_p: torch.Tensor,
                           out: Optional[torch.Tensor] = None, *,
                           impl: str | None = None) -> torch.Tensor:
    """Apply pair-shaped ``(…, N/2, 2)`` tables to ``v``."""
    resolve_rope_impl(impl)
    return rope_rotate_paired(v, cos_p, sin_p, out=out)


def backend_info(device: torch.device | None = None) -> dict:
    from .sm100_attn import has_cuda_kernel

    dev = device or torch.device("cuda" if torch.cuda.is_available() else "cpu")
    return {
        "BDH_ROPE_IMPL": resolve_rope_impl(),
        "fused_kernel": "sm100 in-register RoPE" if has_cuda_kernel() else "unavailable",
        "device": str(dev),
    }


__all__ = [
    "resolve_rope_impl",
    "bdh_rope_rotate",
    "bdh_rope_rotate_paired",
    "backend_info",
    "eager_rope_rotate",
    "rope_rotate_paired",
    "rope_rotate_t1",
]
