"""BDH RoPE apply with precomputed (cos, sin) tables — eager PyTorch forms.

BDH RoPE is pairwise with one phase per element (reference ``kernels/rope.py:1-10``)::

    y[2p]   = x[2p]   * cos[2p]   - x[2p+1] * sin[2p]
    y[2p+1] = x[2p+1] * cos[2p+1] + x[2p]   * sin[2p+1]

When ``x`` is lower precision than the tables (bf16 x, fp32 cos/sin) every product is cast
to x's dtype before the add, exactly as the reference (``kernels/rope.py:108-126``,
``bdh_baseline.py:50-54``) does, so results are bit-identical to it.

The table-free in-register form used on B200 lives in ``kernels.sm100_attn.rope_rotate``.
"""

from __future__ import annotations

from typing import Optional

import torch


def _validate_out(v: torch.Tensor, out: Optional[torch.Tensor], *cis: torch.Tensor) -> None:
    if out is None:
        return
    if out.shape != v.shape or out.device != v.device:
        raise ValueError(
            f"rope out= must match v shape/device, got out={tuple(out.shape)}/"
            f"{out.device} vs v={tuple(v.shape)}/{v.device}"
        )
    for t in (v, *cis):
        if out is t or (out.device == t.device and torch._C._overlaps(out, t)):
            raise ValueError("rope out= must not alias v or cis")


def _validate_inputs(v, cos, sin, out) -> None:
    if v.shape[-1] % 2 != 0:
        raise ValueError(f"RoPE last dim must be even, got {v.shape[-1]}")
    if cos.shape != sin.shape:
        raise ValueError(f"cos/sin shape mismatch: {cos.shape} vs {sin.shape}")
    if cos.shape[-1] != v.shape[-1]:
        raise ValueError(f"cos/sin last dim {cos.shape[-1]} != v last dim {v.shape[-1]}")
    try:
        torch.broadcast_shapes(v.shape[:-1], cos.shape[:-1])
    except RuntimeError as exc:
        raise ValueError(
            f"cos/sin leading dims {cos.shape[:-1]} are not broadcastable "
            f"with v leading dims {v.shape[:-1]}"
        ) from exc
    _validate_out(v, out, cos, sin)


def _validate_paired(v, cos_p, sin_p, out) -> None:
    if v.shape[-1] % 2 != 0:
        raise ValueError(f"RoPE last dim must be even, got {v.shape[-1]}")
    n_pairs = v.shape[-1] // 2
    if cos_p.shape != sin_p.shape:
        raise ValueError(f"paired cos/sin shape mismatch: {cos_p.shape} vs {sin_p.shape}")
    if tuple(cos_p.shape[-2:]) != (n_pairs, 2):
        raise ValueError(f"paired cis trailing dims must be ({n_pairs}, 2), got {cos_p.shape[-2:]}")
    try:
        torch.broadcast_shapes(v.shape[:-1], cos_p.shape[:-2])
    except RuntimeError as exc:
        raise ValueError(
            f"paired cis leading dims {cos_p.shape[:-2]} are not broadcastable "
            f"with v leading dims {v.shape[:-1]}"
        ) from exc
    _validate_out(v, out, cos_p, sin_p)


def _rotate(vp: torch.Tensor, cp: torch.Tensor, sp: torch.Tensor, v_dtype: torch.dtype):
    x0, x1 = vp[..., 0], vp[..., 1]
    c0, c1 = cp[..., 0], cp[..., 1]
    s0, s1 = sp[..., 0], sp[..., 1]
    if v_dtype != cp.dtype:
        y0 = (x0 * c0).to(v_dtype) + ((-x1) * s0).to(v_dtype)
        y1 = (x1 * c1).to(v_dtype) + (x0 * s1).to(v_dtype)
    else:
        y0 = x0 * c0 - x1 * s0
        y1 = x1 * c1 + x0 * s1
    return y0, y1


def _store(y0: torch.Tensor, y1: torch.Tensor, v: torch.Tensor, out: Optional[torch.Tensor]):
    if out is None:
        out = torch.empty(v.shape, dtype=v.dtype, device=v.device)
    op = out.view(*v.shape[:-1], -1, 2) if out.is_contiguous() else out.unflatten(-1, (-1, 2))
    op[..., 0] = y0
    op[..., 1] = y1
    return out


def eager_rope_rotate(v: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                      out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Rotate with full (…, T, N) tables (broadcast over leading dims)."""
    _validate_inputs(v, cos, sin, out)
    vp = v.unflatten(-1, (-1, 2))
    y0, y1 = _rotate(vp, cos.unflatten(-1, (-1, 2)), sin.unflatten(-1, (-1, 2)), v.dtype)
    return _store(y0, y1, v, out)


def rope_rotate_t1(v: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                   out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Single-position form (sequence length 1) of ``eager_rope_rotate``."""
    if v.dim() < 2 or v.shape[-2] != 1:
        raise ValueError(f"rope_rotate_t1 expects sequence length 1, got shape {tuple(v.shape)}")
    return eager_rope_rotate(v, cos, sin, out=out)


def rope_rotate_paired(v: torch.Tensor, cos_p: torch.Tensor, sin_p: torch.Tensor,
                       out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Rotate with pair-shaped tables ``(…, N/2, 2)``."""
    _validate_paired(v, cos_p, sin_p, out)
    y0, y1 = _rotate(v.unflatten(-1, (-1, 2)), cos_p, sin_p, v.dtype)
    return _store(y0, y1, v, out)


def rope_backward(g: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Adjoint of the rotation: dx0 = g0 c0 + g1 s1, dx1 = -g0 s0 + g1 c1."""
    gp = g.unflatten(-1, (-1, 2))
    cp = cos.unflatten(-1, (-1, 2))
    sp = sin.unflatten(-1, (-1, 2))
    g0, g1 = gp[..., 0], gp[..., 1]
    dx0 = g0 * cp[..., 0] + g1 * sp[..., 1]
    dx1 = -g0 * sp[..., 0] + g1 * cp[..., 1]
    return torch.stack((dx0, dx1), dim=-1).flatten(-2).to(g.dtype)


__all__ = ["eager_rope_rotate", "rope_rotate_t1", "rope_rotate_paired", "rope_backward"]
