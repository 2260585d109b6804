"""Autograd for strict-tril BDH attention ``O = tril(Q K^T, -1) V`` (same surface as the
reference ``kernels/attention_bwd.py:218-325``).

Analytic gradients (no softmax, so no saved statistics are needed; M is recomputed):

    M  = tril(Q K^T, -1)          dS = tril(dO V^T, -1)
    dQ = dS K                     dK = dS^T Q
    dV = M^T dO                   (summed over heads when V has one head)

* ``impl="eager"``: dense PyTorch recompute (reference ``attention_bwd.py:45-83``).
* ``impl="cuda_sm100"``: forward and backward both run in libbdh_sm100.so (tcgen05 kernels);
  the self-attention form returns ``dQ + dK`` for Q (K is Q, reference ``:284-291``).
* ``RopeTrilSelfAttnFn``: RoPE fused into the attention; the backward folds the RoPE adjoint
  (reference ``kernels/rope.py:540-557``) into the dQ epilogue and returns the gradient of
  the unrotated latent.

Opt-in exactly as in the reference: ``BDH_ATTN_AUTOGRAD=1`` or ``use_fn=True``.
"""

from __future__ import annotations

import os
from typing import Optional

import torch

from .attention import eager_tril_attn

_SM100 = "cuda_sm100"


def analytic_tril_attn_backward(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor,
                                dO: torch.Tensor):
    """Dense analytic gradients (dQ, dK, dV) of ``tril(Q K^T, -1) V``; dV shaped like V."""
    B, H, T, _ = Q.shape
    D = V.size(-1)
    shared_v = V.size(1) == 1 and H != 1
    Vh = V.expand(B, H, T, D) if shared_v else V
    M = (Q @ K.transpose(-2, -1)).tril(diagonal=-1)
    dS = (dO @ Vh.transpose(-2, -1)).tril(diagonal=-1)
    dQ = dS @ K
    dK = dS.transpose(-2, -1) @ Q
    dVh = M.transpose(-2, -1) @ dO
    dV = dVh.sum(dim=1, keepdim=True) if shared_v else dVh
    return dQ, dK, dV


def _normalize_impl(impl: Optional[str]) -> str:
    from .attention_dispatch import resolve_attn_impl

    return resolve_attn_impl(impl if impl is not None else os.environ.get("BDH_ATTN_IMPL", "eager"))


def _forward_impl(Q, K, V, impl: str) -> torch.Tensor:
    if impl == _SM100:
        from .sm100_attn import tril_score_v

        return tril_score_v(Q, K, V)
    return eager_tril_attn(Q, K, V)


class StrictTrilAttnFn(torch.autograd.Function):
    """``(Q, K, V, impl) -> out`` with analytic ``(dQ, dK, dV, None)`` backward."""

    @staticmethod
    def forward(ctx, Q, K, V, impl: str):
        ctx.impl = impl
        ctx.save_for_backward(Q, K, V)
        with torch.no_grad():
            return _forward_impl(Q, K, V, impl)

    @staticmethod
    def backward(ctx, dO):
        Q, K, V = ctx.saved_tensors
        if ctx.impl == _SM100:
            from .sm100_attn import tril_score_v_bwd

            dQ, dK, dV = tril_score_v_bwd(Q, K, V, dO.contiguous())
        else:
            dQ, dK, dV = analytic_tril_attn_backward(Q, K, V, dO)
        return dQ, dK, dV, None


class StrictTrilSelfAttnFn(torch.autograd.Function):
    """Self form ``(Q, V, impl) -> out`` (K is Q); backward returns ``(dQ + dK, dV, None)``."""

    @staticmethod
    def forward(ctx, Q, V, impl: str):
        ctx.impl = impl
        ctx.save_for_backward(Q, V)
        with torch.no_grad():
            return _forward_impl(Q, Q, V, impl)

    @staticmethod
    def backward(ctx, dO):
        Q, V = ctx.saved_tensors
        if ctx.impl == _SM100:
            from .sm100_attn import tril_score_v_bwd

            dQt, _, dV = tril_score_v_bwd(Q, Q, V, dO.contiguous())
            return dQt, dV, None
        dQ, dK, dV = analytic_tril_attn_backward(Q, Q, V, dO)
        return dQ + dK, dV, None


class RopeTrilSelfAttnFn(torch.autograd.Function):
    """RoPE fused with self-attention on B200: ``(Q, V, freqs, pos0) -> (out, QR)``.

    Forward: QR = RoPE(Q) (in-register cos/sin, ``out_kr`` filled when given), then
    ``tril(QR QR^T, -1) V``. Backward: one native call gives the gradient of the unrotated
    latent (the RoPE adjoint is fused into the dQ epilogue) and dV. QR is returned so callers
    (cache writes) can use it; it carries no gradient of its own.
    """

    @staticmethod
    def forward(ctx, Q, V, freqs, pos0: int, qr_out: Optional[torch.Tensor], relu_input: bool = False):
        from .sm100_attn import rope_rotate, tril_score_v

        with torch.no_grad():
            if qr_out is not None and qr_out.dtype != Q.dtype:
                # a cache slot in another storage dtype: attend in Q's dtype, store the cast
                QR = rope_rotate(Q, freqs, pos0, relu_input=relu_input)
                qr_out.copy_(QR)
            else:
                QR = rope_rotate(Q, freqs, pos0, out=qr_out, relu_input=relu_input)
            out = tril_score_v(QR, QR, V)
        ctx.pos0 = int(pos0)
        ctx.relu_input = bool(relu_input)
        if relu_input:
            ctx.save_for_backward(QR, V, freqs, Q)
        else:
            ctx.save_for_backward(QR, V, freqs)
        ctx.mark_non_differentiable(QR)
        # QR carries no gradient: do not let autograd build a zero (B, H, T, N) tensor for it
        ctx.set_materialize_grads(False)
        return out, QR

    @staticmethod
    def backward(ctx, dO, _dQR):
        from .sm100_attn import tril_score_v_bwd

        if dO is None:
            return None, None, None, None, None, None
        QR, V, freqs = ctx.saved_tensors[:3]
        dQ, _, dV = tril_score_v_bwd(QR, QR, V, dO.contiguous(), freqs=freqs, pos0=ctx.pos0)
        if ctx.relu_input:
            dQ = dQ * (ctx.saved_tensors[3] > 0).to(dQ.dtype)
        return dQ, dV, None, None, None, None


def strict_tril_attn(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, *,
                     impl: Optional[str] = None, use_fn: Optional[bool] = None) -> torch.Tensor:
    """Strict-tril score@V with the optional analytic autograd Function.

    use_fn True → Function (self form when ``Q is K``); False → plain forward; None → env
    ``BDH_ATTN_AUTOGRAD``.
    """
    if use_fn is None:
        use_fn = _env_autograd_enabled()
    name = _normalize_impl(impl)
    if use_fn:
        if Q is K:
            return StrictTrilSelfAttnFn.apply(Q, V, name)
        return StrictTrilAttnFn.apply(Q, K, V, name)
    return _forward_impl(Q, K, V, name)


def _env_autograd_enabled() -> bool:
    raw = os.environ.get("BDH_ATTN_AUTOGRAD", "").strip().lower()
    return raw in ("1", "true", "yes", "on")


__all__ = [
    "analytic_tril_attn_backward",
    "StrictTrilAttnFn",
    "StrictTrilSelfAttnFn",
    "RopeTrilSelfAttnFn",
    "strict_tril_attn",
    "_env_autograd_enabled",
]
