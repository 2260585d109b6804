"""Eager (pure PyTorch) strict-tril attention: the reference semantics as plain tensor ops.

These are the ``eager`` backend of the dispatch (the reference default) and the math the
sm_100a kernels must reproduce:

* ``eager_tril_attn``   = reference ``kernels/attention.py:27-40``: full T x T scores, strict
  lower triangle (``tril(diagonal=-1)``), then ``@ V``; no softmax, no scale.
* ``eager_decode_attn`` = reference ``kernels/attention.py:193-219,1356-1366``: scores against
  the packed past only (every cached key precedes the query), then ``@ V_past``.

The reference's blocked (CPU-tiled) and Triton backends are not part of this package.
"""

from __future__ import annotations

import torch


def eager_tril_attn(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor) -> torch.Tensor:
    """``(Q @ K.mT).tril(-1) @ V``; V may have one head (broadcast over Q's heads)."""
    scores = Q @ K.transpose(-2, -1)
    scores = scores.tril(diagonal=-1)
    return scores @ V


def _two_gemm_decode(Q: torch.Tensor, K_past: torch.Tensor, V_past: torch.Tensor) -> torch.Tensor:
    """``(Q @ K_past.mT) @ V_past`` — no mask: the past never contains the query itself."""
    return (Q @ K_past.transpose(-2, -1)) @ V_past


def eager_decode_attn(Q: torch.Tensor, K_past: torch.Tensor, V_past: torch.Tensor) -> torch.Tensor:
    """Eager decode; an empty past gives zeros of shape ``(B, H, Tq, D)``."""
    if K_past.size(2) == 0:
        B, H, Tq, _ = Q.shape
        return Q.new_zeros(B, H, Tq, V_past.size(-1))
    return _two_gemm_decode(Q, K_past, V_past)


__all__ = ["eager_tril_attn", "eager_decode_attn", "_two_gemm_decode"]
