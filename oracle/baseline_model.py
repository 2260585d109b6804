"""CPU restatement of the reference's baseline BDH forward — TEST INFRASTRUCTURE ONLY (the
timed CPU reference arm and a checker; never part of the product path).

Follows ``bdh_baseline.py`` (eval mode, dropout off): the embedding and its LayerNorm
(:115-119), per layer ``x @ encoder`` + ReLU (:121-124), the attention module with its own
RoPE (:42-72: phases ``t * freq``, ``(phase mod 1) * 2 pi``, pairwise rotation), LayerNorm,
``yKV @ encoder_v`` + ReLU, the sparse product, the decoder product on the transposed latent
(:126-142), the residual double LayerNorm (:143-144), and ``x @ lm_head`` (:146). Everything is
torch CPU fp32. The strictly causal score-times-V product is pluggable: the reference's own C++
extension (``tril_score_v_cpu`` of ``csrc/tril_attn_cpu.cpp``, built into oracle/_ref) when it
is available, else the same arithmetic in torch (``(QR @ QR.mT).tril(-1) @ V``).

Pinned by tests/test_oracle_golden.py against the reference's own fp32 logits.
"""

from __future__ import annotations

import math
from typing import Callable, Optional

import torch
import torch.nn.functional as F


def eager_tril_score_v(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    return (q @ k.mT).tril(diagonal=-1) @ v


def reference_tril_score_v() -> Optional[Callable]:
    """The reference CPU extension's ``tril_score_v_cpu`` from oracle/_ref, or None."""
    try:
        import build_ref

        ext = build_ref.load_module()
    except Exception:  # noqa: BLE001 - not built on this host
        return None
    return lambda q, k, v: ext.tril_score_v_cpu(q, k, v)


@torch.no_grad()
def baseline_forward(idx: torch.Tensor, weights: dict, n_layer: int, n_head: int,
                     attn: Optional[Callable] = None) -> torch.Tensor:
    """Logits (B, T, V) in fp32. weights: embed (V, D), encoder / encoder_v (nh, D, N),
    decoder (nh*N, D), lm_head (D, V), freqs (N,) — torch CPU fp32 tensors."""
    attn = attn or eager_tril_score_v
    B, T = idx.shape
    emb, enc, enc_v = weights["embed"], weights["encoder"], weights["encoder_v"]
    dec, head = weights["decoder"], weights["lm_head"]
    D = emb.shape[1]
    N = enc.shape[-1]
    freqs = weights["freqs"].reshape(1, 1, 1, N).float()
    phase = torch.arange(T, dtype=torch.float32).view(1, 1, T, 1) * freqs
    phase = (phase % 1) * (2 * math.pi)
    cos, sin = torch.cos(phase), torch.sin(phase)

    def ln(t):
        return F.layer_norm(t, (D,))

    def rotate(v):
        pair = torch.stack((-v[..., 1::2], v[..., ::2]), dim=-1).view(v.shape)
        return v * cos + pair * sin

    x = ln(F.embedding(idx, emb).unsqueeze(1))  # B, 1, T, D
    for _ in range(n_layer):
        xs = F.relu(x @ enc)  # B, nh, T, N
        qr = rotate(xs)
        y = ln(attn(qr, qr, x))
        ys = F.relu(y @ enc_v)
        xy = xs * ys
        ymlp = xy.transpose(1, 2).reshape(B, 1, T, N * n_head) @ dec
        x = ln(x + ln(ymlp))
    return x.view(B, T, D) @ head
