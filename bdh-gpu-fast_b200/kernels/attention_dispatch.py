"""Env-gated dispatch for BDH strict-tril attention — the reference API
(``kernels/attention_dispatch.py:169-486``) with the B200 backend.

Backends (``BDH_ATTN_IMPL``)::

    export BDH_ATTN_IMPL=eager        # default — full T x T scores, tril(-1), @ V (PyTorch)
    export BDH_ATTN_IMPL=cuda_sm100   # libbdh_sm100.so: tcgen05 forward/backward, HBM decode
    export BDH_ATTN_IMPL=cuda         # accepted alias of cuda_sm100 (the native backend)
    export BDH_ATTN_AUTOGRAD=1        # analytic autograd.Function (native bwd for cuda_sm100)
    export BDH_ATTN_AUTO=1            # long-sequence switch eager -> cuda_sm100 (CUDA tensors)
    export BDH_ATTN_AUTO_THRESHOLD=512
    export BDH_ATTN_AUTO_COLD_THRESHOLD=...   # unset -> mirrors AUTO_THRESHOLD

The reference's ``blocked`` / ``online`` / ``triton`` backends are not part of this package:
asking for them raises ``ValueError``. ``cuda_sm100`` never falls back: a missing library,
CPU tensors or a failing launch raise instead of silently running another implementation.

New fused entries (RoPE applied inside, from the model's ``freqs`` buffer):
``bdh_rope_attn`` (cold/prefill, returns ``(out, QR)``) and ``bdh_rope_attn_decode``
(T=1 decode that also writes the rotated query into the cache slot).
"""

from __future__ import annotations

import os
from typing import Literal, Optional, Tuple

import torch

from .attention import eager_decode_attn, eager_tril_attn
from .attention_bwd import RopeTrilSelfAttnFn, _env_autograd_enabled, strict_tril_attn

ImplName = Literal["eager", "cuda_sm100"]
_VALID = ("eager", "cuda_sm100")
_ALIASES = {"cuda": "cuda_sm100"}
_REMOVED = ("blocked", "online", "triton")

DEFAULT_ATTN_AUTO_THRESHOLD = 512
DEFAULT_BLOCK_DECODE = 512  # kept for signature compatibility of bdh_attn_decode
_TRUTHY = ("1", "true", "yes", "on")

_ATTN_IMPL_ENV: object = object()
_ATTN_IMPL_RESOLVED: ImplName = "eager"


def resolve_attn_impl(requested: str | None = None) -> ImplName:
    """Resolve ``BDH_ATTN_IMPL`` (or an explicit request) to ``eager`` / ``cuda_sm100``."""
    global _ATTN_IMPL_ENV, _ATTN_IMPL_RESOLVED

    def _normalize(raw: str) -> ImplName:
        raw = (raw or "eager").strip().lower()
        raw = _ALIASES.get(raw, raw)
        if raw in _REMOVED:
            raise ValueError(
                f"BDH_ATTN_IMPL={raw!r} is not provided by this package "
                f"(use eager or cuda_sm100)"
            )
        if raw not in _VALID:
            raise ValueError(f"BDH_ATTN_IMPL must be {'|'.join(_VALID)}|cuda, got {raw!r}")
        return raw  # type: ignore[return-value]

    if requested is not None:
        return _normalize(requested)
    env = os.environ.get("BDH_ATTN_IMPL", "eager")
    if env == _ATTN_IMPL_ENV:
        return _ATTN_IMPL_RESOLVED
    resolved = _normalize(env)
    _ATTN_IMPL_ENV = env
    _ATTN_IMPL_RESOLVED = resolved
    return resolved


def attn_auto_enabled() -> bool:
    """True when ``BDH_ATTN_AUTO`` is truthy (``1|true|yes|on``). Default off."""
    return os.environ.get("BDH_ATTN_AUTO", "").strip().lower() in _TRUTHY


def _int_env(name: str, default: Optional[int]) -> Optional[int]:
    raw = os.environ.get(name, "").strip()
    if not raw:
        return default
    try:
        v = int(raw)
    except ValueError as exc:
        raise ValueError(f"{name} must be an int, got {raw!r}") from exc
    if v < 0:
        raise ValueError(f"{name} must be >= 0, got {v}")
    return v


def attn_auto_threshold() -> int:
    """Decode past-length threshold of the AUTO switch (default 512)."""
    return int(_int_env("BDH_ATTN_AUTO_THRESHOLD", DEFAULT_ATTN_AUTO_THRESHOLD))


def attn_auto_cold_threshold() -> int:
    """Cold/prefill length threshold; mirrors ``attn_auto_threshold`` when unset."""
    v = _int_env("BDH_ATTN_AUTO_COLD_THRESHOLD", None)
    return attn_auto_threshold() if v is None else v


def _native_usable(t: Optional[torch.Tensor]) -> bool:
    from .sm100_attn import has_cuda_kernel

    return t is not None and t.is_cuda and has_cuda_kernel()


def _resolve_auto(length: int, threshold: int, probe: Optional[torch.Tensor]) -> ImplName:
    if int(length) <= int(threshold):
        return "eager"
    return "cuda_sm100" if _native_usable(probe) else "eager"


def resolve_decode_impl(past_len: int, requested: str | None = None,
                        probe: Optional[torch.Tensor] = None) -> ImplName:
    """T=1 decode backend: ``resolve_attn_impl`` plus the optional AUTO long-past switch."""
    name = resolve_attn_impl(requested)
    if name != "eager" or not attn_auto_enabled():
        return name
    return _resolve_auto(past_len, attn_auto_threshold(), probe)


def resolve_cold_impl(seq_len: int, requested: str | None = None,
                      probe: Optional[torch.Tensor] = None) -> ImplName:
    """Cold/prefill backend: ``resolve_attn_impl`` plus the optional AUTO long-T switch."""
    name = resolve_attn_impl(requested)
    if name != "eager" or not attn_auto_enabled():
        return name
    return _resolve_auto(seq_len, attn_auto_cold_threshold(), probe)


def bdh_attn(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, *, impl: str | None = None,
             use_autograd_fn: Optional[bool] = None) -> torch.Tensor:
    """``tril(Q @ K^T, -1) @ V`` with the selected backend (reference ``:360-405``).

    With ``use_autograd_fn`` (or ``BDH_ATTN_AUTOGRAD=1``) the forward is wrapped in the
    analytic autograd Function (``StrictTrilSelfAttnFn`` when ``Q is K``).
    """
    name = resolve_cold_impl(int(Q.size(2)), requested=impl, probe=Q)
    if use_autograd_fn is None:
        use_autograd_fn = _env_autograd_enabled()
    if use_autograd_fn:
        return strict_tril_attn(Q, K, V, impl=name, use_fn=True)
    if name == "eager":
        return eager_tril_attn(Q, K, V)
    from .sm100_attn import tril_score_v

    return tril_score_v(Q, K, V)


def bdh_attn_decode(Q: torch.Tensor, K_past: torch.Tensor, V_past: torch.Tensor, *,
                    impl: str | None = None, block_size: int = DEFAULT_BLOCK_DECODE) -> torch.Tensor:
    """Attend new queries to the packed past only (reference ``:408-444``)."""
    del block_size
    name = resolve_decode_impl(int(K_past.size(2)), requested=impl, probe=Q)
    if name == "eager":
        return eager_decode_attn(Q, K_past, V_past)
    from .sm100_attn import tril_decode

    return tril_decode(Q, K_past, V_past)


def bdh_rope_attn(Q: torch.Tensor, V: torch.Tensor, freqs: torch.Tensor, rope_start: int = 0, *,
                  impl: str | None = None, qr_out: Optional[torch.Tensor] = None,
                  use_autograd_fn: Optional[bool] = None,
                  relu_input: bool = False) -> Tuple[torch.Tensor, torch.Tensor]:
    """Fused RoPE + strict-tril self attention: returns ``(out, QR)``.

    ``Q`` is the unrotated latent (B,H,T,N) (any strides with a contiguous last dim, e.g. the
    permuted encoder output); ``freqs`` the model's (…, N) fp32 buffer; ``qr_out`` an optional
    destination for QR (a cache slot). On ``cuda_sm100`` RoPE runs in-register (no cos/sin
    tables) and autograd (when enabled or when Q requires grad) differentiates through the
    fused native backward. On ``eager`` the tables are built and applied with PyTorch ops.
    ``relu_input``: Q is the encoder pre-activation and ``relu(Q)`` is rotated (the ReLU is
    folded into the RoPE read on ``cuda_sm100``).
    """
    name = resolve_cold_impl(int(Q.size(2)), requested=impl, probe=Q)
    if name == "cuda_sm100":
        if V.dtype != Q.dtype:
            V = V.to(Q.dtype)
        out, QR = RopeTrilSelfAttnFn.apply(Q, V, freqs, int(rope_start), qr_out, bool(relu_input))
        return out, QR
    from .rope import eager_rope_rotate

    if relu_input:
        Q = torch.relu(Q)
    cos, sin = rope_tables(freqs, Q.size(2), rope_start, Q.device)
    QR = eager_rope_rotate(Q, cos, sin, out=qr_out)
    return bdh_attn(QR, QR, V, impl="eager", use_autograd_fn=use_autograd_fn), QR


def bdh_rope_attn_decode(Q: torch.Tensor, K_past: torch.Tensor, V_past: torch.Tensor,
                         freqs: torch.Tensor, pos: int, *, impl: str | None = None,
                         kr_slot: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Fused decode step: rotate Q to ``pos``, write it to ``kr_slot`` (optional) and attend to
    the packed past (which excludes the new position)."""
    name = resolve_decode_impl(int(K_past.size(2)), requested=impl, probe=Q)
    if name == "cuda_sm100":
        from .sm100_attn import tril_decode

        return tril_decode(Q, K_past, V_past, freqs=freqs, pos=int(pos), kr_slot=kr_slot)
    from .rope import eager_rope_rotate

    cos, sin = rope_tables(freqs, Q.size(2), pos, Q.device)
    QR = eager_rope_rotate(Q, cos, sin)
    if kr_slot is not None:
        kr_slot.copy_(QR)
    return eager_decode_attn(QR, K_past.to(QR.dtype), V_past.to(QR.dtype))


def rope_tables(freqs: torch.Tensor, T: int, rope_start: int, device) -> Tuple[torch.Tensor, torch.Tensor]:
    """(cos, sin) of phase = ((rope_start + t) * freqs mod 1) * 2pi, fp32 (reference bdh.py:119-150)."""
    import math

    f = freqs.reshape(1, 1, 1, -1).to(device=device, dtype=torch.float32)
    pos = torch.arange(rope_start, rope_start + T, device=device, dtype=torch.float32).view(1, 1, -1, 1)
    ph = ((pos * f) % 1) * (2 * math.pi)
    return torch.cos(ph), torch.sin(ph)


def backend_info() -> dict:
    """Diagnostics for benchmarks / logs."""
    from .sm100_attn import ext_status, has_cuda_ext, has_cuda_kernel

    impl = resolve_attn_impl()
    return {
        "BDH_ATTN_IMPL": impl,
        "BDH_ATTN_AUTOGRAD": _env_autograd_enabled(),
        "BDH_ATTN_AUTO": attn_auto_enabled(),
        "BDH_ATTN_AUTO_THRESHOLD": attn_auto_threshold(),
        "BDH_ATTN_AUTO_COLD_THRESHOLD": attn_auto_cold_threshold(),
        "has_cuda_ext": has_cuda_ext(),
        "has_cuda_kernel": has_cuda_kernel(),
        "cuda": torch.cuda.is_available(),
        "effective": ("sm100_native" if impl == "cuda_sm100" else "eager"),
        "ext_status": ext_status(),
    }


__all__ = [
    "DEFAULT_ATTN_AUTO_THRESHOLD",
    "resolve_attn_impl",
    "resolve_decode_impl",
    "resolve_cold_impl",
    "attn_auto_enabled",
    "attn_auto_threshold",
    "attn_auto_cold_threshold",
    "bdh_attn",
    "bdh_attn_decode",
    "bdh_rope_attn",
    "bdh_rope_attn_decode",
    "rope_tables",
    "backend_info",
]
