"""BDH ("Dragon Hatchling") language model on the B200 attention path.

A compact restatement of the reference model (``bdh_baseline.py:32-139`` architecture,
``bdh.py:947-1072`` cached forward) that routes its attention through
``kernels.attention_dispatch``. Parameter names, shapes and initialisation match the
reference so ``state_dict``s load in either direction:

    embed (V, D) · encoder (nh, D, N) · encoder_v (nh, D, N) · decoder (nh*N, D) ·
    lm_head (D, V) · attn.freqs (1, 1, 1, N) buffer

Per layer (all LayerNorms affine-free)::

    x_sparse = relu(x @ encoder)                              (B, nh, T, N)
    yKV      = LN( tril(R(x_sparse) R(x_sparse)^T, -1) @ x )  (B, nh, T, D)
    y_sparse = relu(yKV @ encoder_v)
    x        = LN( x + LN( (x_sparse * y_sparse) @ decoder ) )

With ``BDH_ATTN_IMPL=cuda_sm100`` the RoPE is fused into the attention (in-register cos/sin,
no tables), the cached decode step rotates the new query and writes it into the cache slot
inside the decode kernel, and the cache is read in its storage dtype without copies. Prefill
layers in bf16 run on the library's fused latent kernels (``_layer_latent``: encoder GEMM +
ReLU + RoPE, the attention, the encoder_v GEMM + ReLU + product + decoder GEMM in one kernel,
the LayerNorms); the other paths (fp32, decode steps, training) use torch GEMMs for the
projections.
"""

from __future__ import annotations

import contextlib
import dataclasses
import math
import os
from typing import Optional

import torch
import torch.nn.functional as F
from torch import nn

from bdh_cache import CacheManager
from kernels.attention import eager_decode_attn
from kernels.attention_dispatch import (
    bdh_attn,
    bdh_rope_attn,
    bdh_rope_attn_decode,
    resolve_attn_impl,
    rope_tables,
)
from kernels.rope import eager_rope_rotate


@dataclasses.dataclass
class BDHConfig:
    n_layer: int = 6
    n_embd: int = 256
    dropout: float = 0.1
    n_head: int = 4
    mlp_internal_dim_multiplier: int = 128
    vocab_size: int = 256


def get_freqs(n: int, theta: float, dtype: torch.dtype) -> torch.Tensor:
    """freq[i] = theta^(-2*floor(i/2)/n) / (2*pi) (reference bdh.py:41-49)."""
    t = torch.arange(0, n, 1, dtype=dtype)
    q = (t / 2).floor() * 2
    return 1.0 / (theta ** (q / n)) / (2 * math.pi)


def _try_extend_seq(past: torch.Tensor, new: torch.Tensor) -> Optional[torch.Tensor]:
    """past||new as one view when ``new`` directly follows ``past`` in the same storage."""
    if past.untyped_storage().data_ptr() != new.untyped_storage().data_ptr():
        return None
    if past.stride() != new.stride() or past.shape[:-2] != new.shape[:-2]:
        return None
    if new.storage_offset() != past.storage_offset() + past.size(-2) * past.stride(-2):
        return None
    return past.as_strided((*past.shape[:-2], past.size(-2) + new.size(-2), past.size(-1)),
                           past.stride())


class Attention(nn.Module):
    """Strict-causal linear attention with BDH RoPE; K is Q (shared latent)."""

    def __init__(self, config: BDHConfig):
        super().__init__()
        nh, D = config.n_head, config.n_embd
        N = config.mlp_internal_dim_multiplier * D // nh
        self.freqs = nn.Buffer(get_freqs(N, theta=2 ** 16, dtype=torch.float32).view(1, 1, 1, N))
        self._attn_impl_override: Optional[str] = None
        self._rope_table = None       # (cos, sin) of positions [0, max_T), ensure_rope_table
        self._rope_table_key = None   # (max_T, device type, device index)

    @staticmethod
    def phases_cos_sin(phases: torch.Tensor):
        """(cos, sin) of phases given in turns: ((phases mod 1) * 2 pi) (bdh.py:119-122)."""
        phases = (phases % 1) * (2 * math.pi)
        return torch.cos(phases), torch.sin(phases)

    @staticmethod
    def rope(phases, v: torch.Tensor, out: Optional[torch.Tensor] = None, cos_sin=None):
        """Rotate the adjacent pairs of ``v`` by ``phases`` (or by precomputed ``cos_sin``) into
        ``out`` or a fresh tensor, through the ``BDH_ROPE_IMPL`` dispatch (bdh.py:124-140)."""
        from kernels.rope_dispatch import bdh_rope_rotate

        cos, sin = cos_sin if cos_sin is not None else Attention.phases_cos_sin(phases)
        return bdh_rope_rotate(v, cos, sin, out=out)

    def ensure_rope_table(self, max_T: int, device) -> None:
        """Precompute (cos, sin) for positions [0, max_T) once (bdh.py:157-191); rope_cos_sin
        and t1_cis_pairs then narrow into it instead of computing the phases again. Only the
        eager path reads tables: the native kernels compute the phases in registers."""
        if max_T < 1:
            raise ValueError("max_T must be >= 1")
        device = torch.device(device)
        key = (int(max_T), device.type, device.index)
        if self._rope_table is not None and self._rope_table_key == key:
            return
        cos, sin = rope_tables(self.freqs, int(max_T), 0, device)
        self._rope_table, self._rope_table_key = (cos, sin), key

    def _table_covers(self, rope_start: int, T: int, device) -> bool:
        if self._rope_table is None:
            return False
        max_T, dev_type, dev_index = self._rope_table_key
        device = torch.device(device)
        return (0 <= rope_start and rope_start + T <= max_T and device.type == dev_type
                and device.index == dev_index)

    def rope_cos_sin(self, T: int, rope_start: int, device):
        """(cos, sin) of positions [rope_start, rope_start + T), (1, 1, T, N) fp32: a narrow of
        the ensure_rope_table table when it covers them, else computed (bdh.py:193-262)."""
        if self._table_covers(rope_start, T, device):
            cos, sin = self._rope_table
            return cos.narrow(-2, rope_start, T), sin.narrow(-2, rope_start, T)
        return rope_tables(self.freqs, T, rope_start, device)

    def t1_cis_pairs(self, rope_start: int, device):
        """(cos, sin) of one position in the paired layout (1, 1, 1, N / 2, 2) from the
        ensure_rope_table table, or None without a covering table (bdh.py:301-347)."""
        if not self._table_covers(rope_start, 1, device):
            return None
        cos, sin = self._rope_table
        pair = lambda t: t.reshape(*t.shape[:-1], -1, 2).narrow(-3, rope_start, 1)
        return pair(cos), pair(sin)

    def forward(self, Q, K, V, rope_start: int = 0, past_kr=None, past_v=None, out_kr=None,
                past_is_raw: bool = False, relu_input: bool = False, past_kr_scale=None,
                out_kr_scale=None):
        """Returns ``(out, QR, V)``; QR/V are this block's keys/values for the cache.

        ``past_kr``/``past_v``: packed past (``past_is_raw``: in the cache storage dtype).
        ``out_kr``: optional cache slot receiving QR. ``relu_input``: Q is the encoder
        pre-activation; the latent is ``relu(Q)`` (folded into the RoPE read when possible).
        fp8 key cache: ``past_kr_scale`` / ``out_kr_scale`` are the row scales beside the raw
        fp8 past and the fp8 slot (QR is quantized into the slot).
        """
        assert K is Q
        impl = self._attn_impl_override or resolve_attn_impl()
        B, nh, T, _ = Q.shape
        fp8_slot = out_kr is not None and out_kr.dtype == torch.float8_e4m3fn
        if past_kr is None:
            out, QR = bdh_rope_attn(Q, V, self.freqs, rope_start, impl=impl,
                                    qr_out=None if fp8_slot else out_kr, relu_input=relu_input)
            if fp8_slot:
                from kernels.sm100_attn import quantize_rows_fp8

                quantize_rows_fp8(QR, out=out_kr, scale=out_kr_scale)
            return out, QR, V
        if relu_input:
            Q = F.relu(Q)
        S = past_kr.size(2)
        if past_kr.dtype == torch.float8_e4m3fn and impl == "cuda_sm100" and T == 1:
            from kernels.sm100_attn import rope_rotate, tril_decode_fp8

            out = tril_decode_fp8(Q, past_kr, past_kr_scale, past_v, freqs=self.freqs,
                                  pos=rope_start, kr_slot=out_kr, slot_scale=out_kr_scale)
            return out, out_kr, V
        if past_kr.dtype == torch.float8_e4m3fn:  # multi-token block: dequantized past
            past_kr = past_kr.float() * past_kr_scale.unsqueeze(-1)
            past_v = past_v.float()
            past_is_raw = True
        if impl == "cuda_sm100" and T == 1:
            if out_kr is not None:
                out = bdh_rope_attn_decode(Q, past_kr, past_v, self.freqs, rope_start, impl=impl,
                                           kr_slot=out_kr)
                return out, out_kr, V
            from kernels.sm100_attn import rope_rotate, tril_decode

            QR = rope_rotate(Q, self.freqs, rope_start)
            return tril_decode(QR, past_kr, past_v), QR, V
        # eager T=1 decode, or a multi-token block continuing a past
        qr_out = None if fp8_slot else out_kr
        QR = None
        if impl == "eager":
            QR = eager_rope_rotate(Q, *self.rope_cos_sin(T, rope_start, Q.device), out=qr_out)
        if QR is None:
            from kernels.sm100_attn import rope_rotate

            if qr_out is not None and qr_out.dtype != Q.dtype:
                # the block attends in the compute dtype (its own keys unrounded, as the
                # reference's past || block in compute dtype); the cache slot gets the rounded copy
                QR = rope_rotate(Q, self.freqs, rope_start)
                qr_out.copy_(QR)
            else:
                QR = rope_rotate(Q, self.freqs, rope_start, out=qr_out)
        if fp8_slot:
            from bdh_cache import _quantize_into

            _quantize_into(QR, out_kr, out_kr_scale)
        if impl == "cuda_sm100" and 1 < T <= 16:
            # a short block after a past (multi-token decode): the block's own strict past by the
            # tril pass plus the whole cached past by the decode kernel, which reads it in its
            # storage dtype; only the block's rows are computed (the reference recomputes
            # past || block with the cold path and keeps the last T rows, bdh.py:439-461)
            from kernels.sm100_attn import tril_decode, tril_score_v

            Vb = V.to(QR.dtype)
            return tril_score_v(QR, QR, Vb) + tril_decode(QR, past_kr, past_v), QR, V
        if past_is_raw and past_kr.dtype != QR.dtype:
            past_kr, past_v = past_kr.to(QR.dtype), past_v.to(QR.dtype)
        if T == 1:
            return eager_decode_attn(QR, past_kr, past_v.to(QR.dtype)), QR, V
        KR_all = _try_extend_seq(past_kr, QR)
        V_all = _try_extend_seq(past_v, V) if KR_all is not None else None
        if KR_all is None or V_all is None:
            KR_all = torch.cat([past_kr, QR.to(past_kr.dtype)], dim=2)
            V_all = torch.cat([past_v, V.to(past_v.dtype)], dim=2)
        Vq = V_all.to(QR.dtype) if impl == "cuda_sm100" else V_all
        out = bdh_attn(KR_all.to(QR.dtype), KR_all.to(QR.dtype), Vq, impl=impl)[:, :, S:, :]
        return out, QR, V


class BDH(nn.Module):
    def __init__(self, config: BDHConfig):
        super().__init__()
        self.config = config
        nh, D = config.n_head, config.n_embd
        N = config.mlp_internal_dim_multiplier * D // nh
        self.decoder = nn.Parameter(torch.zeros((nh * N, D)).normal_(std=0.02))
        self.encoder = nn.Parameter(torch.zeros((nh, D, N)).normal_(std=0.02))
        self.attn = Attention(config)
        self.ln = nn.LayerNorm(D, elementwise_affine=False, bias=False)
        self.embed = nn.Embedding(config.vocab_size, D)
        self.drop = nn.Dropout(config.dropout)
        self.encoder_v = nn.Parameter(torch.zeros((nh, D, N)).normal_(std=0.02))
        self.lm_head = nn.Parameter(torch.zeros((D, config.vocab_size)).normal_(std=0.02))
        nn.init.normal_(self.embed.weight, mean=0.0, std=0.02)

    def _ln(self, x: torch.Tensor) -> torch.Tensor:
        return F.layer_norm(x, (x.size(-1),), eps=self.ln.eps)

    def _bf16_param(self, name: str, k_major: bool = False) -> torch.Tensor:
        """bf16 copy of a parameter, refreshed when the parameter changes (the cast that
        autocast would make on every use). k_major: an (H, D, N) weight as a view of a
        contiguous (H, N, D) copy, the layout the latent kernels read fastest; a (K, D) matrix
        (the decoder) as a view of a contiguous (D, K) copy."""
        p = getattr(self, name)
        cache = self.__dict__.setdefault("_bf16_cache", {})
        key = (p.data_ptr(), p._version, p.device, k_major)
        hit = cache.get((name, k_major))
        if hit is None or hit[0] != key:
            w = p.detach().to(torch.bfloat16)
            if k_major:
                w = (w.t().contiguous().t() if w.dim() == 2
                     else w.transpose(1, 2).contiguous().transpose(1, 2))
            hit = (key, w)
            cache[(name, k_major)] = hit
        return hit[1]

    def _encoder_lin(self) -> torch.Tensor:
        """The encoder as the (nh * N, D) matrix F.linear reads (the reference's _encoder_relu
        layout, bdh.py:861-889): x_lat[b, t, h, n] = x[b, t] . encoder[h, :, n]. Kept between
        calls while no gradient is needed (an einsum over the (nh, D, N) parameter copies it
        into a GEMM layout on every call); built per call otherwise, so gradients reach the
        parameter."""
        p = self.encoder
        nh, D, N = p.shape
        if torch.is_grad_enabled() and p.requires_grad:
            return p.transpose(1, 2).reshape(nh * N, D)
        cache = self.__dict__.setdefault("_lin_cache", {})
        key = (p.data_ptr(), p._version, p.device, p.dtype)
        hit = cache.get("encoder")
        if hit is None or hit[0] != key:
            hit = (key, p.detach().transpose(1, 2).reshape(nh * N, D).contiguous())
            cache["encoder"] = hit
        return hit[1]

    def _attn_state(self, Q: torch.Tensor, V: torch.Tensor, level: int, rope_start: int, cache,
                    impl: str, relu_input: bool) -> torch.Tensor:
        """Attention of a block against a StateCache, folding the block into the state.

        T = 1 on the sm100 path: one fused step (``state_decode``). Otherwise: RoPE, the strictly
        causal attention inside the block, plus the past as QR . S, then S += QR^T V (fp32)."""
        S = cache.state(level)
        B, nh, T, N = Q.shape
        if impl == "cuda_sm100" and T == 1 and Q.is_cuda:
            from kernels.sm100_attn import state_decode

            out = state_decode(Q, S, V, self.attn.freqs, rope_start, relu_input=relu_input)
            cache.advance(1)
            return out
        if relu_input:
            Q = F.relu(Q)
        if impl == "cuda_sm100":
            from kernels.sm100_attn import rope_rotate

            QR = rope_rotate(Q, self.attn.freqs, rope_start)
        else:
            QR = eager_rope_rotate(Q, *self.attn.rope_cos_sin(T, rope_start, Q.device))
        Vq = V.to(QR.dtype)
        out = bdh_attn(QR, QR, Vq, impl=impl)
        chunk = max(1, (1 << 28) // max(1, nh * T * N))  # bound the fp32 copies of QR
        for b0 in range(0, B, chunk):
            qf = QR[b0:b0 + chunk].float()
            if cache.seq_len > 0:
                out[b0:b0 + chunk] += (qf @ S[b0:b0 + chunk]).to(out.dtype)
            S[b0:b0 + chunk].add_(qf.transpose(-1, -2) @ V[b0:b0 + chunk].float())
        cache.advance(T)
        return out

    def _latent_fusable(self, impl: str, T: int, cache, device) -> bool:
        """The fused encode / gate kernels serve bf16 prefill blocks without a past."""
        if impl != "cuda_sm100" or T < 64 or device.type != "cuda":
            return False
        if torch.is_grad_enabled() or (self.training and self.drop.p != 0.0):
            return False
        if cache is not None and (cache.seq_len != 0 or getattr(cache, "kind", "kv") != "kv"):
            return False
        bf16 = (torch.is_autocast_enabled("cuda") and torch.get_autocast_dtype("cuda") == torch.bfloat16) \
            or self.encoder.dtype == torch.bfloat16
        return bf16 and os.environ.get("BDH_SM100_LATENT", "1") != "0"

    def _decoder_product(self, xy: torch.Tensor, B: int, T: int, impl: str,
                         grad: bool) -> torch.Tensor:
        """y_mlp = xy @ decoder (bdh.py:1050) for xy (B, T, nh, N). An fp32 decode step (at most
        256 rows B*T, no autocast, no autograd) on the native path runs bdh_decoder_f32, which
        splits K = nh*N across the GPU (a library GEMM launches a few CTAs for this shape);
        BDH_SM100_DEC_F32=0 keeps torch's linear for every shape."""
        x2 = xy.reshape(B * T, xy.size(-2) * xy.size(-1))
        if (impl == "cuda_sm100" and not grad and x2.is_cuda and B * T <= 256
                and x2.dtype == torch.float32 and self.decoder.dtype == torch.float32
                and not torch.is_autocast_enabled()
                and os.environ.get("BDH_SM100_DEC_F32", "1") != "0"):
            from kernels.sm100_attn import decoder_f32

            return decoder_f32(x2, self.decoder).view(B, T, -1)
        return F.linear(x2.view(B, T, -1), self.decoder.t())

    def _layer_latent(self, x: torch.Tensor, xb: Optional[torch.Tensor], level: int,
                      rope_start: int, cache):
        """One layer on the fused kernels: encode (+ReLU +RoPE) -> tril attention with its LN in
        the value pass's epilogue -> encoder_v gate (xs * relu(.)) -> decoder -> residual double
        LN. Same arithmetic as the
        bf16-autocast layer of bdh.py:991-1052. With D = 256 and N a multiple of 128 the gate and
        the decoder product run as one kernel (``latent_gate_dec``, ``BDH_SM100_GATE_DEC=0``
        keeps the gate + cuBLAS decoder), so the (B, T, nh, N) xy latent is never stored. ``xb`` is the bf16 copy of ``x`` (made
        here when None); returns the new ``(x, xb)``.

        ``BDH_SM100_GATE_X=1`` (D <= 256): the encode writes only the rotated latent and the
        gate recomputes xs = relu(x @ enc) next to y @ encv (``latent_gate_x``, bit-identical
        xs), so the (B, T, nh, N) xs latent is never stored. It trades 12.9 GB of HBM traffic
        per config-2 step for a second K = 256 GEMM in the gate and measures slower on one
        B200 (1.68M vs 1.74M tokens/s: the gate becomes tensor-bound under the power cap), so
        the default stores xs."""
        from kernels.sm100_attn import latent_gate, latent_gate_x
        from kernels.sm100_ext import model_ops

        ops = model_ops()  # the torch extension when built, else the ctypes binding
        latent_encode, latent_gate_dec = ops.latent_encode, ops.latent_gate_dec
        residual_layer_norm, tril_score_v = ops.residual_layer_norm, ops.tril_score_v

        B, T, _ = x.shape
        nh = self.config.n_head
        eps = self.ln.eps
        if xb is None:
            xb = x.to(torch.bfloat16)
        v_tok = x.unsqueeze(1)
        qr_slot = None
        dst_kr = None
        if cache is not None:
            dst_kr, dst_v = cache.reserve(level, T)
            dst_v.copy_(v_tok)
            if dst_kr.dtype == torch.bfloat16:
                qr_slot = dst_kr
        kmaj = os.environ.get("BDH_SM100_WEIGHT_KMAJOR", "1") != "0"
        gate_x = x.size(-1) <= 256 and os.environ.get("BDH_SM100_GATE_X", "0") == "1"
        enc = self._bf16_param("encoder", kmaj)
        xs, qr = latent_encode(xb, enc, self.attn.freqs, rope_start, qr_out=qr_slot,
                               want_xs=not gate_x)
        if dst_kr is not None and qr_slot is None:
            if dst_kr.dtype == torch.float8_e4m3fn:
                from kernels.sm100_attn import quantize_rows_fp8

                quantize_rows_fp8(qr, out=dst_kr, scale=cache.reserve_scale(level, T))
            else:
                dst_kr.copy_(qr)
        # the attention output's LayerNorm runs in the value pass's epilogue
        yn = tril_score_v(qr, qr, xb.unsqueeze(1), ln_eps=eps)
        encv = self._bf16_param("encoder_v", kmaj)
        N = enc.size(-1)
        gate_dec = (not gate_x and kmaj and x.size(-1) == 256 and N % 128 == 0
                    and os.environ.get("BDH_SM100_GATE_DEC", "1") != "0")
        if gate_dec:  # gate and decoder in one kernel, xy never stored
            y_mlp = latent_gate_dec(yn, encv, xs, self._bf16_param("decoder", True))
        else:
            xy = latent_gate_x(yn, encv, xb, enc) if gate_x else latent_gate(yn, encv, xs)
            y_mlp = F.linear(xy.view(B, T, nh * xy.size(-1)), self._bf16_param("decoder").t())
        if x.dtype == torch.float32:
            return residual_layer_norm(x, y_mlp, eps, want_bf16=True)
        x = self._ln(x + self._ln(y_mlp))
        return x, x.to(torch.bfloat16)

    def forward(self, idx: torch.Tensor, targets: Optional[torch.Tensor] = None,
                cache: Optional[CacheManager] = None, *, logits_out: Optional[torch.Tensor] = None):
        """Logits ``(B, T, V)`` (and the CE loss with ``targets``).

        ``cache``: a ``CacheManager``; ``idx`` is then the next block and RoPE continues at
        ``cache.seq_len``. ``logits_out``: (B, V) fp32 buffer for the last-token logits (T == 1).
        """
        C = self.config
        B, T = idx.shape
        nh, D = C.n_head, C.n_embd
        N = D * C.mlp_internal_dim_multiplier // nh
        x = self._ln(self.embed(idx))  # (B, T, D)
        rope_start = cache.seq_len if cache is not None else 0
        impl = self.attn._attn_impl_override or resolve_attn_impl()
        grad = torch.is_grad_enabled()
        # Inference on B200: both ReLUs are folded into native kernels (the RoPE read and the
        # gated product), so the latents are never rewritten just to clamp them.
        fused = impl == "cuda_sm100" and not grad and (not self.training or self.drop.p == 0.0)
        latent = self._latent_fusable(impl, T, cache, x.device)
        with self._score_rounding(impl):
            x = self._layers(x, impl, grad, fused, latent, rope_start, cache, B, T, N)
        if cache is not None:
            cache.commit()
        if logits_out is not None:
            if T != 1:
                raise ValueError("logits_out requires T==1 decode")
            torch.mm(x[:, -1, :].to(logits_out.dtype), self.lm_head.to(logits_out.dtype), out=logits_out)
            return logits_out, None
        logits = F.linear(x, self.lm_head.t())
        loss = None
        if targets is not None:
            loss = F.cross_entropy(logits.reshape(-1, logits.size(-1)), targets.reshape(-1))
        return logits, loss

    @staticmethod
    def _score_rounding(impl: str):
        """bf16 attention scores on the native path are rounded once to bf16 before their
        product with V, as the reference model's default (eager) attention does under autocast
        (``(QR @ QR.mT).tril_(-1) @ V`` returns bf16 scores, kernels/attention.py:27-40), so the
        model's logits follow the reference's bf16 chain. An explicit process setting
        (``BDH_SM100_SPLIT_SCORES``) wins."""
        if impl != "cuda_sm100" or os.environ.get("BDH_SM100_SPLIT_SCORES"):
            return contextlib.nullcontext()
        from kernels.sm100_attn import score_terms_scope

        return score_terms_scope("bf16")

    def _layers(self, x, impl, grad, fused, latent, rope_start, cache, B, T, N):
        """The layer loop of ``forward`` (bdh.py:992-1052); returns the final residual x."""
        C = self.config
        xb = None
        for level in range(C.n_layer):
            if latent:
                x, xb = self._layer_latent(x, xb, level, rope_start, cache)
                continue
            x_lat = F.linear(x, self._encoder_lin()).view(B, T, C.n_head, N)  # (B, T, nh, N)
            x_bthn = x_lat if fused else F.relu(x_lat)
            x_sparse = x_bthn.permute(0, 2, 1, 3)  # (B, nh, T, N) view
            v_tok = x.unsqueeze(1)
            if cache is not None and getattr(cache, "kind", "kv") == "state":
                y_kv = self._attn_state(x_sparse, v_tok, level, rope_start, cache, impl, fused)
                y_kv = self._ln(y_kv)
                y_lat = torch.einsum("bhtd,hdn->bthn", y_kv, self.encoder_v)
                if fused:
                    from kernels.sm100_attn import relu_mul

                    xy = relu_mul(x_lat, y_lat)
                else:
                    xy = self.drop(x_bthn * F.relu(y_lat))
                y_mlp = self._decoder_product(xy, B, T, impl, grad)
                x = self._ln(x + self._ln(y_mlp))
                continue
            past_kr = past_v = out_kr = past_scale = out_scale = None
            raw = False
            if cache is not None:
                # the native decode reads fp32, bf16 and fp8 caches in place; another storage
                # dtype (fp16) is upcast per step by get_past, as the reference's cache does
                # (bdh_cache.py:240-243), and the native kernels run on the fp32 copy
                native = (impl == "cuda_sm100" and not grad
                          and cache.storage_dtype in (torch.float32, torch.bfloat16,
                                                      torch.float8_e4m3fn))
                eager_inplace = (not grad and cache.storage_matches_compute
                                 and v_tok.dtype == cache.storage_dtype)
                if native or eager_inplace:
                    dst_kr, dst_v = cache.reserve(level, T)
                    if native:
                        past_kr, past_v = cache.get_past_raw(level)
                        raw = True
                        if getattr(cache, "kr_fp8", False):
                            past_scale = cache.get_past_scale(level)
                            out_scale = cache.reserve_scale(level, T)
                    else:
                        past_kr, past_v = cache.get_past(level)
                    dst_v.copy_(v_tok)
                    out_kr = dst_kr
                    if dst_v.dtype == v_tok.dtype:  # the slot view (past || block without a copy)
                        v_tok = dst_v
                else:
                    past_kr, past_v = cache.get_past(level)
            y_kv, new_kr, new_v = self.attn(x_sparse, x_sparse, v_tok, rope_start=rope_start,
                                            past_kr=past_kr, past_v=past_v, out_kr=out_kr,
                                            past_is_raw=raw, relu_input=fused,
                                            past_kr_scale=past_scale, out_kr_scale=out_scale)
            if cache is not None and out_kr is None:
                cache.append(level, new_kr, new_v)
            y_kv = self._ln(y_kv)
            y_lat = torch.einsum("bhtd,hdn->bthn", y_kv, self.encoder_v)
            if fused:
                from kernels.sm100_attn import relu_mul

                xy = relu_mul(x_lat, y_lat)
            else:
                xy = self.drop(x_bthn * F.relu(y_lat))
            y_mlp = self._decoder_product(xy, B, T, impl, grad)
            x = self._ln(x + self._ln(y_mlp))
        return x

    def graphed_forward(self, batch: int, seq_len: int,
                        amp_dtype: Optional[torch.dtype] = torch.bfloat16) -> "GraphedForward":
        """This model's no-grad prefill for one (batch, seq_len) captured as a CUDA graph (see
        ``GraphedForward``)."""
        return GraphedForward(self, batch, seq_len, amp_dtype)

    @staticmethod
    def _sample(logits: torch.Tensor, temperature: float, top_k: Optional[int]) -> torch.Tensor:
        """One token per row of fp32 (B, V) logits, drawing from the RNG exactly as the
        reference's sampler does (bdh.py:680-728), so a seed gives the same tokens: temperature
        as a multiplication by its reciprocal; with top_k < V a softmax over the k largest
        logits, one multinomial draw among them and a gather of its index; with top_k >= V the
        logits below the k-th largest masked to -inf; then a softmax over the vocabulary and
        one multinomial draw."""
        if float(temperature) != 1.0:
            logits = logits * (1.0 / float(temperature))
        if top_k is not None:
            V = logits.size(-1)
            k = min(int(top_k), V)
            values, indices = torch.topk(logits, k, dim=-1)
            if k < V:
                return indices.gather(1, torch.multinomial(F.softmax(values, dim=-1), 1))
            logits = logits.masked_fill(logits < values[:, -1:], float("-inf"))
        return torch.multinomial(torch.softmax(logits, dim=-1), 1)

    def generate(self, idx: torch.Tensor, max_new_tokens: int, temperature: float = 1.0,
                 top_k: Optional[int] = None, *, cache_dtype: Optional[torch.dtype] = None,
                 amp_dtype: Optional[torch.dtype] = None, cache_page_size: Optional[int] = None,
                 cache_kind: str = "kv") -> torch.Tensor:
        """Autoregressive sampling with the packed cache (prefill, then T = 1 steps), the
        reference's ``BDH.generate`` (bdh.py:1076-1190): the same keywords (``cache_dtype`` the
        cache storage dtype, ``cache_page_size`` its paging, ``amp_dtype`` autocast over the
        forward) and the same tokens for a seed. ``cache_kind="state"`` keeps the N x D
        recurrent state instead of the history."""
        was_training = self.training
        self.eval()
        B, T0 = idx.shape
        cache = CacheManager.from_config(self.config, B, T0 + max_new_tokens, idx.device,
                                         storage_dtype=cache_dtype, page_size=cache_page_size,
                                         storage_kind=cache_kind)
        if (self.attn._attn_impl_override or resolve_attn_impl()) == "eager":
            self.attn.ensure_rope_table(T0 + max_new_tokens, idx.device)  # the span's phases once
        out = torch.empty(B, T0 + max_new_tokens, dtype=idx.dtype, device=idx.device)
        out[:, :T0] = idx
        ctx = (torch.autocast(idx.device.type, dtype=amp_dtype) if amp_dtype is not None
               else torch.autocast(idx.device.type, enabled=False))
        try:
            with torch.inference_mode(), ctx:
                logits, _ = self(idx, cache=cache)
                for t in range(max_new_tokens):
                    nxt = self._sample(logits[:, -1, :].float(), temperature, top_k)
                    out[:, T0 + t] = nxt[:, 0]
                    if t + 1 < max_new_tokens:
                        logits, _ = self(nxt, cache=cache)
        finally:
            if was_training:
                self.train()
        return out


class GraphedForward:
    """A model's no-grad forward (no cache) for one input shape, captured once as a CUDA graph
    and replayed per call: the ~36 native launches of a 6-layer step and the host work around
    them (argument checks, tensor maps, workspace sizing) are paid once, at capture, instead of
    every step, which matters when a step's kernels are short (small batches).

    Every library entry point on this path is stream-ordered with no host synchronisation, so
    the capture holds the same kernels with the same arguments an eager call issues (the same
    bits). Two warm-up calls before the capture build the library's per-device tables and the
    model's bf16 weight copies; capture after the weights are final (the graph keeps reading the
    copies it saw). ``__call__(idx)`` copies ``idx`` into the graph's input buffer and returns
    the graph's logits buffer, which the next call overwrites.
    """

    def __init__(self, model: BDH, batch: int, seq_len: int,
                 amp_dtype: Optional[torch.dtype] = torch.bfloat16):
        dev = model.embed.weight.device
        if dev.type != "cuda":
            raise ValueError("graphed_forward needs the model on a CUDA device")
        self.model = model
        self.idx = torch.zeros(batch, seq_len, dtype=torch.long, device=dev)
        self._amp = amp_dtype

        def ctx():
            return (torch.autocast("cuda", dtype=amp_dtype) if amp_dtype is not None
                    else contextlib.nullcontext())

        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side), torch.inference_mode(), ctx():
            for _ in range(2):
                model(self.idx)
        torch.cuda.current_stream(dev).wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.inference_mode(), ctx(), torch.cuda.graph(self.graph):
            self.logits = model(self.idx)[0]

    def __call__(self, idx: torch.Tensor) -> torch.Tensor:
        if tuple(idx.shape) != tuple(self.idx.shape):
            raise ValueError(f"graphed forward was captured for {tuple(self.idx.shape)}, "
                             f"got {tuple(idx.shape)}")
        self.idx.copy_(idx, non_blocking=True)
        self.graph.replay()
        return self.logits
