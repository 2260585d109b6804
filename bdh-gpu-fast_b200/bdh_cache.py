"""Packed decode cache for BDH: rotated keys KR and values V per layer.

Same interface and layout as the reference ``bdh_cache.CacheManager`` (``bdh_cache.py:38-336``):

* ``_kr_buf`` ``(n_layer, B, n_head, capacity, N)`` and ``_v_buf`` ``(n_layer, B, 1, capacity, D)``
  in the storage dtype, layer-major, so a layer's past is a capacity-strided ``narrow`` view;
* ``reserve(level, T)`` returns writable slot views at ``[seq_len, seq_len+T)``;
  ``get_past(level)`` the committed prefix (cast to the compute dtype when storage differs);
  ``append`` / ``stage`` write a block; ``commit()`` advances ``seq_len`` once per step;
* optional paging (``page_size``) with geometric, page-aligned growth capped at ``max_seq``.

Addition for the B200 decode kernel: ``get_past_raw(level)`` returns the storage-dtype views
without any cast; the kernel reads bf16 or fp32 storage directly and widens in registers, so a
bf16 cache never costs a full-past conversion per step.

Opt-in fp8 key storage (``storage_dtype=torch.float8_e4m3fn``, no reference counterpart): each
cached key row is e4m3 with one fp32 scale (``_kr_scale (n_layer, B, n_head, capacity)``,
row ~= e4m3 * scale, scale = max|row| / 448), values stay bf16. ``get_past_scale`` /
``reserve_scale`` give the scale views beside ``get_past_raw`` / ``reserve``; ``get_past``
dequantizes. The decode stream is then ~1 byte per cached key element instead of 2 (bf16) or
4 (fp32); the format is lossy (3 mantissa bits).
"""

from __future__ import annotations

from typing import List, Optional, Tuple

import torch

FP8 = torch.float8_e4m3fn


def quantize_rows_fp8_torch(x: torch.Tensor):
    """Row-scaled e4m3 of the last axis with torch ops (CPU caches): the same arithmetic as the
    native bdh_quantize_rows_fp8 (inv = 448 / amax in fp32, products rounded to fp32, e4m3 round
    to nearest even). Returns (q float8_e4m3fn, scale fp32)."""
    x = x.float()
    amax = x.abs().amax(dim=-1)
    inv = torch.where(amax > 0, 448.0 / amax, torch.zeros_like(amax))
    q = (x * inv.unsqueeze(-1)).to(FP8)
    return q, amax / 448.0


def _quantize_into(x: torch.Tensor, out: torch.Tensor, scale: torch.Tensor) -> None:
    """Quantize rows of x (B,H,T,N) into the fp8 slot `out` and its `scale` (B,H,T): the native
    kernel for CUDA tensors (it raises if the library is missing), torch ops on the CPU."""
    if x.is_cuda:
        from kernels.sm100_attn import quantize_rows_fp8

        quantize_rows_fp8(x, out=out, scale=scale)
        return
    q, sc = quantize_rows_fp8_torch(x)
    out.copy_(q)
    scale.copy_(sc)


class CacheManager:
    """Per-layer packed KR/V in contiguous layer-major buffers (see module docstring)."""

    kind = "kv"

    def __init__(self, n_layer: int, max_seq: int, batch_size: int, n_head: int, n_latent: int,
                 n_embd: int, device, *, compute_dtype: torch.dtype = torch.float32,
                 storage_dtype: Optional[torch.dtype] = None, page_size: Optional[int] = None):
        if max_seq < 1:
            raise ValueError("max_seq must be >= 1")
        if page_size is not None and page_size < 1:
            raise ValueError("page_size must be >= 1 when set")
        self.n_layer = n_layer
        self.max_seq = max_seq
        self.batch_size = batch_size
        self.n_head = n_head
        self.n_latent = n_latent
        self.n_embd = n_embd
        self.device = torch.device(device)
        self.compute_dtype = compute_dtype
        self.storage_dtype = storage_dtype or compute_dtype
        self.kr_fp8 = self.storage_dtype == FP8
        # fp8 keys keep bf16 values (V is 1/32 of the key bytes per position at nh N = 32 D)
        self.v_dtype = torch.bfloat16 if self.kr_fp8 else self.storage_dtype
        self.storage_matches_compute = self.storage_dtype == self.compute_dtype
        self.page_size = page_size
        self.seq_len = 0
        self._pending_t: Optional[int] = None
        self.n_grows = 0
        self.bytes_copied_on_grow = 0
        self.capacity = max_seq if page_size is None else min(max_seq, page_size)
        self._kr_buf = torch.zeros(n_layer, batch_size, n_head, self.capacity, n_latent,
                                   dtype=self.storage_dtype, device=self.device)
        self._v_buf = torch.zeros(n_layer, batch_size, 1, self.capacity, n_embd,
                                  dtype=self.v_dtype, device=self.device)
        self._kr_scale = (torch.zeros(n_layer, batch_size, n_head, self.capacity,
                                      dtype=torch.float32, device=self.device)
                          if self.kr_fp8 else None)

    @property
    def _kr(self) -> List[torch.Tensor]:
        return [self._kr_buf[i] for i in range(self.n_layer)]

    @property
    def _v(self) -> List[torch.Tensor]:
        return [self._v_buf[i] for i in range(self.n_layer)]

    @classmethod
    def from_config(cls, config, batch_size: int, max_seq: int, device, *,
                    compute_dtype: torch.dtype = torch.float32,
                    storage_dtype: Optional[torch.dtype] = None,
                    page_size: Optional[int] = None, storage_kind: str = "kv"):
        """``storage_kind="state"`` returns the opt-in N x D recurrent-state cache
        (``StateCache``) instead of the key/value history."""
        nh = config.n_head
        D = config.n_embd
        N = config.mlp_internal_dim_multiplier * D // nh
        if storage_kind == "state":
            return StateCache(config.n_layer, batch_size, nh, N, D, device, max_seq=max_seq,
                              compute_dtype=compute_dtype)
        if storage_kind != "kv":
            raise ValueError(f"storage_kind must be 'kv' or 'state', got {storage_kind!r}")
        return cls(config.n_layer, max_seq, batch_size, nh, N, D, device,
                   compute_dtype=compute_dtype, storage_dtype=storage_dtype, page_size=page_size)

    # ------------------------------------------------------------------ capacity
    def ensure_capacity(self, need: int) -> None:
        self._ensure_capacity(need)

    def _next_capacity(self, need: int) -> int:
        ps = self.page_size
        assert ps is not None
        target = max(int(need), self.capacity * 2)
        target = ((target + ps - 1) // ps) * ps
        return min(self.max_seq, target)

    def _ensure_capacity(self, need: int) -> None:
        if need <= self.capacity:
            return
        if need > self.max_seq or self.page_size is None:
            raise RuntimeError(f"cache overflow: need {need} slots but max_seq={self.max_seq}")
        self._grow(self._next_capacity(need))

    def _grow(self, new_cap: int) -> None:
        if new_cap <= self.capacity:
            return
        kr = torch.empty(self.n_layer, self.batch_size, self.n_head, new_cap, self.n_latent,
                         dtype=self.storage_dtype, device=self.device)
        v = torch.empty(self.n_layer, self.batch_size, 1, new_cap, self.n_embd,
                        dtype=self.v_dtype, device=self.device)
        sc = (torch.empty(self.n_layer, self.batch_size, self.n_head, new_cap,
                          dtype=torch.float32, device=self.device) if self.kr_fp8 else None)
        used = self.seq_len + (self._pending_t or 0)
        if used > 0:
            kr[:, :, :, :used].copy_(self._kr_buf[:, :, :, :used])
            v[:, :, :, :used].copy_(self._v_buf[:, :, :, :used])
            if sc is not None:
                sc[:, :, :, :used].copy_(self._kr_scale[:, :, :, :used])
            self.bytes_copied_on_grow += used * self.n_layer * self.batch_size * (
                self.n_head * self.n_latent * self._kr_buf.element_size()
                + self.n_embd * self._v_buf.element_size())
        self._kr_buf, self._v_buf = kr, v
        self._kr_scale = sc
        self.capacity = new_cap
        self.n_grows += 1

    # --------------------------------------------------------------------- views
    def get_past_raw(self, level: int) -> Tuple[Optional[torch.Tensor], Optional[torch.Tensor]]:
        """Committed prefix of ``level`` as storage-dtype views (no cast, no copy)."""
        if self.seq_len == 0:
            return None, None
        return (self._kr_buf[level].narrow(2, 0, self.seq_len),
                self._v_buf[level].narrow(2, 0, self.seq_len))

    def get_past_scale(self, level: int) -> Optional[torch.Tensor]:
        """fp8 keys: the (B, n_head, seq_len) fp32 row scales of the committed prefix."""
        if not self.kr_fp8 or self.seq_len == 0:
            return None
        return self._kr_scale[level].narrow(2, 0, self.seq_len)

    def reserve_scale(self, level: int, T: int) -> torch.Tensor:
        """fp8 keys: the scale slots of the block ``reserve(level, T)`` returned."""
        if not self.kr_fp8:
            raise RuntimeError("reserve_scale needs fp8 key storage")
        return self._kr_scale[level].narrow(2, self.seq_len, T)

    def get_past(self, level: int) -> Tuple[Optional[torch.Tensor], Optional[torch.Tensor]]:
        """Committed prefix of ``level``, cast to ``compute_dtype`` when storage differs
        (fp8 keys: dequantized, row * scale)."""
        kr, v = self.get_past_raw(level)
        if kr is not None and self.kr_fp8:
            kr = (kr.float() * self.get_past_scale(level).unsqueeze(-1)).to(self.compute_dtype)
            v = v.to(self.compute_dtype)
        elif kr is not None and not self.storage_matches_compute:
            kr = kr.to(self.compute_dtype)
            v = v.to(self.compute_dtype)
        return kr, v

    def _track_pending(self, T: int) -> int:
        end = self.seq_len + T
        self._ensure_capacity(end)
        if self._pending_t is None:
            self._pending_t = T
        elif self._pending_t != T:
            raise RuntimeError(f"inconsistent append T: layer wrote {T}, pending={self._pending_t}")
        return end

    def reserve(self, level: int, T: int) -> Tuple[torch.Tensor, torch.Tensor]:
        """Writable views of the next block ``[seq_len, seq_len+T)`` of ``level`` (no copy).

        A paging grow may happen first, which invalidates previously returned views.
        """
        if T < 1:
            raise ValueError("reserve T must be >= 1")
        self._track_pending(T)
        return (self._kr_buf[level].narrow(2, self.seq_len, T),
                self._v_buf[level].narrow(2, self.seq_len, T))

    def _write_block(self, level: int, new_kr: torch.Tensor, new_v: torch.Tensor) -> int:
        T = new_kr.size(2)
        if T != new_v.size(2):
            raise ValueError(f"kr T={T} != v T={new_v.size(2)}")
        end = self._track_pending(T)
        if self.kr_fp8:
            _quantize_into(new_kr, self._kr_buf[level].narrow(2, self.seq_len, T),
                           self._kr_scale[level].narrow(2, self.seq_len, T))
        else:
            self._kr_buf[level].narrow(2, self.seq_len, T).copy_(new_kr)
        self._v_buf[level].narrow(2, self.seq_len, T).copy_(new_v)
        return end

    def append(self, level: int, new_kr: torch.Tensor, new_v: torch.Tensor) -> None:
        self._write_block(level, new_kr, new_v)

    def stage(self, level: int, new_kr: torch.Tensor, new_v: torch.Tensor):
        """Write the new block and return past+new views (cast when storage differs)."""
        end = self._write_block(level, new_kr, new_v)
        kr = self._kr_buf[level].narrow(2, 0, end)
        v = self._v_buf[level].narrow(2, 0, end)
        if self.kr_fp8:
            sc = self._kr_scale[level].narrow(2, 0, end).unsqueeze(-1)
            kr, v = (kr.float() * sc).to(self.compute_dtype), v.to(self.compute_dtype)
        elif not self.storage_matches_compute:
            kr, v = kr.to(self.compute_dtype), v.to(self.compute_dtype)
        return kr, v

    def commit(self) -> None:
        if self._pending_t is None:
            return
        self.seq_len += self._pending_t
        self._pending_t = None

    def reset(self) -> None:
        self.seq_len = 0
        self._pending_t = None
        self.n_grows = 0
        self.bytes_copied_on_grow = 0

    @property
    def bytes_allocated(self) -> int:
        n = (self._kr_buf.numel() * self._kr_buf.element_size()
             + self._v_buf.numel() * self._v_buf.element_size())
        if self._kr_scale is not None:
            n += self._kr_scale.numel() * self._kr_scale.element_size()
        return n


class StateCache:
    """Opt-in recurrent-state cache: per layer and (b, h) the N x D fp32 state
    S = sum over the cached positions of k_j v_j^T (k = the rotated latent, K is Q).

    The strictly causal linear attention of a new position t only needs q_t . S_t, so the
    cache stays (n_layer, B, nh, N, D) however long the sequence grows: a decode step reads and
    writes the state once (2 * nh * N * D * 4 bytes per batch row and layer) instead of reading
    the whole key/value history (nh * S * (N + D) * esz). It wins over the history once S
    exceeds about 2 N D / (N + D) * 4 / esz positions (~500 for fp32 histories at N = 8192,
    D = 256). It keeps the CacheManager bookkeeping (``seq_len``, pending block, ``commit``),
    but a past can no longer be read back as keys, so ``get_past`` does not exist here.
    """

    kind = "state"

    def __init__(self, n_layer: int, batch_size: int, n_head: int, n_latent: int, n_embd: int,
                 device, *, max_seq: Optional[int] = None,
                 compute_dtype: torch.dtype = torch.float32):
        self.n_layer = n_layer
        self.batch_size = batch_size
        self.n_head = n_head
        self.n_latent = n_latent
        self.n_embd = n_embd
        self.device = torch.device(device)
        self.compute_dtype = compute_dtype
        self.max_seq = max_seq
        self.seq_len = 0
        self._pending_t: Optional[int] = None
        self._state = torch.zeros(n_layer, batch_size, n_head, n_latent, n_embd,
                                  dtype=torch.float32, device=self.device)

    def state(self, level: int) -> torch.Tensor:
        """The (B, nh, N, D) fp32 state of ``level`` (updated in place by the step)."""
        return self._state[level]

    def advance(self, T: int) -> None:
        """Record that every layer of the current step folds a block of T positions in."""
        end = self.seq_len + T
        if self.max_seq is not None and end > self.max_seq:
            raise RuntimeError(f"cache overflow: need {end} positions but max_seq={self.max_seq}")
        if self._pending_t is None:
            self._pending_t = T
        elif self._pending_t != T:
            raise RuntimeError(f"inconsistent block T: layer folded {T}, pending={self._pending_t}")

    def commit(self) -> None:
        if self._pending_t is None:
            return
        self.seq_len += self._pending_t
        self._pending_t = None

    def reset(self) -> None:
        self.seq_len = 0
        self._pending_t = None
        self._state.zero_()

    @property
    def bytes_allocated(self) -> int:
        return self._state.numel() * self._state.element_size()
