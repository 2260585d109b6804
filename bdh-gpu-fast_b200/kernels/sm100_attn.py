"""ctypes binding of libbdh_sm100.so — the sm_100a tril attention behind ``BDH_ATTN_IMPL=cuda_sm100``.

Mirrors the reference's native wrapper ``kernels/cuda_attn.py`` (``tril_score_v`` :391-414,
``tril_decode`` :490-502, shape checks :103-131, ``has_cuda_ext`` / ``ext_status`` :81-100,
:505-513) with two deliberate differences:

* no silent fallback: a missing library, a CPU tensor or a failing launch raises
  (the reference returned its pure-PyTorch result on any exception, ``cuda_attn.py:401-409``);
* no ``.contiguous()`` of inputs: strided views (permuted Q, capacity-strided cache views) are
  passed to the kernels as they are (the reference copied them, ``csrc/tril_attn_cuda.cu:264-266,
  563-565``).

Semantics (identical to the reference)::

    tril_score_v(q, k, v)        = (q @ k.mT).tril(-1) @ v      # v heads 1 or H (broadcast)
    tril_decode(q, k_past, v_past) = (q @ k_past.mT) @ v_past    # S == 0 -> zeros

Tensors: q, k ``(B, H, T, N)``; v ``(B, Hv, T, D)``; fp32 or bf16 (fp32 accumulation always);
the output is a fresh ``(B, H, T, D)`` tensor in q's dtype. Device memory (outputs and the
library's scratch workspace) comes from the PyTorch caching allocator on the current stream.
"""

from __future__ import annotations

import contextlib
import ctypes
import os
from pathlib import Path
from typing import Optional

import torch

_PKG = Path(__file__).resolve().parent.parent
_LIB_PATH = Path(os.environ.get("BDH_SM100_LIB", str(_PKG / "libbdh_sm100.so")))

_lib: Optional[ctypes.CDLL] = None
_lib_error: Optional[BaseException] = None

_F32 = 0
_BF16 = 1

_c_i64_4 = ctypes.c_int64 * 4
ABI_VERSION = 9  # BDH_ABI_VERSION of include/bdh_sm100.h
FP8 = torch.float8_e4m3fn  # the opt-in fp8 key-cache storage dtype
_vp = ctypes.c_void_p
_i64 = ctypes.c_int64


def _declare(lib: ctypes.CDLL) -> None:
    P = ctypes.POINTER(ctypes.c_int64)
    lib.bdh_abi_version.restype = ctypes.c_int
    lib.bdh_last_error.restype = ctypes.c_char_p
    lib.bdh_device_error.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_int), ctypes.c_int]
    lib.bdh_rope_rotate.argtypes = [_vp, ctypes.c_int, P, _vp, ctypes.c_int, P, _vp, _vp,
                                    _i64, _i64, _i64, _i64, _i64, ctypes.c_int, _vp]
    lib.bdh_relu_mul.argtypes = [_vp, P, _vp, P, _vp, P, ctypes.c_int, _i64, _i64, _i64, _i64, _vp]
    lib.bdh_decoder_f32_slices.argtypes = [_i64]
    lib.bdh_decoder_f32_slices.restype = _i64
    lib.bdh_decoder_f32.argtypes = [_vp, _i64, _vp, _i64, _vp, _i64, _vp, _i64, _i64, _i64, _vp]
    lib.bdh_set_forward_algo.argtypes = [ctypes.c_int]
    lib.bdh_set_forward_algo.restype = ctypes.c_int
    lib.bdh_set_score_terms.argtypes = [ctypes.c_int]
    lib.bdh_set_score_terms.restype = ctypes.c_int
    lib.bdh_tril_score_v_workspace_size.restype = ctypes.c_size_t
    lib.bdh_tril_score_v_workspace_size.argtypes = [ctypes.c_int, _i64, _i64, _i64, _i64, _i64,
                                                    _i64, ctypes.c_int]
    lib.bdh_tril_score_v.argtypes = [_vp, P, _vp, P, _vp, P, ctypes.c_int, _vp, P, ctypes.c_int,
                                     _i64, _i64, _i64, _i64, _i64, _i64, _vp, ctypes.c_size_t, _vp]
    lib.bdh_tril_score_v_layernorm.argtypes = [_vp, P, _vp, P, _vp, P, ctypes.c_int, _vp, P,
                                               ctypes.c_int, _i64, _i64, _i64, _i64, _i64, _i64,
                                               ctypes.c_float, _vp, ctypes.c_size_t, _vp]
    lib.bdh_tril_decode_workspace_size.restype = ctypes.c_size_t
    lib.bdh_tril_decode_workspace_size.argtypes = [_i64, _i64, _i64, _i64, _i64, _i64]
    lib.bdh_tril_decode.argtypes = [_vp, P, ctypes.c_int, _vp, P, _vp, P, ctypes.c_int, _vp, P,
                                    _i64, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _i64, _vp, P,
                                    _vp, ctypes.c_size_t, _vp]
    lib.bdh_tril_score_v_bwd_workspace_size.restype = ctypes.c_size_t
    lib.bdh_tril_score_v_bwd_workspace_size.argtypes = [ctypes.c_int, _i64, _i64, _i64, _i64,
                                                        _i64, _i64, ctypes.c_int]
    lib.bdh_tril_score_v_bwd.argtypes = [_vp, P, _vp, P, _vp, P, _vp, P, ctypes.c_int, _vp, P,
                                         _vp, P, _vp, P, _i64, _i64, _i64, _i64, _i64, _i64, _vp,
                                         _i64, _vp, ctypes.c_size_t, _vp]
    _c_i64_3p = ctypes.POINTER(ctypes.c_int64)
    lib.bdh_latent_encode.argtypes = [_vp, _c_i64_3p, _vp, _c_i64_3p, _vp, P, _vp, P, _vp,
                                      _i64, _i64, _i64, _i64, _i64, _i64, _vp]
    lib.bdh_latent_gate.argtypes = [_vp, P, _vp, _c_i64_3p, _vp, P, _vp, P,
                                    _i64, _i64, _i64, _i64, _i64, _vp]
    lib.bdh_latent_gate_x.argtypes = [_vp, P, _vp, _c_i64_3p, _vp, _c_i64_3p, _vp, _c_i64_3p,
                                      _vp, P, _i64, _i64, _i64, _i64, _i64, _vp]
    _c_i64_2p = ctypes.POINTER(ctypes.c_int64)
    lib.bdh_latent_gate_dec.argtypes = [_vp, P, _vp, _c_i64_3p, _vp, P, _vp, _c_i64_2p, _vp,
                                        _c_i64_3p, _i64, _i64, _i64, _i64, _i64, _vp]
    lib.bdh_latent_gate_dec_ws.argtypes = [_vp, P, _vp, _c_i64_3p, _vp, P, _vp, _c_i64_2p, _vp,
                                           _c_i64_3p, _i64, _i64, _i64, _i64, _i64, _vp,
                                           ctypes.c_size_t, _vp]
    lib.bdh_latent_gate_dec_workspace_size.restype = ctypes.c_size_t
    lib.bdh_latent_gate_dec_workspace_size.argtypes = [_i64, _i64, _i64, _i64, _i64]
    lib.bdh_quantize_rows_fp8.argtypes = [_vp, P, ctypes.c_int, _i64, _i64, _i64, _i64, _vp, P,
                                          _vp, P, _vp]
    lib.bdh_tril_decode_fp8.argtypes = [_vp, P, ctypes.c_int, _vp, P, _vp, P, _vp, P, ctypes.c_int,
                                        _vp, P, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _vp,
                                        _i64, _vp, P, _vp, P, _vp, ctypes.c_size_t, _vp]
    lib.bdh_layernorm.argtypes = [_vp, ctypes.c_int, _i64, _vp, ctypes.c_int, _i64, _i64, _i64,
                                  ctypes.c_float, _vp]
    lib.bdh_residual_layernorm.argtypes = [_vp, _i64, _vp, ctypes.c_int, _i64, _vp, _i64, _vp,
                                           _i64, _i64, _i64, ctypes.c_float, _vp]
    lib.bdh_state_decode_workspace_size.restype = ctypes.c_size_t
    lib.bdh_state_decode_workspace_size.argtypes = [_i64, _i64, _i64, _i64]
    lib.bdh_state_decode.argtypes = [_vp, P, ctypes.c_int, _vp, P, _vp, P, ctypes.c_int, _vp, P,
                                     _i64, _i64, _i64, _i64, _i64, _vp, _i64, ctypes.c_int, _vp,
                                     ctypes.c_size_t, _vp]
    for name in ("bdh_rope_rotate", "bdh_tril_score_v", "bdh_tril_score_v_layernorm",
                 "bdh_tril_decode", "bdh_tril_score_v_bwd",
                 "bdh_relu_mul", "bdh_latent_encode", "bdh_latent_gate", "bdh_latent_gate_x",
                 "bdh_latent_gate_dec", "bdh_latent_gate_dec_ws",
                 "bdh_layernorm", "bdh_quantize_rows_fp8", "bdh_tril_decode_fp8",
                 "bdh_residual_layernorm", "bdh_state_decode"):
        getattr(lib, name).restype = ctypes.c_int


def load_library(path: Optional[os.PathLike] = None) -> ctypes.CDLL:
    """Load (once) and return the C-ABI library; raises if it cannot be loaded."""
    global _lib, _lib_error
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path is not None else _LIB_PATH
    try:
        lib = ctypes.CDLL(str(p))
        _declare(lib)
        ver = lib.bdh_abi_version()
        if ver != ABI_VERSION:
            raise RuntimeError(f"{p}: unexpected ABI version {ver}")
    except BaseException as exc:  # noqa: BLE001 - remembered for ext_status()
        _lib_error = exc
        raise
    if path is None:
        _lib = lib
    return lib


def _try_load() -> Optional[ctypes.CDLL]:
    try:
        return load_library()
    except BaseException:  # noqa: BLE001
        return None


def has_cuda_ext() -> bool:
    """True if libbdh_sm100.so loads (it always carries the sm_100a kernels)."""
    return _try_load() is not None


def has_cuda_kernel() -> bool:
    """True if the library loads and a CUDA device is present to run it."""
    return has_cuda_ext() and torch.cuda.is_available()


def ext_status() -> str:
    """Human-readable status (same role as the reference's ``cuda_attn.ext_status``)."""
    if _try_load() is None:
        err = _lib_error
        detail = f"{type(err).__name__}: {err}" if err is not None else "not attempted"
        return f"native=unavailable ({detail})"
    cuda = "yes" if torch.cuda.is_available() else "no"
    return f"native=loaded lib={_LIB_PATH.name} has_cuda_kernel={cuda} has_decode=yes has_bwd=yes"


def _require_lib() -> ctypes.CDLL:
    lib = _try_load()
    if lib is None:
        raise RuntimeError(
            f"cuda_sm100: {_LIB_PATH} is not loadable ({_lib_error!r}); build it with "
            "`python bdh-gpu-fast_b200/build_lib.py`"
        )
    return lib


def _check(rc: int, what: str) -> None:
    if rc != 0:
        msg = _require_lib().bdh_last_error().decode(errors="replace")
        raise RuntimeError(f"cuda_sm100 {what} failed (code {rc}): {msg}")


def device_error(device: Optional[torch.device] = None, reset: bool = True) -> int:
    """Synchronise and return the device error word (0 = no kernel reported a failure)."""
    lib = _require_lib()
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    code = ctypes.c_int(0)
    _check(lib.bdh_device_error(dev.index or 0, ctypes.byref(code), 1 if reset else 0), "device_error")
    return int(code.value)


# --------------------------------------------------------------------------- checks
def _check_cold_shapes(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> None:
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        raise ValueError("q, k, v must be 4D (B, H, T, D)")
    if q.shape != k.shape:
        raise ValueError(f"q and k shapes must match, got {tuple(q.shape)} vs {tuple(k.shape)}")
    if v.size(0) != q.size(0) or v.size(2) != q.size(2):
        raise ValueError("v batch/seq must match q")
    if v.size(1) not in (1, q.size(1)):
        raise ValueError("v heads must equal q heads or 1")


def _check_decode_shapes(q: torch.Tensor, k_past: torch.Tensor, v_past: torch.Tensor):
    if q.dim() != 4 or k_past.dim() != 4 or v_past.dim() != 4:
        raise ValueError("q, k_past, v_past must be 4D")
    B, H, Tq, Dk = q.shape
    S = k_past.size(2)
    if k_past.shape[:2] != (B, H) or k_past.size(-1) != Dk:
        raise ValueError(f"k_past shape {tuple(k_past.shape)} incompatible with q {tuple(q.shape)}")
    if v_past.size(0) != B or v_past.size(2) != S:
        raise ValueError(f"v_past shape {tuple(v_past.shape)} incompatible with k_past S={S}")
    if v_past.size(1) not in (1, H):
        raise ValueError("v_past heads must equal q heads or 1")
    return B, H, Tq, S, v_past.size(-1)


def _code(dtype: torch.dtype) -> int:
    if dtype == torch.float32:
        return _F32
    if dtype == torch.bfloat16:
        return _BF16
    raise TypeError(f"cuda_sm100 supports float32 and bfloat16 tensors, got {dtype}")


def _require_cuda(*ts: torch.Tensor) -> torch.device:
    dev = ts[0].device
    for t in ts:
        if not t.is_cuda:
            raise RuntimeError("cuda_sm100 requires CUDA tensors (no CPU fallback)")
        if t.device != dev:
            raise RuntimeError("cuda_sm100: all tensors must be on the same device")
    return dev


def _strides(t: torch.Tensor):
    return _c_i64_4(*t.stride())


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _tma_ready(x: torch.Tensor) -> torch.Tensor:
    """Return x if TMA can read it in place, else a zero-padded contiguous copy.

    TMA needs a 16-byte aligned base and 16-byte multiple strides; the padding (zeros on the
    last dimension) does not change any dot product over that dimension.
    """
    esz = x.element_size()
    ok = x.stride(-1) == 1 and x.data_ptr() % 16 == 0
    if ok:
        for d in range(x.dim() - 1):
            if x.size(d) > 1 and (x.stride(d) * esz) % 16 != 0:
                ok = False
                break
    if ok:
        return x
    mult = 16 // esz
    n = x.size(-1)
    npad = (n + mult - 1) // mult * mult
    y = torch.zeros(*x.shape[:-1], npad, dtype=x.dtype, device=x.device)
    y[..., :n].copy_(x)
    return y


# Kernel kinds of the launch-timing hook, in the order of bdh_profile_end's arrays
# (BDH_PROF_KINDS in include/bdh_sm100.h).
PROF_KINDS = ("score", "value", "rope", "decode", "grad_q", "grad_v", "split", "gated_product",
              "state", "encode", "gate", "norm", "decoder")


def profile_begin() -> None:
    """Start timing every launch of the library (CUDA events around each kernel)."""
    lib = _require_lib()
    lib.bdh_profile_begin.restype = ctypes.c_int
    _check(lib.bdh_profile_begin(), "profile_begin")


def profile_end() -> dict:
    """Stop timing; returns {kind: {"ms": summed device ms, "launches": count}}."""
    lib = _require_lib()
    n = len(PROF_KINDS)
    ms = (ctypes.c_double * n)()
    cnt = (ctypes.c_int * n)()
    lib.bdh_profile_end.restype = ctypes.c_int
    _check(lib.bdh_profile_end(ms, cnt), "profile_end")
    return {k: {"ms": ms[i], "launches": cnt[i]} for i, k in enumerate(PROF_KINDS)}


FWD_ALGOS = {"auto": 0, "quadratic": 1, "chunked": 2}


def set_forward_algo(algo: str) -> str:
    """Select the forward form process-wide: ``auto`` (chunked for bf16 at T >= 1536),
    ``quadratic`` or ``chunked``. Returns the previous setting."""
    if algo not in FWD_ALGOS:
        raise ValueError(f"forward algo must be one of {sorted(FWD_ALGOS)}, got {algo!r}")
    prev = _require_lib().bdh_set_forward_algo(FWD_ALGOS[algo])
    return {v: k for k, v in FWD_ALGOS.items()}[prev]


SCORE_TERMS = {"default": -1, "bf16": 0, "split": 1}


@contextlib.contextmanager
def score_terms_scope(mode: Optional[str]):
    """For the calling thread, how bf16 score-like operands enter their second tensor-core
    product: ``"bf16"`` rounds each fp32 score once to bf16 (the reference's autocast chain,
    ``(q @ k.mT).tril_(-1) @ v`` with bf16 scores), ``"split"`` keeps it exact as a bf16 hi + lo
    pair, ``"default"``/None the process default. fp32 inputs are unaffected."""
    if mode is None:
        yield
        return
    if mode not in SCORE_TERMS:
        raise ValueError(f"score terms must be one of {sorted(SCORE_TERMS)}, got {mode!r}")
    lib = _require_lib()
    prev = lib.bdh_set_score_terms(SCORE_TERMS[mode])
    try:
        yield
    finally:
        lib.bdh_set_score_terms(prev)


# -------------------------------------------------------------------------- forward
def tril_score_v(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *,
                 score_terms: Optional[str] = None, ln_eps: Optional[float] = None) -> torch.Tensor:
    """``(q @ k.mT).tril(-1) @ v`` on the sm_100a tensor cores (fp32 accumulation).

    ``score_terms`` (bf16 inputs): ``"bf16"`` rounds the scores to bf16 before the product with
    ``v`` as the reference's eager autocast path does, ``"split"`` keeps them exact; None: the
    process default (exact for the quadratic form). ``ln_eps``: each output row is LayerNormed
    (affine-free, over D, that eps) before the store (``bdh_tril_score_v_layernorm``: in the value
    pass's epilogue for the quadratic bf16 form)."""
    if score_terms is not None:
        with score_terms_scope(score_terms):
            return tril_score_v(q, k, v, ln_eps=ln_eps)
    _check_cold_shapes(q, k, v)
    dev = _require_cuda(q, k, v)
    lib = _require_lib()
    B, H, T, N = q.shape
    Hv, D = v.size(1), v.size(-1)
    dt = _code(q.dtype)
    if k.dtype != q.dtype or v.dtype != q.dtype:
        raise TypeError(f"cuda_sm100: q, k, v dtypes must match, got {q.dtype}, {k.dtype}, {v.dtype}")
    out = torch.empty(B, H, T, D, dtype=q.dtype, device=dev)
    if out.numel() == 0:
        return out
    same = k is q
    qq = _tma_ready(q)
    kk = qq if same else _tma_ready(k)
    vv = _tma_ready(v)
    Np = qq.size(-1)
    Dp = vv.size(-1)
    if Dp != D:
        out_full = torch.empty(B, H, T, Dp, dtype=q.dtype, device=dev)
    else:
        out_full = out
    k_is_q = 1 if kk is qq else 0
    if ln_eps is not None and Dp != D:
        raise ValueError("tril_score_v: the fused LayerNorm needs D a multiple of 16 bytes")
    wsz = lib.bdh_tril_score_v_workspace_size(dt, B, H, Hv, T, Np, Dp, k_is_q)
    ws = torch.empty(max(int(wsz), 1), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        if ln_eps is None:
            rc = lib.bdh_tril_score_v(
                qq.data_ptr(), _strides(qq), kk.data_ptr(), _strides(kk), vv.data_ptr(),
                _strides(vv), dt, out_full.data_ptr(), _strides(out_full), dt, B, H, Hv, T, Np,
                Dp, ws.data_ptr(), int(wsz), _stream(dev))
        else:
            rc = lib.bdh_tril_score_v_layernorm(
                qq.data_ptr(), _strides(qq), kk.data_ptr(), _strides(kk), vv.data_ptr(),
                _strides(vv), dt, out_full.data_ptr(), _strides(out_full), dt, B, H, Hv, T, Np,
                Dp, float(ln_eps), ws.data_ptr(), int(wsz), _stream(dev))
    _check(rc, "tril_score_v")
    if out_full is not out:
        out.copy_(out_full[..., :D])
    return out


def rope_rotate(x: torch.Tensor, freqs: torch.Tensor, pos0: int = 0,
                out: Optional[torch.Tensor] = None, relu_input: bool = False) -> torch.Tensor:
    """BDH RoPE of ``x`` (B,H,T,N) at positions ``pos0 .. pos0+T-1`` computed in registers.

    Same arithmetic as ``Attention.rope`` with the ``rope_cos_sin`` tables (bdh.py:119-150,
    kernels/rope.py:108-126) but without materialising the tables. ``out`` may be a strided
    view (e.g. a cache slot) of another dtype; it must not overlap ``x``. ``relu_input``
    rotates ``relu(x)`` (the encoder's ReLU folded into the read).
    """
    if x.dim() != 4:
        raise ValueError("rope_rotate expects a 4-D (B, H, T, N) tensor")
    if x.size(-1) % 2 != 0:
        raise ValueError(f"RoPE last dim must be even, got {x.size(-1)}")
    dev = _require_cuda(x, freqs)
    lib = _require_lib()
    f = freqs.reshape(-1)
    if f.dtype != torch.float32 or f.numel() != x.size(-1):
        raise ValueError("freqs must be float32 with one entry per latent dimension")
    f = f.contiguous()
    if out is None:
        out = torch.empty(x.shape, dtype=x.dtype, device=dev)
    elif out.shape != x.shape or out.device != x.device:
        raise ValueError("rope out= must match x shape/device")
    elif torch._C._overlaps(out, x):
        raise ValueError("rope out= must not alias x")
    if x.stride(-1) != 1:
        x = x.contiguous()
    if out.stride(-1) != 1:
        raise ValueError("rope out= must have a contiguous last dimension")
    B, H, T, N = x.shape
    with torch.cuda.device(dev):
        rc = lib.bdh_rope_rotate(x.data_ptr(), _code(x.dtype), _strides(x), out.data_ptr(),
                                 _code(out.dtype), _strides(out), None, f.data_ptr(),
                                 B, H, T, N, int(pos0), 1 if relu_input else 0, _stream(dev))
    _check(rc, "rope_rotate")
    return out


def relu_mul(x: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
    """``relu(x) * relu(y)`` for 4-D tensors of one dtype (contiguous last dim, any strides),
    returned contiguous in ``x``'s shape — the gated product of a BDH layer."""
    if x.dim() != 4 or x.shape != y.shape or x.dtype != y.dtype:
        raise ValueError("relu_mul expects two 4-D tensors of the same shape and dtype")
    dev = _require_cuda(x, y)
    lib = _require_lib()
    if x.stride(-1) != 1:
        x = x.contiguous()
    if y.stride(-1) != 1:
        y = y.contiguous()
    out = torch.empty(x.shape, dtype=x.dtype, device=dev)
    B, H, T, N = x.shape
    with torch.cuda.device(dev):
        rc = lib.bdh_relu_mul(x.data_ptr(), _strides(x), y.data_ptr(), _strides(y), out.data_ptr(),
                              _strides(out), _code(x.dtype), B, H, T, N, _stream(dev))
    _check(rc, "relu_mul")
    return out


def decoder_f32(x: torch.Tensor, w: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """fp32 ``x @ w`` for a decode step's decoder product (x: (M, K) with unit column stride,
    w: (K, D) row-major, D a multiple of 4), K split across the GPU and summed in a fixed order
    (bdh_decoder_f32). ``out``: optional (M, D) fp32 destination with unit column stride."""
    if x.dim() != 2 or w.dim() != 2 or x.size(1) != w.size(0):
        raise ValueError("decoder_f32 expects x (M, K) and w (K, D)")
    if x.dtype != torch.float32 or w.dtype != torch.float32:
        raise ValueError("decoder_f32 expects fp32 tensors")
    dev = _require_cuda(x, w)
    lib = _require_lib()
    if x.stride(1) != 1:
        x = x.contiguous()
    if w.stride(1) != 1 or w.stride(0) % 4 != 0 or w.data_ptr() % 16 != 0:
        w = w.contiguous()
    M, K = x.shape
    D = w.size(1)
    if out is None:
        out = torch.empty((M, D), dtype=torch.float32, device=dev)
    elif out.shape != (M, D) or out.dtype != torch.float32 or out.stride(1) != 1:
        raise ValueError("decoder_f32: out must be an fp32 (M, D) tensor with unit column stride")
    part = torch.empty(int(lib.bdh_decoder_f32_slices(K)) * M * D, dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        rc = lib.bdh_decoder_f32(x.data_ptr(), x.stride(0), w.data_ptr(), w.stride(0),
                                 out.data_ptr(), out.stride(0), part.data_ptr(), M, K, D,
                                 _stream(dev))
    _check(rc, "decoder_f32")
    return out


# ------------------------------------------------------------ latent projections
_PAIRED: dict = {}


def _check_paired_freqs(f: torch.Tensor) -> None:
    """The fused encode shares one (cos, sin) per column pair: freqs[2p] must equal freqs[2p+1]
    (BDH's get_freqs, bdh.py:41-49). Checked once per freqs tensor version."""
    key = (f.data_ptr(), f._version, f.numel())
    ok = _PAIRED.get(key)
    if ok is None:
        ok = bool(torch.equal(f[0::2], f[1::2]))
        _PAIRED[key] = ok
    if not ok:
        raise ValueError("latent_encode requires paired frequencies (freqs[2p] == freqs[2p+1])")


_c_i64_2 = ctypes.c_int64 * 2
_c_i64_3 = ctypes.c_int64 * 3


def _check_latent(name: str, *ts: torch.Tensor, weight: Optional[torch.Tensor] = None) -> None:
    for t in ts:
        if t.dtype != torch.bfloat16:
            raise TypeError(f"{name}: bf16 tensors required, got {t.dtype}")
        if t.stride(-1) != 1 or t.data_ptr() % 16 != 0 or any(
                st % 8 != 0 for st, sz in zip(t.stride()[:-1], t.shape[:-1]) if sz > 1):
            raise ValueError(f"{name}: tensors need a contiguous last dim, 16-byte aligned base "
                             "and strides that are multiples of 8 elements")
    if weight is not None:
        if weight.dtype != torch.bfloat16:
            raise TypeError(f"{name}: bf16 weights required, got {weight.dtype}")
        s = weight.stride()
        k_major = s[1] == 1 and s[2] != 1 and s[0] % 8 == 0 and s[2] % 8 == 0
        if not k_major:
            _check_latent(name, weight)
        elif weight.data_ptr() % 16 != 0:
            raise ValueError(f"{name}: weights need a 16-byte aligned base")


def weight_k_major(w: torch.Tensor) -> torch.Tensor:
    """(H, D, N) weights as a view of a contiguous (H, N, D) copy: the layout the latent kernels
    read K-major (faster than the n-contiguous layout)."""
    return w.transpose(1, 2).contiguous().transpose(1, 2)


def _st(t: torch.Tensor, n: int):
    # strides of size-1 dims are never stepped; give them a legal value
    st = [s if (sz > 1 or s % 8 == 0 or s == 1) else 8 for s, sz in zip(t.stride(), t.shape)]
    st[-1] = t.stride(-1)
    return {2: _c_i64_2, 3: _c_i64_3, 4: _c_i64_4}[n](*st)


def latent_encode(x: torch.Tensor, enc: torch.Tensor, freqs: torch.Tensor, pos0: int = 0, *,
                  xs_out: Optional[torch.Tensor] = None,
                  qr_out: Optional[torch.Tensor] = None, want_xs: bool = True):
    """Fused ``xs = relu(x @ enc)`` (B,T,H,N) and ``qr = RoPE(xs)`` (B,H,T,N), bf16.

    ``x`` (B,T,D), ``enc`` (H,D,N). ``qr_out`` may be a strided view (a cache slot); returns
    ``(xs, qr)``, with ``xs`` None when ``want_xs`` is False (qr only: the caller recomputes xs
    in ``latent_gate_x``). Replaces ``BDH._encoder_relu`` (bdh.py:861-889) followed by the
    attention's RoPE apply (bdh.py:396-412).
    """
    if x.dim() != 3 or enc.dim() != 3 or x.size(-1) != enc.size(1):
        raise ValueError("latent_encode expects x (B,T,D) and enc (H,D,N)")
    dev = _require_cuda(x, enc, freqs)
    lib = _require_lib()
    B, T, D = x.shape
    H, _, N = enc.shape
    f = freqs.reshape(-1)
    if f.dtype != torch.float32 or f.numel() != N:
        raise ValueError("freqs must be float32 with one entry per latent dimension")
    f = f.contiguous()
    _check_paired_freqs(f)
    if xs_out is None and want_xs:
        xs_out = torch.empty(B, T, H, N, dtype=torch.bfloat16, device=dev)
    if qr_out is None:
        qr_out = torch.empty(B, H, T, N, dtype=torch.bfloat16, device=dev)
    if (xs_out is not None and tuple(xs_out.shape) != (B, T, H, N)) or \
            tuple(qr_out.shape) != (B, H, T, N):
        raise ValueError("latent_encode: xs_out must be (B,T,H,N) and qr_out (B,H,T,N)")
    outs = (qr_out,) if xs_out is None else (xs_out, qr_out)
    _check_latent("latent_encode", x, *outs, weight=enc)
    xs_ptr = None if xs_out is None else xs_out.data_ptr()
    xs_st = None if xs_out is None else _st(xs_out, 4)
    with torch.cuda.device(dev):
        rc = lib.bdh_latent_encode(x.data_ptr(), _st(x, 3), enc.data_ptr(), _st(enc, 3),
                                   xs_ptr, xs_st, qr_out.data_ptr(),
                                   _st(qr_out, 4), f.data_ptr(), B, T, H, D, N, int(pos0),
                                   _stream(dev))
    _check(rc, "latent_encode")
    return xs_out, qr_out


def latent_gate(y: torch.Tensor, encv: torch.Tensor, xs: torch.Tensor, *,
                out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Fused ``xy = xs * relu(y @ encv)`` in the (B,T,H,N) latent layout, bf16.

    ``y`` (B,H,T,D) (the LayerNormed attention output), ``encv`` (H,D,N), ``xs`` (B,T,H,N).
    Replaces ``BDH._encoder_v_relu`` and the product of ``_mlp_merge`` (bdh.py:914-945).
    """
    if y.dim() != 4 or encv.dim() != 3 or xs.dim() != 4 or y.size(-1) != encv.size(1):
        raise ValueError("latent_gate expects y (B,H,T,D), encv (H,D,N), xs (B,T,H,N)")
    dev = _require_cuda(y, encv, xs)
    lib = _require_lib()
    B, H, T, D = y.shape
    N = encv.size(-1)
    if tuple(xs.shape) != (B, T, H, N) or encv.size(0) != H:
        raise ValueError("latent_gate: shapes of y, encv and xs disagree")
    if out is None:
        out = torch.empty(B, T, H, N, dtype=torch.bfloat16, device=dev)
    elif tuple(out.shape) != (B, T, H, N):
        raise ValueError("latent_gate: out must be (B,T,H,N)")
    _check_latent("latent_gate", y, xs, out, weight=encv)
    with torch.cuda.device(dev):
        rc = lib.bdh_latent_gate(y.data_ptr(), _st(y, 4), encv.data_ptr(), _st(encv, 3),
                                 xs.data_ptr(), _st(xs, 4), out.data_ptr(), _st(out, 4),
                                 B, T, H, D, N, _stream(dev))
    _check(rc, "latent_gate")
    return out


def latent_gate_x(y: torch.Tensor, encv: torch.Tensor, x: torch.Tensor, enc: torch.Tensor, *,
                  out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``xy = relu(x @ enc) * relu(y @ encv)`` in the (B,T,H,N) latent layout, bf16, with the
    encoder product recomputed in the gate kernel instead of read back (bit-identical to
    ``latent_encode``'s xs), so no xs latent is stored.

    ``y`` (B,H,T,D), ``encv`` and ``enc`` (H,D,N) with one layout, ``x`` (B,T,D); D <= 256.
    Replaces ``BDH._encoder_relu``'s output use, ``_encoder_v_relu`` and the product of
    ``_mlp_merge`` (bdh.py:861-945).
    """
    if y.dim() != 4 or encv.dim() != 3 or enc.dim() != 3 or x.dim() != 3:
        raise ValueError("latent_gate_x expects y (B,H,T,D), encv (H,D,N), x (B,T,D), enc (H,D,N)")
    dev = _require_cuda(y, encv, x, enc)
    lib = _require_lib()
    B, H, T, D = y.shape
    N = encv.size(-1)
    if tuple(x.shape) != (B, T, D) or tuple(enc.shape) != (H, D, N) or tuple(encv.shape) != (H, D, N):
        raise ValueError("latent_gate_x: shapes of y, encv, x and enc disagree")
    if out is None:
        out = torch.empty(B, T, H, N, dtype=torch.bfloat16, device=dev)
    elif tuple(out.shape) != (B, T, H, N):
        raise ValueError("latent_gate_x: out must be (B,T,H,N)")
    _check_latent("latent_gate_x", y, x, out, weight=encv)
    _check_latent("latent_gate_x", weight=enc)
    with torch.cuda.device(dev):
        rc = lib.bdh_latent_gate_x(y.data_ptr(), _st(y, 4), encv.data_ptr(), _st(encv, 3),
                                   x.data_ptr(), _st(x, 3), enc.data_ptr(), _st(enc, 3),
                                   out.data_ptr(), _st(out, 4), B, T, H, D, N, _stream(dev))
    _check(rc, "latent_gate_x")
    return out


def decoder_k_major(dec: torch.Tensor) -> torch.Tensor:
    """(H*N, D) decoder as a view of a contiguous (D, H*N) copy: the layout
    ``latent_gate_dec`` reads (the latent index contiguous)."""
    return dec.t().contiguous().t()


def latent_gate_dec(y: torch.Tensor, encv: torch.Tensor, xs: torch.Tensor, dec: torch.Tensor, *,
                    out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``(xs * relu(y @ encv)) @ dec`` in one kernel: the gate of ``latent_gate`` followed by
    the decoder product (bdh.py:914-945 and :1050 under bf16 autocast), each xy tile kept in
    shared memory, never written to HBM. Returns (B, T, D) bf16.

    ``y`` (B,H,T,D), ``encv`` (H,D,N) with d contiguous (``weight_k_major``), ``xs``
    (B,T,H,N), ``dec`` (H*N, D) with the latent index contiguous (``decoder_k_major``);
    D = 256 and N a multiple of 128.
    """
    if y.dim() != 4 or encv.dim() != 3 or xs.dim() != 4 or dec.dim() != 2:
        raise ValueError("latent_gate_dec expects y (B,H,T,D), encv (H,D,N), xs (B,T,H,N), "
                         "dec (H*N,D)")
    dev = _require_cuda(y, encv, xs, dec)
    lib = _require_lib()
    B, H, T, D = y.shape
    N = encv.size(-1)
    if tuple(xs.shape) != (B, T, H, N) or tuple(encv.shape) != (H, D, N) or \
            tuple(dec.shape) != (H * N, D):
        raise ValueError("latent_gate_dec: shapes of y, encv, xs and dec disagree")
    if D != 256 or N % 128 != 0:
        raise ValueError("latent_gate_dec: needs D = 256 and N a multiple of 128")
    if dec.dtype != torch.bfloat16 or encv.dtype != torch.bfloat16:
        raise TypeError("latent_gate_dec: bf16 weights required")
    if out is None:
        out = torch.empty(B, T, D, dtype=torch.bfloat16, device=dev)
    elif tuple(out.shape) != (B, T, D):
        raise ValueError("latent_gate_dec: out must be (B,T,D)")
    _check_latent("latent_gate_dec", y, xs, out, weight=encv)
    with torch.cuda.device(dev):
        # few rows (a small batch): the latent walk is split across the GPU, its range sums in
        # a workspace from the caching allocator
        wsz = int(lib.bdh_latent_gate_dec_workspace_size(B, T, H, D, N))
        ws = torch.empty(max(wsz, 1), dtype=torch.uint8, device=dev) if wsz else None
        rc = lib.bdh_latent_gate_dec_ws(y.data_ptr(), _st(y, 4), encv.data_ptr(), _st(encv, 3),
                                        xs.data_ptr(), _st(xs, 4), dec.data_ptr(), _st(dec, 2),
                                        out.data_ptr(), _st(out, 3), B, T, H, D, N,
                                        ws.data_ptr() if ws is not None else None, wsz,
                                        _stream(dev))
    _check(rc, "latent_gate_dec")
    return out


# ---------------------------------------------------------------------- layer norms
def _rows_view(t: torch.Tensor):
    """(rows, D) with one row stride, or None when t's leading dims do not flatten to one."""
    if t.stride(-1) != 1:
        return None
    try:
        v = t.view(-1, t.size(-1))
    except RuntimeError:
        return None
    return v


def layer_norm(x: torch.Tensor, eps: float = 1e-5, out_dtype: Optional[torch.dtype] = None,
               out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Affine-free LayerNorm over the last dim (``F.layer_norm(x, (D,), eps=eps)``), fp32 math,
    result stored in ``out_dtype`` (default: x's dtype). One kernel, no fp32 intermediate."""
    dev = _require_cuda(x)
    lib = _require_lib()
    D = x.size(-1)
    xv = _rows_view(x)
    if xv is None:
        xv = x.contiguous().view(-1, D)
    if out is None:
        out = torch.empty(x.shape, dtype=out_dtype or x.dtype, device=dev)
    ov = _rows_view(out)
    if ov is None or ov.size(0) != xv.size(0):
        raise ValueError("layer_norm: out must be row-contiguous with x's shape")
    with torch.cuda.device(dev):
        rc = lib.bdh_layernorm(xv.data_ptr(), _code(xv.dtype), xv.stride(0) if xv.size(0) > 1 else D,
                               ov.data_ptr(), _code(ov.dtype), ov.stride(0) if ov.size(0) > 1 else D,
                               xv.size(0), D, float(eps), _stream(dev))
    _check(rc, "layer_norm")
    return out


def residual_layer_norm(x: torch.Tensor, y: torch.Tensor, eps: float = 1e-5,
                        want_bf16: bool = False):
    """``LN(x + LN(y))`` over the last dim (BDH._residual_ln): x fp32, y fp32 or bf16. Returns
    the fp32 result and, with ``want_bf16``, its bf16 copy (else None)."""
    if x.dtype != torch.float32 or x.shape != y.shape:
        raise ValueError("residual_layer_norm: x must be fp32 and y of x's shape")
    dev = _require_cuda(x, y)
    lib = _require_lib()
    D = x.size(-1)
    xv = _rows_view(x)
    if xv is None:
        xv = x.contiguous().view(-1, D)
    yv = _rows_view(y)
    if yv is None:
        yv = y.contiguous().view(-1, D)
    out = torch.empty(x.shape, dtype=torch.float32, device=dev)
    out16 = torch.empty(x.shape, dtype=torch.bfloat16, device=dev) if want_bf16 else None
    rs = lambda v: v.stride(0) if v.size(0) > 1 else D  # noqa: E731
    with torch.cuda.device(dev):
        rc = lib.bdh_residual_layernorm(
            xv.data_ptr(), rs(xv), yv.data_ptr(), _code(yv.dtype), rs(yv), out.data_ptr(), D,
            out16.data_ptr() if out16 is not None else None, D, xv.size(0), D, float(eps),
            _stream(dev))
    _check(rc, "residual_layer_norm")
    return out, out16


# --------------------------------------------------------------------------- decode
def tril_decode(q: torch.Tensor, k_past: torch.Tensor, v_past: torch.Tensor, *,
                freqs: Optional[torch.Tensor] = None, pos: int = 0,
                kr_slot: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``(q @ k_past.mT) @ v_past`` streaming the (possibly capacity-strided) cache in place.

    ``k_past``/``v_past`` may be stored in another dtype than ``q`` (e.g. bf16 cache storage
    with fp32 compute): they are widened in registers, never copied. With ``freqs`` the query
    is RoPE-rotated to positions ``pos..`` first, and with ``kr_slot`` the rotated rows are
    also written there (the cache write of this step).
    """
    B, H, Tq, S, D = _check_decode_shapes(q, k_past, v_past)
    dev = _require_cuda(q, k_past, v_past)
    lib = _require_lib()
    if k_past.dtype != v_past.dtype:
        raise TypeError("k_past and v_past must share the cache storage dtype")
    qd = _code(q.dtype)
    kd = _code(k_past.dtype)
    out = torch.empty(B, H, Tq, D, dtype=q.dtype, device=dev)
    if out.numel() == 0:
        if kr_slot is not None and freqs is not None and Tq > 0:
            rope_rotate(q, freqs, pos, out=kr_slot)
        return out
    if q.stride(-1) != 1:
        q = q.contiguous()
    if k_past.stride(-1) != 1 or v_past.stride(-1) != 1:
        raise ValueError("cache views must have a contiguous last dimension")
    N = q.size(-1)
    fptr = None
    if freqs is not None:
        f = freqs.reshape(-1)
        if f.dtype != torch.float32 or f.numel() != N:
            raise ValueError("freqs must be float32 with one entry per latent dimension")
        f = f.contiguous()
        fptr = f.data_ptr()
    slot_ptr = None
    slot_strides = None
    if kr_slot is not None:
        if freqs is None:
            raise ValueError("kr_slot requires freqs (the slot receives the rotated query)")
        if kr_slot.shape != q.shape or kr_slot.dtype != k_past.dtype or kr_slot.stride(-1) != 1:
            raise ValueError("kr_slot must match q's shape, the cache dtype and have unit last stride")
        slot_ptr = kr_slot.data_ptr()
        slot_strides = _strides(kr_slot)
    wsz = lib.bdh_tril_decode_workspace_size(B, H, Tq, S, N, D)
    ws = torch.empty(max(int(wsz), 4), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        rc = lib.bdh_tril_decode(
            q.data_ptr(), _strides(q), qd, k_past.data_ptr(), _strides(k_past), v_past.data_ptr(),
            _strides(v_past), kd, out.data_ptr(), _strides(out), B, H, v_past.size(1), Tq, S, N, D,
            fptr, int(pos), slot_ptr, slot_strides, ws.data_ptr(), int(wsz), _stream(dev))
    _check(rc, "tril_decode")
    return out


def _strides3(t: torch.Tensor):
    return (ctypes.c_int64 * 3)(*t.stride())


def quantize_rows_fp8(x: torch.Tensor, *, out: Optional[torch.Tensor] = None,
                      scale: Optional[torch.Tensor] = None):
    """Row-scaled e4m3 of ``x`` (B,H,T,N) f32 / bf16: ``out`` (B,H,T,N) float8_e4m3fn with
    x ~= out * scale[..., None], ``scale`` (B,H,T) fp32 = max|row| / 448. Either may be a
    strided view (a cache slot). Returns ``(out, scale)``."""
    if x.dim() != 4:
        raise ValueError("quantize_rows_fp8 expects x (B,H,T,N)")
    dev = _require_cuda(x)
    lib = _require_lib()
    B, H, T, N = x.shape
    if out is None:
        out = torch.empty(B, H, T, N, dtype=FP8, device=dev)
    if scale is None:
        scale = torch.empty(B, H, T, dtype=torch.float32, device=dev)
    if out.dtype != FP8 or tuple(out.shape) != (B, H, T, N) or out.stride(-1) != 1:
        raise ValueError("quantize_rows_fp8: out must be float8_e4m3fn (B,H,T,N) with unit last stride")
    if scale.dtype != torch.float32 or tuple(scale.shape) != (B, H, T):
        raise ValueError("quantize_rows_fp8: scale must be float32 (B,H,T)")
    if x.stride(-1) != 1:
        x = x.contiguous()
    with torch.cuda.device(dev):
        rc = lib.bdh_quantize_rows_fp8(x.data_ptr(), _strides(x), _code(x.dtype), B, H, T, N,
                                       out.data_ptr(), _strides(out), scale.data_ptr(),
                                       _strides3(scale), _stream(dev))
    _check(rc, "quantize_rows_fp8")
    return out, scale


def tril_decode_fp8(q: torch.Tensor, k_past: torch.Tensor, k_scale: torch.Tensor,
                    v_past: torch.Tensor, *, freqs: Optional[torch.Tensor] = None, pos: int = 0,
                    kr_slot: Optional[torch.Tensor] = None,
                    slot_scale: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``tril_decode`` against an fp8 key history: ``k_past`` (B,H,S,N) float8_e4m3fn rows
    with ``k_scale`` (B,H,S) fp32, ``v_past`` f32 / bf16 (capacity-strided views read in place).
    With ``freqs`` the query is rotated first; with ``kr_slot`` / ``slot_scale`` the rotated
    rows are quantized into this step's cache slot."""
    B, H, Tq, S, D = _check_decode_shapes(q, k_past, v_past)
    dev = _require_cuda(q, k_past, v_past, k_scale)
    lib = _require_lib()
    if k_past.dtype != FP8:
        raise TypeError("tril_decode_fp8: k_past must be float8_e4m3fn")
    if k_scale.dtype != torch.float32 or tuple(k_scale.shape) != (B, H, S):
        raise ValueError("tril_decode_fp8: k_scale must be float32 (B,H,S)")
    out = torch.empty(B, H, Tq, D, dtype=q.dtype, device=dev)
    if q.stride(-1) != 1:
        q = q.contiguous()
    if k_past.stride(-1) != 1 or v_past.stride(-1) != 1:
        raise ValueError("cache views must have a contiguous last dimension")
    N = q.size(-1)
    fptr = None
    if freqs is not None:
        f = freqs.reshape(-1)
        if f.dtype != torch.float32 or f.numel() != N:
            raise ValueError("freqs must be float32 with one entry per latent dimension")
        f = f.contiguous()
        fptr = f.data_ptr()
    slot_ptr = slot_st = sc_ptr = sc_st = None
    if kr_slot is not None:
        if freqs is None or slot_scale is None:
            raise ValueError("kr_slot requires freqs and slot_scale")
        if kr_slot.shape != q.shape or kr_slot.dtype != FP8 or kr_slot.stride(-1) != 1:
            raise ValueError("kr_slot must be float8_e4m3fn with q's shape and unit last stride")
        if slot_scale.dtype != torch.float32 or tuple(slot_scale.shape) != (B, H, Tq):
            raise ValueError("slot_scale must be float32 (B,H,Tq)")
        slot_ptr, slot_st = kr_slot.data_ptr(), _strides(kr_slot)
        sc_ptr, sc_st = slot_scale.data_ptr(), _strides3(slot_scale)
    if out.numel() == 0:
        return out
    wsz = lib.bdh_tril_decode_workspace_size(B, H, Tq, S, N, D)
    ws = torch.empty(max(int(wsz), 4), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        rc = lib.bdh_tril_decode_fp8(
            q.data_ptr(), _strides(q), _code(q.dtype), k_past.data_ptr(), _strides(k_past),
            k_scale.data_ptr(), _strides3(k_scale), v_past.data_ptr(), _strides(v_past),
            _code(v_past.dtype), out.data_ptr(), _strides(out), B, H, v_past.size(1), Tq, S, N, D,
            fptr, int(pos), slot_ptr, slot_st, sc_ptr, sc_st, ws.data_ptr(), int(wsz),
            _stream(dev))
    _check(rc, "tril_decode_fp8")
    return out


def state_decode(q: torch.Tensor, state: torch.Tensor, v: torch.Tensor, freqs: torch.Tensor,
                 pos: int, *, relu_input: bool = False) -> torch.Tensor:
    """One decode step against an N x D recurrent state (updated in place).

    ``q`` (B,H,1,N) un-rotated query (``relu_input``: pre-activation), ``state`` (B,H,N,D) fp32
    holding sum_j k_j v_j^T over the past, ``v`` (B,Hv,1,D) this step's value. Returns
    ``RoPE(q) . state`` (the past only) in q's dtype and folds ``RoPE(q)^T v`` into the state.
    """
    if q.dim() != 4 or q.size(2) != 1 or state.dim() != 4 or v.dim() != 4:
        raise ValueError("state_decode expects q (B,H,1,N), state (B,H,N,D), v (B,Hv,1,D)")
    B, H, _, N = q.shape
    D = state.size(-1)
    if tuple(state.shape) != (B, H, N, D) or state.dtype != torch.float32:
        raise ValueError("state must be fp32 (B,H,N,D) matching q")
    if v.size(0) != B or v.size(1) not in (1, H) or v.size(2) != 1 or v.size(3) != D:
        raise ValueError("v must be (B,1 or H,1,D)")
    dev = _require_cuda(q, state, v, freqs)
    lib = _require_lib()
    f = freqs.reshape(-1)
    if f.dtype != torch.float32 or f.numel() != N:
        raise ValueError("freqs must be float32 with one entry per latent dimension")
    f = f.contiguous()
    if q.stride(-1) != 1:
        q = q.contiguous()
    if v.stride(-1) != 1:
        v = v.contiguous()
    out = torch.empty(B, H, 1, D, dtype=q.dtype, device=dev)
    wsz = lib.bdh_state_decode_workspace_size(B, H, N, D)
    ws = torch.empty(max(int(wsz), 4), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        rc = lib.bdh_state_decode(q.data_ptr(), _strides(q), _code(q.dtype), state.data_ptr(),
                                  _strides(state), v.data_ptr(), _strides(v), _code(v.dtype),
                                  out.data_ptr(), _strides(out), B, H, v.size(1), N, D,
                                  f.data_ptr(), int(pos), 1 if relu_input else 0, ws.data_ptr(),
                                  int(wsz), _stream(dev))
    _check(rc, "state_decode")
    return out


# ------------------------------------------------------------------------- backward
def tril_score_v_bwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, dout: torch.Tensor,
                     *, freqs: Optional[torch.Tensor] = None, pos0: int = 0):
    """Analytic gradients of ``tril(q k^T, -1) v``: returns ``(dq, dk, dv)``.

    When ``k is q`` the returned ``dq`` already holds ``dq + dk`` and ``dk`` is None (the
    self-attention form of ``StrictTrilSelfAttnFn``). With ``freqs`` (self form only) ``q`` is
    the rotated QR and ``dq`` is the gradient with respect to the unrotated latent.
    """
    _check_cold_shapes(q, k, v)
    dev = _require_cuda(q, k, v, dout)
    lib = _require_lib()
    B, H, T, N = q.shape
    Hv, D = v.size(1), v.size(-1)
    if dout.shape != (B, H, T, D):
        raise ValueError(f"dout shape {tuple(dout.shape)} must be {(B, H, T, D)}")
    dt = _code(q.dtype)
    same = k is q
    if freqs is not None and not same:
        raise ValueError("the fused RoPE adjoint needs the self-attention form (k is q)")
    qq = _tma_ready(q)
    kk = qq if same else _tma_ready(k)
    vv = _tma_ready(v)
    dd = _tma_ready(dout.to(q.dtype))
    Np, Dp = qq.size(-1), vv.size(-1)
    if dd.size(-1) != Dp:
        dd = torch.nn.functional.pad(dd, (0, Dp - dd.size(-1)))
    dq = torch.empty(B, H, T, Np, dtype=q.dtype, device=dev)
    dk = None if same else torch.empty(B, H, T, Np, dtype=q.dtype, device=dev)
    dv = torch.empty(B, Hv, T, Dp, dtype=q.dtype, device=dev)
    fptr = None
    if freqs is not None:
        f = freqs.reshape(-1).contiguous()
        if f.dtype != torch.float32 or f.numel() != N:
            raise ValueError("freqs must be float32 with one entry per latent dimension")
        if Np != N:
            raise ValueError("the fused RoPE adjoint needs an aligned latent width")
        fptr = f.data_ptr()
    k_is_q = 1 if same else 0
    wsz = lib.bdh_tril_score_v_bwd_workspace_size(dt, B, H, Hv, T, Np, Dp, k_is_q)
    ws = torch.empty(max(int(wsz), 1), dtype=torch.uint8, device=dev)
    dk_ptr = dk.data_ptr() if dk is not None else None
    dk_str = _strides(dk) if dk is not None else _strides(dq)
    with torch.cuda.device(dev):
        rc = lib.bdh_tril_score_v_bwd(
            qq.data_ptr(), _strides(qq), kk.data_ptr(), _strides(kk), vv.data_ptr(), _strides(vv),
            dd.data_ptr(), _strides(dd), dt, dq.data_ptr(), _strides(dq), dk_ptr, dk_str,
            dv.data_ptr(), _strides(dv), B, H, Hv, T, Np, Dp, fptr, int(pos0),
            ws.data_ptr(), int(wsz), _stream(dev))
    _check(rc, "tril_score_v_bwd")
    if Np != N:
        dq = dq[..., :N].contiguous()
        dk = dk[..., :N].contiguous() if dk is not None else None
    if Dp != D:
        dv = dv[..., :D].contiguous()
    return dq, dk, dv


__all__ = [
    "load_library",
    "has_cuda_ext",
    "has_cuda_kernel",
    "ext_status",
    "device_error",
    "tril_score_v",
    "tril_decode",
    "tril_score_v_bwd",
    "rope_rotate",
    "relu_mul",
    "set_forward_algo",
    "score_terms_scope",
]
