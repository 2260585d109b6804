"""CPU oracle for the BDH tril-attention path — TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg may import this
module, and only as the checker; the product path (libbdh_sm100.so through the ``kernels``
package) never routes through it.

A numpy restatement of the reference algorithm (katulevskiy/bdh-gpu-fast), each function
citing the reference lines it follows:

* ``get_freqs``        bdh.py:41-49 / bdh_baseline.py:21-29
* ``rope``             bdh.py:119-150 (phases, mod 1, 2pi, cos/sin) + kernels/rope.py:108-126
                        (pair rotation; bf16 inputs round each product before the add) /
                        bdh_baseline.py:50-54
* ``tril_score_v``     csrc/tril_attn_cpu.cpp:94-107,223-237; kernels/cuda_attn.py:293-310
* ``tril_decode``      csrc/tril_attn_cpu.cpp:241-300; kernels/attention.py:193-219
* ``tril_backward``    kernels/attention_bwd.py:45-83 (+ the K-is-Q sum of :284-291)
* ``rope_backward``    kernels/rope.py:540-557 (analytic adjoint of the rotation)
* ``bdh_forward``      bdh_baseline.py:96-139 (eval mode, dropout 0)
* ``quantize_rows_fp8`` / ``tril_decode_fp8``  the opt-in fp8 key-cache wire format (no
                        reference counterpart: the reference caches fp32 / fp16 / bf16,
                        bdh_cache.py:62-80,240-243); the decode over it is ``tril_decode`` on the
                        dequantized keys

Parity pinning: tests/golden/*.npz hold outputs of the reference itself (generated in the
build container by tests/golden/make_golden.py from the reference sources); the tests check
this oracle against them before using it as the GPU checker.

Accumulation is float64 by default (``acc=np.float64``): the GPU results are compared with a
relative-Frobenius tolerance, so the oracle is the more exact side of the comparison.
"""

from __future__ import annotations

import math

import numpy as np

TWO_PI_F32 = np.float32(2 * math.pi)  # the fp32 scalar torch multiplies by (bdh.py:121)


# ----------------------------------------------------------------------------- bf16
def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even); returns float32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    r = ((u + 0x7FFF + lsb) >> 16) << 16
    out = r.astype(np.uint32).view(np.float32)
    nan = np.isnan(x)
    if nan.any():
        out = out.copy()
        out[nan] = np.nan
    return out


def tf32_round(x: np.ndarray) -> np.ndarray:
    """Round float32 values to tf32 (10-bit mantissa, ties away from zero like cvt.rna)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    r = ((u + 0x1000) >> 13) << 13
    return r.astype(np.uint32).view(np.float32)


# ----------------------------------------------------------------------------- RoPE
def get_freqs(n: int, theta: float = 2.0 ** 16) -> np.ndarray:
    """freq[i] = 1 / theta^(2*floor(i/2)/n) / (2*pi) in float32 (bdh.py:41-49)."""
    t = np.arange(0, n, 1, dtype=np.float32)
    q = np.floor(t / np.float32(2)) * np.float32(2)
    e = (q / np.float32(n)).astype(np.float32)
    p = np.power(np.float32(theta), e, dtype=np.float32)
    return (np.float32(1.0) / p / np.float32(2 * math.pi)).astype(np.float32)


def rope_cos_sin(freqs: np.ndarray, T: int, pos0: int = 0):
    """(cos, sin) tables (T, N) float32: phase = ((pos0+t) * f mod 1) * 2pi (bdh.py:119-150)."""
    pos = np.arange(pos0, pos0 + T, dtype=np.float32)[:, None]
    ph = (pos * freqs.reshape(1, -1).astype(np.float32)).astype(np.float32)
    ph = (ph - np.floor(ph)).astype(np.float32)
    ph = (ph * TWO_PI_F32).astype(np.float32)
    return np.cos(ph).astype(np.float32), np.sin(ph).astype(np.float32)


def rope(x: np.ndarray, freqs: np.ndarray, pos0: int = 0, bf16: bool = False) -> np.ndarray:
    """Rotate adjacent pairs of x (..., T, N) (kernels/rope.py:108-126).

    bf16=True reproduces the bf16-input path: every product is rounded to bf16 and the bf16
    sum is rounded again (x must already hold bf16-representable values).
    """
    x = np.asarray(x, dtype=np.float32)
    T, N = x.shape[-2], x.shape[-1]
    c, s = rope_cos_sin(freqs, T, pos0)
    x0, x1 = x[..., 0::2], x[..., 1::2]
    c0, c1 = c[:, 0::2], c[:, 1::2]
    s0, s1 = s[:, 0::2], s[:, 1::2]
    if bf16:
        y0 = bf16_round(bf16_round(x0 * c0) + bf16_round(-x1 * s0))
        y1 = bf16_round(bf16_round(x1 * c1) + bf16_round(x0 * s1))
    else:
        y0 = (x0 * c0).astype(np.float32) - (x1 * s0).astype(np.float32)
        y1 = (x1 * c1).astype(np.float32) + (x0 * s1).astype(np.float32)
    y = np.empty_like(x)
    y[..., 0::2] = y0
    y[..., 1::2] = y1
    return y


def rope_backward(g: np.ndarray, freqs: np.ndarray, pos0: int = 0, acc=np.float64) -> np.ndarray:
    """dL/dx from dL/dy of the rotation: dx0 = g0 c0 + g1 s1, dx1 = -g0 s0 + g1 c1."""
    g = np.asarray(g, dtype=acc)
    T = g.shape[-2]
    c, s = rope_cos_sin(freqs, T, pos0)
    c = c.astype(acc)
    s = s.astype(acc)
    g0, g1 = g[..., 0::2], g[..., 1::2]
    dx = np.empty_like(g)
    dx[..., 0::2] = g0 * c[:, 0::2] + g1 * s[:, 1::2]
    dx[..., 1::2] = -g0 * s[:, 0::2] + g1 * c[:, 1::2]
    return dx


# ------------------------------------------------------------------------ attention
def tril_score_v(q: np.ndarray, k: np.ndarray, v: np.ndarray, acc=np.float64) -> np.ndarray:
    """out[b,h] = tril(q k^T, -1) v[b, h or 0] — no softmax, no scale, diagonal excluded."""
    q = np.asarray(q, dtype=acc)
    k = np.asarray(k, dtype=acc)
    v = np.asarray(v, dtype=acc)
    s = q @ np.swapaxes(k, -1, -2)
    s = np.tril(s, -1)
    return s @ v  # broadcasts v over heads when it has one head


def tril_decode(q: np.ndarray, k_past: np.ndarray, v_past: np.ndarray, acc=np.float64) -> np.ndarray:
    """out = (q k_past^T) v_past — every cached key precedes the query; S == 0 gives zeros."""
    q = np.asarray(q, dtype=acc)
    k_past = np.asarray(k_past, dtype=acc)
    v_past = np.asarray(v_past, dtype=acc)
    B, H, Tq, _ = q.shape
    D = v_past.shape[-1]
    if k_past.shape[2] == 0:
        return np.zeros((B, H, Tq, D), dtype=acc)
    return (q @ np.swapaxes(k_past, -1, -2)) @ v_past


# ------------------------------------------------------------------ fp8 key cache
def e4m3_rne(y: np.ndarray) -> np.ndarray:
    """float32 values rounded to the nearest finite e4m3 value (1 sign, 4 exponent bits with
    bias 7, 3 mantissa bits; smallest normal 2^-6, subnormal step 2^-9, largest 448), ties to
    even, saturating at +-448. Returns the rounded values as float32."""
    y = np.asarray(y, dtype=np.float32).astype(np.float64)
    a = np.abs(y)
    _, ex = np.frexp(np.maximum(a, 2.0 ** -6))  # a = m 2^ex, m in [0.5, 1): binade 2^(ex-1)
    quantum = np.ldexp(1.0, ex - 1 - 3)         # 3 mantissa bits (the subnormal step below 2^-6)
    r = np.round(a / quantum) * quantum          # exact division by a power of two; half to even
    r = np.minimum(r, 448.0)
    return np.copysign(r, y).astype(np.float32)


def quantize_rows_fp8(x: np.ndarray):
    """Row-scaled e4m3 of the last axis: amax = max |x|, inv = 448 / amax (0 for an all-zero
    row), q = e4m3(x * inv) (products in float32), scale = amax / 448 (float32).
    Returns (q as float32 e4m3 values, scale) with x ~= q * scale[..., None]."""
    x = np.asarray(x, dtype=np.float32)
    amax = np.max(np.abs(x), axis=-1)
    with np.errstate(divide="ignore"):
        inv = np.where(amax > 0, np.float32(448.0) / amax, np.float32(0.0)).astype(np.float32)
    q = e4m3_rne((x * inv[..., None]).astype(np.float32))
    scale = (amax / np.float32(448.0)).astype(np.float32)
    return q, scale


def tril_decode_fp8(q: np.ndarray, k8: np.ndarray, k_scale: np.ndarray, v_past: np.ndarray,
                    acc=np.float64) -> np.ndarray:
    """``tril_decode`` against the dequantized fp8 key history k8 * k_scale."""
    k = np.asarray(k8, dtype=acc) * np.asarray(k_scale, dtype=acc)[..., None]
    return tril_decode(q, k, v_past, acc=acc)


def state_from_history(k_past: np.ndarray, v_past: np.ndarray, acc=np.float64) -> np.ndarray:
    """N x D recurrent state of a key/value history: S[b,h] = sum_j k_j^T v_j (v heads 1 or H)."""
    k = np.asarray(k_past, dtype=acc)
    v = np.asarray(v_past, dtype=acc)
    if v.shape[1] == 1 and k.shape[1] != 1:
        v = np.broadcast_to(v, (v.shape[0], k.shape[1]) + v.shape[2:])
    return np.swapaxes(k, -1, -2) @ v


def state_decode(q_rot: np.ndarray, state: np.ndarray, v_new: np.ndarray, acc=np.float64):
    """One step of the state form of tril_decode: out = q . S (the past only), then
    S_new = S + q^T v_new. q_rot (B,H,1,N), state (B,H,N,D), v_new (B,Hv,1,D)."""
    q = np.asarray(q_rot, dtype=acc)
    S = np.asarray(state, dtype=acc)
    v = np.asarray(v_new, dtype=acc)
    if v.shape[1] == 1 and q.shape[1] != 1:
        v = np.broadcast_to(v, (v.shape[0], q.shape[1]) + v.shape[2:])
    out = q @ S
    return out, S + np.swapaxes(q, -1, -2) @ v


def tril_backward(q, k, v, dout, acc=np.float64, k_is_q: bool = False):
    """Analytic gradients of O = tril(q k^T, -1) v (kernels/attention_bwd.py:45-83).

    Returns (dq, dk, dv) with dv summed over heads when v has one head; with k_is_q the
    first result is dq + dk (StrictTrilSelfAttnFn, kernels/attention_bwd.py:284-291).
    """
    q = np.asarray(q, dtype=acc)
    k = np.asarray(k, dtype=acc)
    v = np.asarray(v, dtype=acc)
    dout = np.asarray(dout, dtype=acc)
    H = q.shape[1]
    vh = np.broadcast_to(v, (v.shape[0], H) + v.shape[2:]) if v.shape[1] == 1 else v
    m = np.tril(q @ np.swapaxes(k, -1, -2), -1)
    ds = np.tril(dout @ np.swapaxes(vh, -1, -2), -1)
    dq = ds @ k
    dk = np.swapaxes(ds, -1, -2) @ q
    dvh = np.swapaxes(m, -1, -2) @ dout
    dv = dvh.sum(axis=1, keepdims=True) if v.shape[1] == 1 and H != 1 else dvh
    if k_is_q:
        return dq + dk, None, dv
    return dq, dk, dv


# ---------------------------------------------------------------------------- model
def layer_norm(x: np.ndarray, eps: float = 1e-5, acc=np.float64) -> np.ndarray:
    x = np.asarray(x, dtype=acc)
    mu = x.mean(-1, keepdims=True)
    var = ((x - mu) ** 2).mean(-1, keepdims=True)
    return (x - mu) / np.sqrt(var + eps)


def bdh_forward(idx: np.ndarray, weights: dict, n_layer: int, n_head: int, acc=np.float64):
    """Logits of the baseline BDH forward in eval mode (bdh_baseline.py:96-139).

    weights: embed (V,D), encoder (nh,D,N), encoder_v (nh,D,N), decoder (nh*N,D),
    lm_head (D,V), freqs (N,).
    """
    emb = np.asarray(weights["embed"], dtype=acc)
    enc = np.asarray(weights["encoder"], dtype=acc)
    enc_v = np.asarray(weights["encoder_v"], dtype=acc)
    dec = np.asarray(weights["decoder"], dtype=acc)
    head = np.asarray(weights["lm_head"], dtype=acc)
    freqs = np.asarray(weights["freqs"], dtype=np.float32)
    B, T = idx.shape
    D = emb.shape[1]
    nh = n_head
    N = enc.shape[-1]
    x = layer_norm(emb[idx])[:, None]  # B,1,T,D
    for _ in range(n_layer):
        xs = np.maximum(x @ enc, 0.0)  # B,nh,T,N
        qr = rope(xs.astype(np.float32), freqs).astype(acc)
        y = tril_score_v(qr, qr, x, acc=acc)
        y = layer_norm(y)
        ys = np.maximum(y @ enc_v, 0.0)
        xy = xs * ys
        ymlp = np.swapaxes(xy, 1, 2).reshape(B, 1, T, N * nh) @ dec
        x = layer_norm(x + layer_norm(ymlp))
    return x.reshape(B, T, D) @ head


def bdh_layer_bf16(x: np.ndarray, weights: dict, n_head: int, rounding: bool = True,
                   round_scores: bool = True):
    """One BDH layer under bf16 autocast with fp32 accumulation (bdh.py:991-1052 as
    torch.autocast(bfloat16) runs it on a GPU): returns (x_out, attention output).

    Every GEMM takes bf16 operands, accumulates exactly and rounds its output to bf16; LayerNorm
    runs in fp32 on its (bf16 or fp32) input (CUDA autocast's fp32 policy for layer_norm; the
    CPU autocast leaves it in bf16, bdh.py:731-750 then keeps a bf16 residual stream); the RoPE
    rotates bf16 values with fp32 cos/sin as kernels/rope.py:108-126; the sparse product is
    rounded to bf16. round_scores: the T x T scores are rounded to bf16 before their product
    with V, as the reference's default eager attention returns them under autocast
    (kernels/attention.py:27-40); False keeps them exact (its native tril_score_v,
    csrc/tril_attn_cuda.cu, accumulates them in fp32). rounding=False removes every bf16
    rounding. x: (B, T, D) float32 residual stream entering the layer.
    """
    r = bf16_round if rounding else (lambda a: np.asarray(a, np.float32))
    enc = r(np.asarray(weights["encoder"], np.float32)).astype(np.float64)
    enc_v = r(np.asarray(weights["encoder_v"], np.float32)).astype(np.float64)
    dec = r(np.asarray(weights["decoder"], np.float32)).astype(np.float64)
    freqs = np.asarray(weights["freqs"], dtype=np.float32)
    B, T, _ = x.shape
    nh = n_head
    N = enc.shape[-1]

    def gemm(a, w, eq):
        return r(np.einsum(eq, r(a).astype(np.float64), w, optimize=True).astype(np.float32))

    x = np.asarray(x, np.float32)
    xs = np.maximum(gemm(x, enc, "btd,hdn->bthn"), np.float32(0.0))  # B,T,nh,N
    qr = rope(np.swapaxes(xs, 1, 2), freqs, bf16=rounding).astype(np.float64)  # B,nh,T,N
    s = np.einsum("bhtn,bhsn->bhts", qr, qr, optimize=True).astype(np.float32)
    if round_scores:
        s = r(s)
    s = np.tril(s, -1).astype(np.float64)
    v = r(x)[:, None].astype(np.float64)
    y = r(np.einsum("bhts,bxsd->bhtd", s, v, optimize=True).astype(np.float32))
    yn = layer_norm(y).astype(np.float32)
    ys = np.maximum(gemm(yn, enc_v, "bhtd,hdn->bthn"), np.float32(0.0))
    xy = r(xs * ys)
    ymlp = gemm(xy.reshape(B, T, nh * N), dec, "btk,kd->btd")
    return layer_norm(x + layer_norm(ymlp).astype(np.float32)).astype(np.float32), y


def bdh_forward_bf16(idx: np.ndarray, weights: dict, n_layer: int, n_head: int,
                     rounding: bool = True, round_scores: bool = True):
    """Logits of the BDH forward under bf16 autocast with fp32 accumulation everywhere
    (bdh.py:947-1072): the embedding's LayerNorm in fp32, ``bdh_layer_bf16`` per layer, then
    the bf16 lm_head GEMM. Arguments as ``bdh_layer_bf16``."""
    r = bf16_round if rounding else (lambda a: np.asarray(a, np.float32))
    emb = np.asarray(weights["embed"], np.float32)
    head = r(np.asarray(weights["lm_head"], np.float32)).astype(np.float64)
    x = layer_norm(emb[idx]).astype(np.float32)  # B,T,D fp32
    for _ in range(n_layer):
        x, _ = bdh_layer_bf16(x, weights, n_head, rounding, round_scores)
    return r(np.einsum("btd,dv->btv", r(x).astype(np.float64), head, optimize=True).astype(np.float32))


def latent_encode(x: np.ndarray, enc: np.ndarray, freqs: np.ndarray, pos0: int = 0,
                  bf16: bool = True, acc=np.float64):
    """Encoder projection + ReLU, then the RoPE of the attention input.

    xs[b,t,h,n] = relu(x[b,t,:] . enc[h,:,n])   (BDH._encoder_relu, bdh.py:861-889)
    qr[b,h,t,n] = rope(xs[b,:,h,:])[t,n]          (Attention.rope, bdh.py:396-412)
    bf16: the projection output is rounded to bf16 before the ReLU (a bf16 GEMM with fp32
    accumulation, as under autocast) and the rotation rounds as kernels/rope.py:108-126 does
    for bf16 values. Returns (xs (B,T,H,N), qr (B,H,T,N)) as float32.
    """
    lat = np.einsum("btd,hdn->bthn", np.asarray(x, acc), np.asarray(enc, acc))
    lat = lat.astype(np.float32)
    if bf16:
        lat = bf16_round(lat)
    xs = np.maximum(lat, np.float32(0.0))
    qr = rope(np.swapaxes(xs, 1, 2), freqs, pos0, bf16=bf16)
    return xs, qr


def latent_gate(y: np.ndarray, encv: np.ndarray, xs: np.ndarray, bf16: bool = True,
                acc=np.float64) -> np.ndarray:
    """xy[b,t,h,n] = xs[b,t,h,n] * relu(y[b,h,t,:] . encv[h,:,n])  (BDH._encoder_v_relu and the
    product of _mlp_merge, bdh.py:914-945); bf16 rounds the projection and the product."""
    lat = np.einsum("bhtd,hdn->bthn", np.asarray(y, acc), np.asarray(encv, acc)).astype(np.float32)
    if bf16:
        lat = bf16_round(lat)
    ys = np.maximum(lat, np.float32(0.0))
    xy = np.asarray(xs, np.float32) * ys
    return bf16_round(xy) if bf16 else xy


def rel_fro(a, b) -> float:
    """Relative Frobenius error ||a - b|| / ||b|| in float64."""
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    nb = np.linalg.norm(b)
    if nb == 0.0:
        return float(np.linalg.norm(a))
    return float(np.linalg.norm(a - b) / nb)
