"""GPU parity of the sm_100a kernels (called through the C-ABI library via kernels.sm100_attn)
against the reference's own outputs (tests/golden) and the pinned numpy oracle.

Tolerances (relative Frobenius, from the task's north star): fp32 path <= 1e-5; bf16 inputs
with fp32 accumulation <= 3e-3. RoPE is checked element-wise (it is bit-exact arithmetic up to
the cos/sin implementations).
"""

import numpy as np
import pytest
import torch

import tril_oracle as O
from conftest import golden

pytestmark = pytest.mark.gpu

DEV = "cuda"
TOL = {torch.float32: 1e-5, torch.bfloat16: 3e-3}


def sa():
    from kernels import sm100_attn

    return sm100_attn


def rel(a, b):
    return O.rel_fro(np.asarray(a, dtype=np.float64), np.asarray(b, dtype=np.float64))


def t(x, dtype=torch.float32):
    return torch.as_tensor(np.asarray(x)).to(device=DEV, dtype=dtype)


def np64(x):
    return x.detach().double().cpu().numpy()


@pytest.fixture(autouse=True)
def _device_error_clean():
    yield
    assert sa().device_error() == 0, "a kernel reported a pipeline timeout"


# --------------------------------------------------------------------------- RoPE
@pytest.mark.parametrize("pos0", [0, 37, 4000])
def test_rope_fp32_golden(pos0):
    g = golden("rope")
    y = sa().rope_rotate(t(g["x"]), t(g["freqs_64"]), pos0)
    np.testing.assert_allclose(y.cpu().numpy(), g[f"y_f32_pos{pos0}"], rtol=0, atol=2e-6)


@pytest.mark.parametrize("pos0", [0, 37, 4000])
def test_rope_bf16_golden(pos0):
    g = golden("rope")
    y = sa().rope_rotate(t(g["x"], torch.bfloat16), t(g["freqs_64"]), pos0).float().cpu().numpy()
    ref = g[f"y_bf16_pos{pos0}"]
    assert np.mean(y != ref) < 2e-3
    np.testing.assert_allclose(y, ref, rtol=0, atol=2 ** -7 * np.abs(ref).max())


def test_rope_permuted_view_into_strided_slot_of_other_dtype():
    N = 256
    f = torch.tensor(O.get_freqs(N), device=DEV)
    x = torch.relu(torch.randn(2, 9, 3, N, device=DEV)).permute(0, 2, 1, 3)  # (B,H,T,N) view
    buf = torch.zeros(2, 3, 20, N, device=DEV, dtype=torch.bfloat16)        # capacity 20
    slot = buf.narrow(2, 5, 9)
    sa().rope_rotate(x, f, 5, out=slot)
    ref = O.rope(x.cpu().numpy(), O.get_freqs(N), 5)
    np.testing.assert_allclose(slot.float().cpu().numpy(), O.bf16_round(ref), rtol=0, atol=2e-2)
    assert torch.all(buf[:, :, :5] == 0) and torch.all(buf[:, :, 14:] == 0)


def test_rope_bf16_bit_pattern_large_batch():
    N, T = 8192, 64
    f = O.get_freqs(N)
    x = torch.relu(torch.randn(4, 4, T, N, device=DEV)).to(torch.bfloat16)
    y = sa().rope_rotate(x, torch.tensor(f, device=DEV), 100).float().cpu().numpy()
    ref = O.rope(x.float().cpu().numpy(), f, 100, bf16=True)
    assert np.mean(y != ref) < 1e-3  # rare one-ulp cos/sin differences flip a bf16 rounding
    assert rel(y, ref) < 1e-3


# ------------------------------------------------------------------------ forward
@pytest.mark.parametrize("name", ["shared_v", "per_head_v", "t1", "t2", "distinct_k", "bf16", "tiled"])
def test_forward_golden(name):
    g = golden("fwd")
    dt = torch.bfloat16 if name == "bf16" else torch.float32
    q = t(g[f"{name}_q"], dt)
    k = t(g[f"{name}_k"], dt) if f"{name}_k" in g else q
    v = t(g[f"{name}_v"], dt)
    out = sa().tril_score_v(q, k, v)
    assert out.dtype == dt and out.shape == (q.size(0), q.size(1), q.size(2), v.size(-1))
    ext = g[f"{name}_out_ext"]
    exact = O.tril_score_v(np64(q), np64(k), np64(v))
    o = out.float().cpu().numpy()
    assert np.all(o[:, :, 0] == 0)
    if np.abs(exact).max() == 0:
        assert np.all(o == 0)
        return
    assert rel(o, exact) <= TOL[dt]
    assert rel(o, ext) <= TOL[dt] * (2 if dt == torch.bfloat16 else 1.5)


def test_baseline_attention_with_fused_rope():
    from kernels.attention_dispatch import bdh_rope_attn

    g = golden("fwd")
    out, qr = bdh_rope_attn(t(g["baseline_attn_q"]), t(g["baseline_attn_v"]),
                            t(g["baseline_attn_freqs"]), 0, impl="cuda_sm100")
    assert rel(out.cpu().numpy(), g["baseline_attn_out"]) < 1e-5


SHAPES = [  # B, H, Hv, T, N, D
    (1, 1, 1, 1, 16, 8),
    (1, 2, 1, 2, 16, 8),
    (2, 3, 1, 3, 64, 32),
    (1, 2, 2, 17, 72, 40),
    (1, 2, 1, 127, 64, 256),
    (1, 1, 1, 128, 128, 256),
    (2, 2, 1, 129, 200, 256),
    (1, 4, 4, 300, 512, 300),
    (1, 2, 1, 257, 8192, 256),
]


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("shape", SHAPES)
def test_forward_shapes_vs_oracle(shape, dt):
    B, H, Hv, T, N, D = shape
    gen = torch.Generator(device=DEV).manual_seed(hash(shape) % 1000)
    q = torch.relu(torch.randn(B, H, T, N, device=DEV, generator=gen)).to(dt)
    v = torch.randn(B, Hv, T, D, device=DEV, generator=gen).to(dt)
    out = sa().tril_score_v(q, q, v)
    ref = O.tril_score_v(np64(q), np64(q), np64(v))
    assert rel(out.float().cpu().numpy(), ref) <= TOL[dt]
    assert torch.all(out[:, :, 0] == 0)


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
def test_forward_distinct_k_and_permuted_views(dt):
    B, H, T, N, D = 2, 3, 200, 256, 64
    q = torch.relu(torch.randn(B, T, H, N, device=DEV)).to(dt).permute(0, 2, 1, 3)
    k = torch.relu(torch.randn(B, T, H, N, device=DEV)).to(dt).permute(0, 2, 1, 3)
    v = torch.randn(B, T, D, device=DEV).to(dt).unsqueeze(1)
    out = sa().tril_score_v(q, k, v)
    ref = O.tril_score_v(np64(q), np64(k), np64(v))
    assert rel(out.float().cpu().numpy(), ref) <= TOL[dt]


def test_forward_empty_and_zero_cases():
    q = torch.zeros(2, 3, 0, 64, device=DEV)
    v = torch.zeros(2, 1, 0, 32, device=DEV)
    assert sa().tril_score_v(q, q, v).shape == (2, 3, 0, 32)
    q = torch.randn(1, 2, 1, 64, device=DEV)
    v = torch.randn(1, 1, 1, 32, device=DEV)
    assert torch.all(sa().tril_score_v(q, q, v) == 0)


def test_forward_linear_in_v_full_size_bf16():
    """Config-1 shapes (B=4, nh=4, T=512, N=8192, D=256): linearity in V and row 0 == 0,
    plus agreement with a float64 torch reference on the device."""
    B, H, T, N, D = 4, 4, 512, 8192, 256
    q = torch.relu(torch.randn(B, H, T, N, device=DEV)).to(torch.bfloat16)
    v1 = torch.randn(B, 1, T, D, device=DEV).to(torch.bfloat16)
    v2 = torch.randn(B, 1, T, D, device=DEV).to(torch.bfloat16)
    o1 = sa().tril_score_v(q, q, v1).double()
    o2 = sa().tril_score_v(q, q, v2).double()
    o12 = sa().tril_score_v(q, q, (v1.float() + v2.float()).to(torch.bfloat16)).double()
    assert ((o12 - o1 - o2).norm() / o12.norm()).item() < 6e-3  # v1+v2 rounded to bf16
    assert torch.all(o1[:, :, 0] == 0)
    qd = q.double()
    ref = ((qd @ qd.mT).tril(-1)) @ v1.double()
    assert ((o1 - ref).norm() / ref.norm()).item() <= 3e-3


@pytest.mark.parametrize("B,N", [(32, 8192), (1, 2048)])
def test_forward_bf16_last_wave(B, N):
    """bf16 forward at config 2's attention (B = 32, 4 heads, T = 512, N = 8192: 384 pair tiles
    on 74 pairs, a partial last wave of 14) and a problem smaller than one wave (12 tiles): the
    last wave's units against float64 at the bf16 bar, strictly causal, the same bits on a second
    call. With BDH_SM100_SCORE_TAIL=1 the last wave runs as narrow tiles (the same bits)."""
    H, T, D = 4, 512, 256
    g = torch.Generator(device=DEV).manual_seed(17)
    q = torch.relu(torch.randn(B, H, T, N, device=DEV, generator=g)).to(torch.bfloat16)
    v = torch.randn(B, 1, T, D, device=DEV, generator=g).to(torch.bfloat16)
    out = sa().tril_score_v(q, q, v)
    again = sa().tril_score_v(q, q, v)
    torch.cuda.synchronize()
    assert torch.equal(out, again)
    assert torch.all(out[:, :, 0] == 0)
    # the last wave's tiles are the last ones of the tile list: the highest units
    for u in sorted({B * H - 1, B * H - 2, B * H - 5, 0}):
        b, h = divmod(u, H)
        qd = q[b, h].double()
        ref = (qd @ qd.T).tril(-1) @ v[b, 0].double()
        err = ((out[b, h].double() - ref).norm() / ref.norm()).item()
        assert err <= 3e-3, (u, err)


def test_forward_full_size_fp32_config1():
    B, H, T, N, D = 4, 4, 512, 8192, 256
    q = torch.relu(torch.randn(B, H, T, N, device=DEV))
    v = torch.randn(B, 1, T, D, device=DEV)
    out = sa().tril_score_v(q, q, v).double()
    qd = q.double()
    ref = ((qd @ qd.mT).tril(-1)) @ v.double()
    assert ((out - ref).norm() / ref.norm()).item() <= 1e-5


# ------------------------------------------------------------------------- decode
@pytest.mark.parametrize("S", [0, 1, 25])
def test_decode_golden_capacity_views(S):
    g = golden("decode")
    kbuf, vbuf = t(g["kbuf"]), t(g["vbuf"])
    out = sa().tril_decode(t(g["q"]), kbuf.narrow(2, 0, S), vbuf.narrow(2, 0, S))
    ref = g[f"out_ext_S{S}"]
    if S == 0:
        assert torch.all(out == 0) and out.shape == ref.shape
    else:
        assert rel(out.cpu().numpy(), ref) < 1e-6


def test_decode_multi_query_rows():
    g = golden("decode")
    out = sa().tril_decode(t(g["q_tq3"]), t(g["kbuf"])[:1].narrow(2, 0, 25), t(g["vbuf"])[:1].narrow(2, 0, 25))
    assert rel(out.cpu().numpy(), g["out_ext_tq3"]) < 1e-6


@pytest.mark.parametrize("qdt,kvdt", [(torch.float32, torch.float32), (torch.float32, torch.bfloat16),
                                      (torch.bfloat16, torch.bfloat16), (torch.bfloat16, torch.float32)])
def test_decode_storage_dtypes(qdt, kvdt):
    B, H, S, cap, N, D = 3, 4, 700, 1024, 8192, 256
    kbuf = torch.randn(B, H, cap, N, device=DEV).to(kvdt)
    vbuf = torch.randn(B, 1, cap, D, device=DEV).to(kvdt)
    q = torch.randn(B, H, 1, N, device=DEV).to(qdt)
    kp, vp = kbuf.narrow(2, 0, S), vbuf.narrow(2, 0, S)
    out = sa().tril_decode(q, kp, vp)
    assert out.dtype == qdt
    ref = (q.double() @ kp.double().mT) @ vp.double()
    assert ((out.double() - ref).norm() / ref.norm()).item() <= TOL[qdt] * (1 if qdt == torch.float32 else 1)


@pytest.mark.parametrize("qdt,kvdt,S", [(torch.float32, torch.float32, 700),
                                        (torch.float32, torch.bfloat16, 1023),
                                        (torch.bfloat16, torch.bfloat16, 129)])
def test_decode_exact_small_integers(qdt, kvdt, S):
    """Integer query and cache (scores <= 32, sums below 2^24): the decode step, with its split
    plan and fixed-order reduction, returns (q K^T) V exactly, rounded once to the query dtype."""
    B, H, N, D = 3, 4, 8, 64
    g = torch.Generator().manual_seed(S)
    q64 = torch.randint(0, 3, (B, H, 1, N), generator=g).double()
    k64 = torch.randint(0, 3, (B, H, S, N), generator=g).double()
    v64 = torch.randint(-2, 3, (B, 1, S, D), generator=g).double()
    out = sa().tril_decode(q64.to(qdt).to(DEV), k64.to(kvdt).to(DEV), v64.to(kvdt).to(DEV))
    assert torch.equal(out.cpu(), ((q64 @ k64.mT) @ v64).to(qdt))


def test_decode_equals_last_row_of_forward():
    B, H, T, N, D = 2, 4, 300, 1024, 256
    q = torch.relu(torch.randn(B, H, T, N, device=DEV))
    v = torch.randn(B, 1, T, D, device=DEV)
    full = sa().tril_score_v(q, q, v)
    last = sa().tril_decode(q[:, :, -1:], q[:, :, :-1], v[:, :, :-1])
    assert ((last - full[:, :, -1:]).norm() / full[:, :, -1:].norm()).item() < 1e-5


@pytest.mark.parametrize("kvdt", [torch.float32, torch.bfloat16])
def test_decode_fused_rope_writes_slot(kvdt):
    B, H, S, cap, N, D = 2, 4, 33, 40, 512, 64
    f = O.get_freqs(N)
    kbuf = torch.randn(B, H, cap, N, device=DEV).to(kvdt)
    vbuf = torch.randn(B, 1, cap, D, device=DEV).to(kvdt)
    q = torch.relu(torch.randn(B, H, 1, N, device=DEV))
    slot = kbuf.narrow(2, S, 1)
    out = sa().tril_decode(q, kbuf.narrow(2, 0, S), vbuf.narrow(2, 0, S),
                           freqs=torch.tensor(f, device=DEV), pos=S, kr_slot=slot)
    qr = O.rope(q.cpu().numpy(), f, S)
    np.testing.assert_allclose(slot.float().cpu().numpy(), qr if kvdt == torch.float32 else O.bf16_round(qr),
                               rtol=0, atol=2e-6 if kvdt == torch.float32 else 3e-2)
    ref = O.tril_decode(qr, np64(kbuf[:, :, :S]), np64(vbuf[:, :, :S]))
    assert rel(out.cpu().numpy(), ref) < 1e-5


@pytest.mark.parametrize("kvdt", [torch.float32, torch.bfloat16])
def test_decode_fused_rope_bf16_query(kvdt):
    """bf16 queries with fused RoPE (the bf16-autocast model's decode step): the rotation runs in
    a separate pass, the kernel reads fp32 rotated queries, the output stays bf16."""
    B, H, S, cap, N, D = 3, 4, 150, 160, 1024, 256
    f = O.get_freqs(N)
    kbuf = torch.randn(B, H, cap, N, device=DEV).to(kvdt)
    vbuf = torch.randn(B, 1, cap, D, device=DEV).to(kvdt)
    q = torch.relu(torch.randn(B, 1, H, N, device=DEV)).to(torch.bfloat16).permute(0, 2, 1, 3)
    slot = kbuf.narrow(2, S, 1)
    guard = kbuf.narrow(2, S + 1, cap - S - 1).clone()
    out = sa().tril_decode(q, kbuf.narrow(2, 0, S), vbuf.narrow(2, 0, S),
                           freqs=torch.tensor(f, device=DEV), pos=S, kr_slot=slot)
    assert out.dtype == torch.bfloat16 and out.shape == (B, H, 1, D)
    qr = O.rope(q.float().cpu().numpy(), f, S, bf16=True)
    np.testing.assert_allclose(slot.float().cpu().numpy(), qr if kvdt == torch.float32 else O.bf16_round(qr),
                               rtol=0, atol=2e-2)
    assert torch.equal(kbuf.narrow(2, S + 1, cap - S - 1), guard)
    ref = O.tril_decode(qr.astype(np.float64), np64(kbuf[:, :, :S]), np64(vbuf[:, :, :S]))
    assert rel(out.float().cpu().numpy(), ref) < 3e-3


@pytest.mark.parametrize("B,S", [(1, 700), (4, 1023), (64, 40)])
def test_decode_split_plans(B, S):
    """Batch sizes that pick different split plans (16..128 cached rows per CTA)."""
    H, N, D = 4, 2048, 256
    k = torch.randn(B, H, S, N, device=DEV)
    v = torch.randn(B, 1, S, D, device=DEV)
    q = torch.randn(B, H, 1, N, device=DEV)
    out = sa().tril_decode(q, k, v)
    ref = (q.double() @ k.double().mT) @ v.double()
    assert ((out.double() - ref).norm() / ref.norm()).item() < 1e-5


# ----------------------------------------------------------------------- backward
def test_backward_golden_fp32():
    g = golden("bwd")
    q, k, v, do = (t(g[n]) for n in ("Q", "K", "V", "dO"))
    dq, dk, dv = sa().tril_score_v_bwd(q, k, v, do)
    assert rel(dq.cpu().numpy(), g["dQ"]) < 1e-5
    assert rel(dk.cpu().numpy(), g["dK"]) < 1e-5
    assert rel(dv.cpu().numpy(), g["dV"]) < 1e-5
    dqt, none, dvs = sa().tril_score_v_bwd(q, q, v, do)
    assert none is None
    assert rel(dqt.cpu().numpy(), g["self_dQ"]) < 1e-5
    assert rel(dvs.cpu().numpy(), g["self_dV"]) < 1e-5


BWD_SHAPES = [  # B, H, Hv, T, N, D
    (1, 2, 1, 5, 16, 8),
    (1, 2, 2, 130, 64, 32),
    (2, 3, 1, 257, 256, 256),
    (1, 4, 1, 512, 1024, 256),
    # T on and just below the 128- and 256-row tile edges, latent and value widths that are not
    # multiples of the 64-element k-block (zero-filled tails), the value rows of D = 300 not
    # 16-byte aligned in bf16, and a long odd T: the strict past must hold at every tile edge
    # (tests/test_attn_bwd.py of the reference checks it at its default tile boundary)
    (1, 2, 1, 128, 72, 40),
    (2, 2, 2, 255, 136, 96),
    (1, 1, 1, 256, 200, 300),
    (1, 1, 1, 1537, 72, 40),
]


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("shape", BWD_SHAPES)
@pytest.mark.parametrize("self_form", [True, False])
def test_backward_vs_oracle(shape, dt, self_form):
    B, H, Hv, T, N, D = shape
    # seeded draws: the bf16 bar leaves little room on the smallest shape (40 outputs), so the
    # inputs are fixed instead of new on every run
    g = torch.Generator().manual_seed(1000 * T + N + D + (7 if self_form else 0))
    rnd = lambda *s: torch.randn(*s, generator=g).to(DEV)
    q = torch.relu(rnd(B, H, T, N)).to(dt)
    k = q if self_form else torch.relu(rnd(B, H, T, N)).to(dt)
    v = rnd(B, Hv, T, D).to(dt)
    do = rnd(B, H, T, D).to(dt)
    dq, dk, dv = sa().tril_score_v_bwd(q, k, v, do)
    rq, rk, rv = O.tril_backward(np64(q), np64(k), np64(v), np64(do), k_is_q=self_form)
    assert rel(dq.float().cpu().numpy(), rq) <= TOL[dt]
    assert rel(dv.float().cpu().numpy(), rv) <= TOL[dt]
    if not self_form:
        assert rel(dk.float().cpu().numpy(), rk) <= TOL[dt]


@pytest.mark.parametrize("dt,T,j0,N,D", [(torch.float32, 65, 63, 16, 8),
                                          (torch.float32, 129, 127, 16, 8),
                                          (torch.float32, 257, 128, 16, 8),
                                          (torch.bfloat16, 256, 255, 16, 8),
                                          (torch.bfloat16, 1537, 255, 128, 64),
                                          (torch.bfloat16, 1537, 256, 128, 64),
                                          (torch.bfloat16, 1600, 1535, 128, 64)])
def test_forward_strict_past_at_tile_edges(dt, T, j0, N, D):
    """V nonzero on one key row j0 only: every output row t <= j0 is exactly zero (no diagonal,
    no future), across the 128- and 256-row tile edges and, for bf16 at T >= 1536, the chunked
    form's 256-key chunk edges (intra-chunk scores and carried prefix state); the rest matches
    fp64 (Q K^T).tril(-1) V."""
    g = torch.Generator().manual_seed(4099 + T + j0)
    q64 = torch.randn(1, 2, T, N, generator=g, dtype=torch.float64)
    k64 = torch.randn(1, 2, T, N, generator=g, dtype=torch.float64)
    v64 = torch.zeros(1, 1, T, D, dtype=torch.float64)
    v64[:, :, j0, :] = torch.randn(1, 1, D, generator=g, dtype=torch.float64)
    q, k, v = (x.to(dt).to(DEV) for x in (q64, k64, v64))
    out = sa().tril_score_v(q, k, v)
    assert torch.count_nonzero(out[:, :, : j0 + 1, :]).item() == 0
    if j0 == T - 1:  # no row after the key: the whole output is zero
        return
    qr, kr, vr = (x.to(dt).double() for x in (q64, k64, v64))
    ref = (qr @ kr.mT).tril(-1) @ vr
    tol = 1e-5 if dt == torch.float32 else 3e-3
    assert ((out.double().cpu() - ref).norm() / ref.norm()).item() <= tol


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("T,queries", [(65, (63,)), (65, (64,)), (128, (127,)), (129, (128,)),
                                       (257, (255,)), (257, (256,)), (257, (127, 128, 255))])
def test_backward_strict_past_at_tile_edges(T, queries, dt):
    """Upstream gradient on a few rows only, next to the 64-, 128- and 256-row tile edges: dK and
    dV of every key at or after the last such row are exactly zero (strict past, no diagonal, no
    future), and all three gradients match fp64 autograd of (Q K^T).tril(-1) V (the reference's
    tests/test_attn_bwd_v4_contract.py:611-667 strict-past and multi-tile accumulation cases,
    with N = 3 and D = 4 padded by the wrapper)."""
    g = torch.Generator().manual_seed(2031 + T + sum(queries))
    q64 = torch.randn(1, 2, T, 3, generator=g, dtype=torch.float64)
    k64 = torch.randn(1, 2, T, 3, generator=g, dtype=torch.float64)
    v64 = torch.randn(1, 1, T, 4, generator=g, dtype=torch.float64)
    do64 = torch.zeros(1, 2, T, 4, dtype=torch.float64)
    for i in queries:
        do64[:, :, i, :] = torch.randn(1, 2, 4, generator=g, dtype=torch.float64)
    q, k, v, do = (x.to(dt).to(DEV) for x in (q64, k64, v64, do64))
    dq, dk, dv = sa().tril_score_v_bwd(q, k, v, do)
    last = max(queries)
    assert torch.count_nonzero(dk[:, :, last:, :]).item() == 0
    assert torch.count_nonzero(dv[:, :, last:, :]).item() == 0
    quiet = [i for i in range(T) if i not in queries]  # rows without upstream gradient
    assert torch.count_nonzero(dq[:, :, quiet, :]).item() == 0
    # the reference math on the operands as the kernel saw them (rounded to dt), in fp64
    qr, kr, vr = (x.to(dt).double().requires_grad_(True) for x in (q64, k64, v64))
    dod = do.double().cpu()
    ((qr @ kr.mT).tril(-1) @ vr).backward(dod)
    got = {"dq": dq, "dk": dk, "dv": dv}
    ref = {"dq": qr.grad, "dk": kr.grad, "dv": vr.grad}
    if dt == torch.float32:
        for n in got:
            assert ((got[n].double().cpu() - ref[n]).norm() / ref[n].norm()).item() <= 1e-5
        return
    # bf16: with one upstream row and N = 3 a handful of values carry the whole norm, so the
    # relative-Frobenius bar (held on full tensors by test_backward_vs_oracle) is replaced by an
    # elementwise bound: one bf16 rounding of every score the products read (P = Q K^T and
    # dS = dO V^T, both masked) and of every output, at 2^-8 (twice bf16's unit roundoff)
    qd, kd, vd = qr.detach(), kr.detach(), vr.detach()
    P = (qd @ kd.mT).tril(-1).abs()
    dS = (dod @ vd.mT).tril(-1).abs()
    eps = 2.0 ** -8
    bound = {"dq": eps * (dS @ kd.abs() + ref["dq"].abs()),
             "dk": eps * (dS.mT @ qd.abs() + ref["dk"].abs()),
             "dv": eps * ((P.mT @ dod.abs()).sum(dim=1, keepdim=True) + ref["dv"].abs())}
    for n in got:
        err = (got[n].double().cpu() - ref[n]).abs()
        assert torch.all(err <= bound[n]), (n, (err - bound[n]).max().item())


def test_raw_score_contract_exact_small_integers():
    """The reference's raw-score contract (tests/test_prefill_blocked.py:47-87): integer Q, K, V
    give an exactly representable tril(Q K^T, -1) V, so the fp32 path must return it bit for bit;
    the backward of out.sum() has no gradient on Q's first row and on K's and V's last rows, and
    is exact as well."""
    Q = torch.tensor([2.0, 3.0, 5.0, 7.0, 11.0], dtype=torch.float64).view(1, 1, 5, 1)
    K = torch.tensor([13.0, 17.0, 19.0, 23.0, 29.0], dtype=torch.float64).view(1, 1, 5, 1)
    V = torch.tensor([[[[1.0, -1.0], [2.0, -2.0], [4.0, -4.0], [8.0, -8.0], [16.0, -16.0]]]],
                     dtype=torch.float64)
    exact = (Q @ K.mT).tril(-1) @ V
    got = sa().tril_score_v(Q.float().to(DEV), K.float().to(DEV), V.float().to(DEV))
    assert torch.equal(got.double().cpu(), exact)
    v1 = V[..., :1]
    qd, kd, vd = (x.clone().requires_grad_(True) for x in (Q, K, v1))
    ((qd @ kd.mT).tril(-1) @ vd).sum().backward()
    dq, dk, dv = sa().tril_score_v_bwd(Q.float().to(DEV), K.float().to(DEV), v1.float().to(DEV),
                                       torch.ones(1, 1, 5, 1, device=DEV))
    assert torch.count_nonzero(dq[:, :, 0]).item() == 0
    assert torch.count_nonzero(dk[:, :, -1]).item() == 0 and torch.count_nonzero(dv[:, :, -1]).item() == 0
    for got_g, ref_g in ((dq, qd.grad), (dk, kd.grad), (dv, vd.grad)):
        assert torch.equal(got_g.double().cpu(), ref_g)


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
def test_exact_small_integers_across_tiles(dt):
    """Integer operands small enough that every score (<= 32) and dS is exact in bf16 and every
    sum exact in fp32: across the 128- and 256-row tile edges (T = 300) the forward and all three
    gradients equal the exact result, rounded once to the output dtype (bit for bit)."""
    B, H, T, N, D = 1, 2, 300, 8, 8
    g = torch.Generator().manual_seed(77)
    q64 = torch.randint(0, 3, (B, H, T, N), generator=g).double()
    k64 = torch.randint(0, 3, (B, H, T, N), generator=g).double()
    v64 = torch.randint(-2, 3, (B, 1, T, D), generator=g).double()
    do64 = torch.randint(-2, 3, (B, H, T, D), generator=g).double()
    q, k, v, do = (x.to(dt).to(DEV) for x in (q64, k64, v64, do64))
    out = sa().tril_score_v(q, k, v)
    exact = (q64 @ k64.mT).tril(-1) @ v64
    assert torch.equal(out.cpu(), exact.to(dt))
    qd, kd, vd = (x.clone().requires_grad_(True) for x in (q64, k64, v64))
    ((qd @ kd.mT).tril(-1) @ vd).backward(do64)
    dq, dk, dv = sa().tril_score_v_bwd(q, k, v, do)
    for got_g, ref_g in ((dq, qd.grad), (dk, kd.grad), (dv, vd.grad)):
        assert torch.equal(got_g.cpu(), ref_g.to(dt))


@pytest.mark.parametrize("value_heads", [1, 2])
@pytest.mark.parametrize("padding", ["feature", "sequence"])
def test_autograd_through_padded_storage(padding, value_heads):
    """The reference's padded-storage autograd contracts (tests/test_prefill_blocked.py:262-300
    and the capacity-padded sequence variant): Q and K are views of larger buffers (one spare
    latent column, or spare capacity rows, as a cache keeps them); the gradients land in the
    right elements of the buffers, none in the padding, and match fp64 eager attention."""
    import kernels

    T, B, H, N, D = 257, 2, 2, 5, 4
    g = torch.Generator().manual_seed(327 + value_heads)
    shape = (B, H, T, N + 1) if padding == "feature" else (B, H, T + 7, N)
    qs0 = torch.randn(*shape, dtype=torch.float64, generator=g)
    ks0 = torch.randn(*shape, dtype=torch.float64, generator=g)
    v0 = torch.randn(B, value_heads, T, D, dtype=torch.float64, generator=g)
    w = torch.randn(B, H, T, D, dtype=torch.float64, generator=g)

    def run(fn, dev, dt):
        qs = qs0.to(dev, dt).requires_grad_(True)
        ks = ks0.to(dev, dt).requires_grad_(True)
        v = v0.to(dev, dt).requires_grad_(True)
        q, k = ((x[..., :N] if padding == "feature" else x[:, :, :T]) for x in (qs, ks))
        assert not q.is_contiguous() and not k.is_contiguous()
        out = fn(q, k, v)
        grads = torch.autograd.grad((out * w.to(dev, dt)).sum(), (qs, ks, v))
        return out, grads

    ref, ref_g = run(lambda q, k, v: (q @ k.mT).tril(-1) @ v, "cpu", torch.float64)
    got, got_g = run(lambda q, k, v: kernels.bdh_attn(q, k, v, impl="cuda_sm100", use_autograd_fn=True),
                     DEV, torch.float32)
    assert ((got.double().cpu() - ref).norm() / ref.norm()).item() < 1e-5
    for a, b in zip(got_g, ref_g):
        assert ((a.double().cpu() - b).norm() / b.norm()).item() < 1e-5
    assert torch.count_nonzero(got[:, :, 0]).item() == 0
    for gs in got_g[:2]:
        pad = gs[..., N] if padding == "feature" else gs[:, :, T:]
        assert torch.count_nonzero(pad).item() == 0


@pytest.mark.parametrize("T", [1600, 4100])
def test_chunked_forward_exact_sparse_binary(T):
    """The chunked form (bf16, T >= 1536; 256-key chunks at T = 1600, 512 at 4100, ragged last
    chunks) on sparse binary latents (5% ones) and V in {-1, 0, 1}: every intra-chunk score and
    every prefix-state entry stays an integer below 256, exact in its bf16 storage, and every sum
    below 2^24, so the output equals tril(Q Q^T, -1) V rounded once to bf16."""
    B, H, N, D = 1, 2, 128, 64
    g = torch.Generator().manual_seed(T)
    q64 = (torch.rand(B, H, T, N, generator=g) < 0.05).double()
    v64 = torch.randint(-1, 2, (B, 1, T, D), generator=g).double()
    q = q64.to(torch.bfloat16).to(DEV)
    sa().profile_begin()
    out = sa().tril_score_v(q, q, v64.to(torch.bfloat16).to(DEV))
    torch.cuda.synchronize()
    assert sa().profile_end()["state"]["launches"] == 1  # the prefix-state pass ran: chunked form
    exact = (q64 @ q64.mT).tril(-1) @ v64
    states = torch.einsum("bhtn,bhtd->bhnd", q64, v64.abs().expand(B, H, T, D))
    assert states.max().item() < 256  # the largest possible prefix-state entry
    assert torch.equal(out.cpu(), exact.to(torch.bfloat16))


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
def test_backward_fused_rope_adjoint(dt):
    B, H, T, N, D, pos0 = 1, 2, 200, 512, 64, 7
    f = O.get_freqs(N)
    x = torch.relu(torch.randn(B, H, T, N, device=DEV)).to(dt)
    qr = sa().rope_rotate(x, torch.tensor(f, device=DEV), pos0)
    v = torch.randn(B, 1, T, D, device=DEV).to(dt)
    do = torch.randn(B, H, T, D, device=DEV).to(dt)
    dx, _, dv = sa().tril_score_v_bwd(qr, qr, v, do, freqs=torch.tensor(f, device=DEV), pos0=pos0)
    gq, _, gv = O.tril_backward(np64(qr), np64(qr), np64(v), np64(do), k_is_q=True)
    ref = O.rope_backward(gq, f, pos0)
    assert rel(dx.float().cpu().numpy(), ref) <= TOL[dt]
    assert rel(dv.float().cpu().numpy(), gv) <= TOL[dt]


def test_autograd_functions_native_match_eager(monkeypatch):
    import kernels

    monkeypatch.setenv("BDH_ATTN_AUTOGRAD", "1")
    B, H, T, N, D = 2, 4, 150, 256, 64
    q0 = torch.relu(torch.randn(B, H, T, N, device=DEV))
    v0 = torch.randn(B, 1, T, D, device=DEV)
    g = torch.randn(B, H, T, D, device=DEV)
    grads = {}
    for impl in ("eager", "cuda_sm100"):
        q = q0.clone().requires_grad_(True)
        v = v0.clone().requires_grad_(True)
        out = kernels.bdh_attn(q, q, v, impl=impl)
        out.backward(g)
        grads[impl] = (out.detach(), q.grad, v.grad)
    for a, b in zip(grads["eager"], grads["cuda_sm100"]):
        assert ((a.double() - b.double()).norm() / a.double().norm()).item() < 1e-5


def test_rope_attn_autograd_matches_eager():
    from kernels.attention_dispatch import bdh_rope_attn

    B, H, T, N, D = 1, 2, 96, 128, 32
    f = torch.tensor(O.get_freqs(N), device=DEV)
    x0 = torch.relu(torch.randn(B, H, T, N, device=DEV))
    v0 = torch.randn(B, 1, T, D, device=DEV)
    g = torch.randn(B, H, T, D, device=DEV)
    res = {}
    for impl in ("eager", "cuda_sm100"):
        x = x0.clone().requires_grad_(True)
        v = v0.clone().requires_grad_(True)
        out, _ = bdh_rope_attn(x, v, f, 3, impl=impl, use_autograd_fn=False)
        out.backward(g)
        res[impl] = (out.detach(), x.grad, v.grad)
    for a, b in zip(res["eager"], res["cuda_sm100"]):
        assert ((a.double() - b.double()).norm() / a.double().norm()).item() < 1e-5


# -------------------------------------------------------------------------- model
def _golden_model(impl, monkeypatch):
    import bdh_model

    monkeypatch.setenv("BDH_ATTN_IMPL", impl)
    g = golden("model")
    cfg = bdh_model.BDHConfig(n_layer=2, n_embd=32, n_head=2, mlp_internal_dim_multiplier=4,
                              dropout=0.0, vocab_size=256)
    m = bdh_model.BDH(cfg)
    sd = {k[2:]: torch.tensor(g[k]) for k in g.files if k.startswith("w_")}
    m.load_state_dict(sd)
    return m.to(DEV).eval(), g


@pytest.mark.parametrize("impl", ["eager", "cuda_sm100"])
def test_model_logits_match_reference(impl, monkeypatch):
    m, g = _golden_model(impl, monkeypatch)
    idx = torch.tensor(g["idx"], device=DEV)
    with torch.no_grad():
        logits, _ = m(idx)
    assert rel(logits.cpu().numpy(), g["logits_baseline"]) < 1e-5


@pytest.mark.parametrize("impl", ["eager", "cuda_sm100"])
@pytest.mark.parametrize("storage", [None, torch.bfloat16])
def test_model_cached_decode_matches_reference(impl, storage, monkeypatch):
    from bdh_cache import CacheManager

    m, g = _golden_model(impl, monkeypatch)
    idx = torch.tensor(g["idx"], device=DEV)
    cache = CacheManager.from_config(m.config, batch_size=2, max_seq=24, device=DEV, storage_dtype=storage)
    ref = g["logits_cached_steps"]
    with torch.inference_mode():
        lg, _ = m(idx[:, :16], cache=cache)
        steps = [lg[:, -1].float().cpu().numpy()]
        for s in range(16, 24):
            lg, _ = m(idx[:, s:s + 1], cache=cache)
            steps.append(lg[:, -1].float().cpu().numpy())
    tol = 1e-5 if storage is None else 3e-3
    for a, b in zip(steps, ref):
        assert rel(a, b) < tol


# ------------------------------------------------------- fused ReLU / gated product
@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
def test_rope_relu_input_equals_rope_of_relu(dt):
    N = 1024
    f = torch.tensor(O.get_freqs(N), device=DEV)
    x = torch.randn(2, 33, 4, N, device=DEV).to(dt).permute(0, 2, 1, 3)  # pre-activation view
    a = sa().rope_rotate(x, f, 11, relu_input=True)
    b = sa().rope_rotate(torch.relu(x), f, 11)
    assert torch.equal(a, b)


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
def test_relu_mul_matches_torch_on_einsum_layouts(dt):
    B, T, H, N, D = 2, 40, 4, 512, 32
    x = torch.randn(B, T, H, N, device=DEV).to(dt)                       # contiguous (b,t,h,n)
    yk = torch.randn(B, H, T, D, device=DEV).to(dt)
    w = torch.randn(H, D, N, device=DEV).to(dt)
    y = torch.einsum("bhtd,hdn->bthn", yk, w)                            # strided view
    out = sa().relu_mul(x, y)
    ref = torch.relu(x) * torch.relu(y)
    assert out.is_contiguous() and torch.equal(out, ref)


# ------------------------------------------------------------- chunked long-T forward
@pytest.fixture
def chunked_algo():
    prev = sa().set_forward_algo("chunked")
    yield
    sa().set_forward_algo(prev)


@pytest.mark.parametrize("T", [257, 300, 512, 768, 1000])
@pytest.mark.parametrize("Hv", [1, 2])
def test_chunked_forward_vs_oracle(T, Hv, chunked_algo):
    B, H, N, D = 1, 2, 512, 256
    q = torch.relu(torch.randn(B, H, T, N, device=DEV)).to(torch.bfloat16)
    v = torch.randn(B, Hv, T, D, device=DEV).to(torch.bfloat16)
    out = sa().tril_score_v(q, q, v)
    ref = O.tril_score_v(np64(q), np64(q), np64(v))
    assert rel(out.float().cpu().numpy(), ref) <= 3e-3
    assert torch.all(out[:, :, 0] == 0)


def test_chunked_forward_distinct_k_permuted(chunked_algo):
    B, H, T, N, D = 2, 2, 600, 256, 128
    q = torch.relu(torch.randn(B, T, H, N, device=DEV)).to(torch.bfloat16).permute(0, 2, 1, 3)
    k = torch.relu(torch.randn(B, T, H, N, device=DEV)).to(torch.bfloat16).permute(0, 2, 1, 3)
    v = torch.randn(B, T, D, device=DEV).to(torch.bfloat16).unsqueeze(1)
    out = sa().tril_score_v(q, k, v)
    ref = O.tril_score_v(np64(q), np64(k), np64(v))
    assert rel(out.float().cpu().numpy(), ref) <= 3e-3


@pytest.mark.parametrize("T,Hv", [(4096, 1), (4100, 2), (5000, 1)])
def test_chunked_forward_c512_vs_oracle(T, Hv):
    """From T = 4096 the chunked form uses 512-key chunks (256-row pair tiles covering half a
    chunk each, 8-k-block accumulation rounds in the state pass); ragged last chunks included."""
    B, H, N, D = 1, 2, 512, 256
    g = torch.Generator(device=DEV).manual_seed(T)
    q = torch.relu(torch.randn(B, H, T, N, device=DEV, generator=g)).to(torch.bfloat16)
    v = torch.randn(B, Hv, T, D, device=DEV, generator=g).to(torch.bfloat16)
    out = sa().tril_score_v(q, q, v)
    ref = O.tril_score_v(np64(q), np64(q), np64(v))
    assert rel(out.float().cpu().numpy(), ref) <= 3e-3
    assert torch.all(out[:, :, 0] == 0)


def test_chunked_forward_config3_shape_vs_fp64():
    """Config-3 shapes for two (b, h) units: T = 8192, N = 8192, ~5% dense latents,
    LayerNormed V; the automatic selection takes the chunked form at this length."""
    B, H, T, N, D = 1, 2, 8192, 8192, 256
    g = torch.Generator(device=DEV).manual_seed(3)
    q = torch.relu(torch.randn(B, H, T, N, device=DEV, generator=g) - 1.645).to(torch.bfloat16)
    v = torch.nn.functional.layer_norm(torch.randn(B, 1, T, D, device=DEV, generator=g), (D,)).to(torch.bfloat16)
    out = sa().tril_score_v(q, q, v).double()
    for h in range(H):
        qd = q[0, h].double()
        ref = (qd @ qd.T).tril(-1) @ v[0, 0].double()
        assert ((out[0, h] - ref).norm() / ref.norm()).item() <= 3e-3


# --------------------------------------------------------------- recurrent-state decode
@pytest.mark.parametrize("qdt,vdt", [(torch.float32, torch.float32), (torch.bfloat16, torch.bfloat16),
                                     (torch.float32, torch.bfloat16)])
def test_state_decode_equals_history_decode(qdt, vdt):
    """One state step equals the history decode (same past, same rotated query), updates the
    state by q^T v, and leaves the rows of zero rotated query untouched."""
    B, H, S, N, D = 3, 4, 300, 1024, 256
    f = torch.tensor(O.get_freqs(N), device=DEV)
    k = torch.relu(torch.randn(B, H, S, N, device=DEV))
    v = torch.randn(B, 1, S, D, device=DEV)
    state = (k.double().transpose(-1, -2) @ v.double().expand(-1, H, -1, -1)).float()
    x = torch.randn(B, H, 1, N, device=DEV)
    x[..., 0:N // 2:2] = -1.0            # pairs where both entries are negative: relu -> 0
    x[..., 1:N // 2:2] = -1.0
    q = x.to(qdt)
    v_new = torch.randn(B, 1, 1, D, device=DEV).to(vdt)
    s0 = state.clone()
    out = sa().state_decode(q, state, v_new, f, S, relu_input=True)
    assert out.dtype == qdt and out.shape == (B, H, 1, D)
    qr = sa().rope_rotate(torch.relu(q), f, S).float()
    ref = sa().tril_decode(qr, k.to(torch.float32), v)
    tol = 1e-5 if qdt == torch.float32 else 3e-3
    assert ((out.double() - ref.double()).norm() / ref.double().norm()).item() < tol
    upd = s0.double() + qr.double().transpose(-1, -2) @ v_new.double().expand(-1, H, -1, -1)
    assert ((state.double() - upd).norm() / upd.norm()).item() < 1e-6
    zero_rows = (qr[:, :, 0, :] == 0)
    assert bool(zero_rows[:, :, : N // 2].all())
    assert torch.equal(state[zero_rows], s0[zero_rows])


@pytest.mark.parametrize("storage,bar", [(None, 1e-5), (torch.bfloat16, 3e-3),
                                         (torch.float8_e4m3fn, 3e-2)])
def test_model_multi_token_blocks_after_a_past(storage, bar):
    """Prefill, then blocks of 4 and 16 tokens (the block's tril pass plus the decode kernel over
    the cached past, read in its storage dtype), a block of 20 (past || block through the cold
    path, as the reference does) and single tokens: the logits of every position match one full
    forward of the whole sequence, for fp32, bf16 and fp8-key caches."""
    import bdh_model
    from bdh_cache import CacheManager

    cfg = bdh_model.BDHConfig(n_layer=2, n_embd=128, n_head=4, mlp_internal_dim_multiplier=16,
                              vocab_size=256, dropout=0.0)
    torch.manual_seed(31)
    m = bdh_model.BDH(cfg).to(DEV).eval()
    m.attn._attn_impl_override = "cuda_sm100"
    B, blocks = 2, [40, 4, 16, 20, 1, 1]
    total = sum(blocks)
    idx = torch.randint(0, 256, (B, total), generator=torch.Generator().manual_seed(32)).to(DEV)
    cache = CacheManager.from_config(m.config, B, total, DEV, storage_dtype=storage)
    parts, t = [], 0
    with torch.no_grad():
        full, _ = m(idx)
        for n in blocks:
            parts.append(m(idx[:, t:t + n], cache=cache)[0])
            t += n
    assert cache.seq_len == total
    got = torch.cat(parts, 1)
    r = ((got.double() - full.double()).norm() / full.double().norm()).item()
    assert r < bar, r  # fp8: the e4m3 keys of the past (the fp8 cache's own bar)


@pytest.mark.parametrize("kw", [{}, {"top_k": 8, "temperature": 0.8},
                                {"cache_dtype": torch.float16}, {"cache_page_size": 4},
                                {"cache_kind": "state"}])
def test_generate_native_matches_eager_tokens(kw, monkeypatch):
    """BDH.generate on the native path (prefill kernels, decode kernel with the fused RoPE and
    cache-slot write, or the state decode) against the eager path on the same GPU: one seed,
    the same sampled tokens (the sampler draws identically; the logits agree to ~1e-6)."""
    import bdh_model

    cfg = bdh_model.BDHConfig(n_layer=2, n_embd=128, n_head=4, mlp_internal_dim_multiplier=16,
                              vocab_size=256, dropout=0.0)
    torch.manual_seed(51)
    m = bdh_model.BDH(cfg).to(DEV).eval()
    prompt = torch.randint(0, 256, (3, 20), generator=torch.Generator().manual_seed(52)).to(DEV)
    toks = {}
    for impl in ("eager", "cuda_sm100"):
        monkeypatch.setenv("BDH_ATTN_IMPL", impl)
        torch.manual_seed(53)
        toks[impl] = m.generate(prompt, 12, **kw)
    assert torch.equal(toks["eager"], toks["cuda_sm100"])
    assert torch.equal(toks["eager"][:, :20], prompt)


@pytest.mark.parametrize("amp", [False, True])
def test_model_state_cache_matches_history(amp):
    """Prefill + decode on the sm100 path with the N x D state cache vs the history cache."""
    import bdh_model
    from bdh_cache import CacheManager

    cfg = bdh_model.BDHConfig(n_layer=2, n_embd=256, n_head=4, mlp_internal_dim_multiplier=32,
                              vocab_size=256, dropout=0.0)
    torch.manual_seed(11)
    m = bdh_model.BDH(cfg).to(DEV).eval()
    m.attn._attn_impl_override = "cuda_sm100"
    B, P, steps = 3, 96, 6
    idx = torch.randint(0, 256, (B, P + steps), generator=torch.Generator().manual_seed(12)).to(DEV)
    res = {}
    for kind in ("kv", "state"):
        cache = CacheManager.from_config(m.config, B, P + steps, DEV, storage_kind=kind)
        ctx = torch.autocast("cuda", dtype=torch.bfloat16) if amp else torch.autocast("cuda", enabled=False)
        out = []
        with torch.no_grad(), ctx:
            lg, _ = m(idx[:, :P], cache=cache)
            out.append(lg[:, -1].float())
            for t in range(P, P + steps):
                lg, _ = m(idx[:, t:t + 1], cache=cache)
                out.append(lg[:, -1].float())
        res[kind] = torch.stack(out)
    r = ((res["state"] - res["kv"]).norm() / res["kv"].norm()).item()
    assert r < (1e-2 if amp else 1e-5), r
