"""bdh_sm100_ext on the GPU: the reference module's entry points and the new ops give the same
bits as the ctypes binding of the same library (kernels.sm100_attn) on the same inputs, the
reference extension's golden outputs (tests/golden) within the parity bars, capacity-strided
cache views in place, the RoPE forms equal to RoPE then the op, and capture in a CUDA graph."""

import numpy as np
import pytest
import torch

import tril_oracle as O
from conftest import golden

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(scope="module")
def ext():
    from kernels import sm100_ext

    return sm100_ext.load_ext()


def sa():
    from kernels import sm100_attn

    return sm100_attn


def t(a, dt=torch.float32):
    return torch.from_numpy(np.asarray(a)).to(DEV).to(dt)


def rel(a, b):
    return O.rel_fro(np.asarray(a, np.float64), np.asarray(b, np.float64))


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("shape", [(1, 2, 1, 17, 72, 40), (2, 4, 1, 300, 512, 256),
                                   (1, 2, 2, 257, 8192, 256)])
def test_tril_score_v_same_bits_as_ctypes(ext, shape, dt):
    B, H, Hv, T, N, D = shape
    g = torch.Generator(device=DEV).manual_seed(T)
    q = torch.relu(torch.randn(B, H, T, N, device=DEV, generator=g)).to(dt)
    k = torch.relu(torch.randn(B, H, T, N, device=DEV, generator=g)).to(dt)
    v = torch.randn(B, Hv, T, D, device=DEV, generator=g).to(dt)
    for kk in (q, k):
        a = ext.tril_score_v(q, kk, v)
        b = sa().tril_score_v(q, kk, v)
        assert a.dtype == dt and a.shape == (B, H, T, D)
        assert torch.equal(a, b)


@pytest.mark.parametrize("name", ["shared_v", "per_head_v", "t1", "t2", "distinct_k", "bf16"])
def test_tril_score_v_golden(ext, name):
    g = golden("fwd")
    dt = torch.bfloat16 if name == "bf16" else torch.float32
    q = t(g[f"{name}_q"], dt)
    k = t(g[f"{name}_k"], dt) if f"{name}_k" in g else q
    v = t(g[f"{name}_v"], dt)
    out = ext.tril_score_v(q, k, v).float().cpu().numpy()
    assert np.all(out[:, :, 0] == 0)
    ref = g[f"{name}_out_ext"]
    if np.abs(ref).max() == 0:
        assert np.all(out == 0)
        return
    assert rel(out, ref) <= (6e-3 if dt == torch.bfloat16 else 1.5e-5)


@pytest.mark.parametrize("S", [0, 1, 25])
def test_tril_decode_golden_capacity_views(ext, S):
    g = golden("decode")
    kbuf, vbuf = t(g["kbuf"]), t(g["vbuf"])
    out = ext.tril_decode(t(g["q"]), kbuf.narrow(2, 0, S), vbuf.narrow(2, 0, S))
    if S == 0:
        assert torch.all(out == 0) and tuple(out.shape) == g["out_ext_S0"].shape
    else:
        assert rel(out.cpu().numpy(), g[f"out_ext_S{S}"]) < 1e-6


@pytest.mark.parametrize("kvdt", [torch.float32, torch.bfloat16])
def test_rope_tril_decode_same_bits_as_ctypes(ext, kvdt):
    B, H, S, cap, N, D = 2, 4, 300, 512, 8192, 256
    g = torch.Generator(device=DEV).manual_seed(7)
    kbuf = torch.randn(B, H, cap, N, device=DEV, generator=g).to(kvdt)
    vbuf = torch.randn(B, 1, cap, D, device=DEV, generator=g).to(kvdt)
    q = torch.relu(torch.randn(B, H, 1, N, device=DEV, generator=g))
    freqs = torch.tensor(O.get_freqs(N), device=DEV)
    kb2 = kbuf.clone()
    a = ext.rope_tril_decode(q, freqs, S, kbuf[:, :, :S], vbuf[:, :, :S], kbuf[:, :, S:S + 1])
    b = sa().tril_decode(q, kb2[:, :, :S], vbuf[:, :, :S], freqs=freqs, pos=S,
                         kr_slot=kb2[:, :, S:S + 1])
    assert torch.equal(a, b)
    assert torch.equal(kbuf, kb2)  # the same rotated rows written to the slot


def test_rope_tril_score_v_is_rope_then_forward(ext):
    B, H, T, N, D = 2, 4, 384, 2048, 256
    g = torch.Generator(device=DEV).manual_seed(11)
    x = torch.relu(torch.randn(B, H, T, N, device=DEV, generator=g)).bfloat16()
    v = torch.randn(B, 1, T, D, device=DEV, generator=g).bfloat16()
    freqs = torch.tensor(O.get_freqs(N), device=DEV)
    out, qr = ext.rope_tril_score_v(x, v, freqs, 5)
    qr2 = sa().rope_rotate(x, freqs, 5)
    assert torch.equal(qr, qr2)
    assert torch.equal(out, sa().tril_score_v(qr2, qr2, v))
    assert torch.equal(ext.rope_rotate(x, freqs, 5), qr2)
    slot = torch.empty_like(qr)
    out3, qr3 = ext.rope_tril_score_v(x, v, freqs, 5, slot)
    assert qr3.data_ptr() == slot.data_ptr() and torch.equal(slot, qr2) and torch.equal(out3, out)


@pytest.mark.parametrize("self_form", [True, False])
def test_backward_same_bits_as_ctypes(ext, self_form):
    B, H, T, N, D = 1, 2, 257, 512, 64
    g = torch.Generator(device=DEV).manual_seed(3)
    q = torch.relu(torch.randn(B, H, T, N, device=DEV, generator=g)).bfloat16()
    k = q if self_form else torch.relu(torch.randn(B, H, T, N, device=DEV, generator=g)).bfloat16()
    v = torch.randn(B, 1, T, D, device=DEV, generator=g).bfloat16()
    do = torch.randn(B, H, T, D, device=DEV, generator=g).bfloat16()
    a = ext.tril_score_v_bwd(q, k, v, do)
    b = sa().tril_score_v_bwd(q, k, v, do)
    assert torch.equal(a[0], b[0]) and torch.equal(a[2], b[2])
    assert (a[1] is None) == self_form and (b[1] is None) == self_form
    if not self_form:
        assert torch.equal(a[1], b[1])
    if self_form:
        freqs = torch.tensor(O.get_freqs(N), device=DEV)
        a = ext.tril_score_v_bwd(q, q, v, do, freqs, 0)
        b = sa().tril_score_v_bwd(q, q, v, do, freqs=freqs, pos0=0)
        assert torch.equal(a[0], b[0]) and torch.equal(a[2], b[2])


def test_backward_golden(ext):
    g = golden("bwd")
    q, k, v, do = (t(g[n]) for n in ("Q", "K", "V", "dO"))
    dq, dk, dv = ext.tril_score_v_bwd(q, k, v, do)
    assert rel(dq.cpu().numpy(), g["dQ"]) < 1e-5 and rel(dk.cpu().numpy(), g["dK"]) < 1e-5
    assert rel(dv.cpu().numpy(), g["dV"]) < 1e-5
    dq, dk, dv = ext.tril_score_v_bwd(q, q, v, do)
    assert dk is None
    assert rel(dq.cpu().numpy(), g["self_dQ"]) < 1e-5 and rel(dv.cpu().numpy(), g["self_dV"]) < 1e-5


def test_cuda_attn_module_runs_the_extension(ext):
    from kernels import cuda_attn

    q = torch.relu(torch.randn(2, 4, 200, 1024, device=DEV)).bfloat16()
    v = torch.randn(2, 1, 200, 128, device=DEV).bfloat16()
    assert torch.equal(cuda_attn.tril_score_v(q, q, v), ext.tril_score_v(q, q, v))
    assert "binding=bdh_sm100_ext" in cuda_attn.ext_status()


def test_extension_calls_capture_in_a_cuda_graph(ext):
    q = torch.relu(torch.randn(2, 4, 512, 2048, device=DEV)).bfloat16()
    v = torch.randn(2, 1, 512, 256, device=DEV).bfloat16()
    eager = ext.tril_score_v(q, q, v)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        ext.tril_score_v(q, q, v)  # warm-up off the default stream (workspace, attributes)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = ext.tril_score_v(q, q, v)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
    assert sa().device_error() == 0


def test_fused_layer_ops_same_bits_as_ctypes(ext):
    """latent_encode, latent_gate_dec, layer_norm and residual_layer_norm through the extension
    against the ctypes binding on config-2 layer shapes (B = 2, T = 256)."""
    B, T, D, H, N = 2, 256, 256, 4, 8192
    g = torch.Generator(device=DEV).manual_seed(21)
    x = torch.randn(B, T, D, device=DEV, generator=g)
    xb = x.bfloat16()
    enc = sa().weight_k_major((0.02 * torch.randn(H, D, N, device=DEV, generator=g)).bfloat16())
    encv = sa().weight_k_major((0.02 * torch.randn(H, D, N, device=DEV, generator=g)).bfloat16())
    dec = sa().decoder_k_major((0.02 * torch.randn(H * N, D, device=DEV, generator=g)).bfloat16())
    freqs = torch.tensor(O.get_freqs(N), device=DEV)
    xs_a, qr_a = ext.latent_encode(xb, enc, freqs, 3)
    xs_b, qr_b = sa().latent_encode(xb, enc, freqs, 3)
    assert torch.equal(xs_a, xs_b) and torch.equal(qr_a, qr_b)
    none, qr_c = ext.latent_encode(xb, enc, freqs, 3, want_xs=False)
    assert none is None and torch.equal(qr_c, qr_b)
    y = sa().tril_score_v(qr_a, qr_a, xb.unsqueeze(1), score_terms="bf16")
    yn_a = ext.layer_norm(y, 1e-5, torch.bfloat16)
    yn_b = sa().layer_norm(y, 1e-5, out_dtype=torch.bfloat16)
    assert yn_a.dtype == torch.bfloat16 and torch.equal(yn_a, yn_b)
    m_a = ext.latent_gate_dec(yn_a, encv, xs_a, dec)
    m_b = sa().latent_gate_dec(yn_b, encv, xs_b, dec)
    assert torch.equal(m_a, m_b)
    r_a = ext.residual_layer_norm(x, m_a, 1e-5, True)
    r_b = sa().residual_layer_norm(x, m_b, 1e-5, want_bf16=True)
    assert torch.equal(r_a[0], r_b[0]) and torch.equal(r_a[1], r_b[1])
    assert ext.residual_layer_norm(x, m_a, 1e-5, False)[1] is None
    with pytest.raises(RuntimeError, match="paired frequencies"):
        ext.latent_encode(xb, enc, torch.arange(N, device=DEV, dtype=torch.float32), 0)


def test_model_logits_same_bits_through_either_binding(ext, monkeypatch):
    """The fused model's bf16 forward with the layer ops through the extension (the default when
    built) and through the ctypes binding (BDH_SM100_EXT=0): the same logits."""
    import bdh_model

    cfg = bdh_model.BDHConfig(n_layer=2, n_embd=256, n_head=4, mlp_internal_dim_multiplier=128,
                              vocab_size=256, dropout=0.0)
    torch.manual_seed(5)
    m = bdh_model.BDH(cfg).to(DEV).eval()
    m.attn._attn_impl_override = "cuda_sm100"
    idx = torch.randint(0, 256, (4, 256), device=DEV)
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        a = m(idx)[0]
        monkeypatch.setenv("BDH_SM100_EXT", "0")
        b = m(idx)[0]
    assert torch.equal(a, b)


def test_rope_into_a_strided_cache_slot(ext):
    """RoPE written straight into a capacity-strided cache slot (a view that the overlap check
    cannot classify), as the prefill of a cached model does."""
    B, H, T, cap, N = 2, 4, 48, 128, 1024
    g = torch.Generator(device=DEV).manual_seed(13)
    x = torch.relu(torch.randn(B, H, T, N, device=DEV, generator=g)).bfloat16()
    freqs = torch.tensor(O.get_freqs(N), device=DEV)
    a = torch.zeros(B, H, cap, N, device=DEV, dtype=torch.bfloat16)
    b = torch.zeros_like(a)
    ext.rope_rotate(x, freqs, 7, a[:, :, 10:10 + T])
    sa().rope_rotate(x, freqs, 7, out=b[:, :, 10:10 + T])
    assert torch.equal(a, b) and bool(a[:, :, 10:10 + T].abs().sum() > 0)
    with pytest.raises(RuntimeError, match="must not alias"):
        ext.rope_rotate(x, freqs, 0, x)
