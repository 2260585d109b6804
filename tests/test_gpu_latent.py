"""GPU parity of the fused latent projections (bdh_latent_encode / bdh_latent_gate /
bdh_latent_gate_x) against the reference's own bf16 outputs (tests/golden/golden_latent.npz),
the pinned numpy oracle and torch's cuBLAS path, and of the BDH model layer that uses them.

The projections are K = D dot products accumulated in fp32 and rounded once to bf16, so a
different accumulation order can move an output to the neighbouring bf16 value; those flips
are bounded by a mismatch fraction, everything else is compared exactly. Model stages use the
bf16 tolerance (relative Frobenius <= 3e-3).
"""

import os

import numpy as np
import pytest
import torch
import torch.nn.functional as F

import tril_oracle as O
from conftest import golden

pytestmark = pytest.mark.gpu

DEV = "cuda"


def sa():
    from kernels import sm100_attn

    return sm100_attn


def b16(x):
    return torch.as_tensor(np.asarray(x, dtype=np.float32)).to(DEV).to(torch.bfloat16)


def f32(t):
    return t.detach().float().cpu().numpy()


@pytest.fixture(autouse=True)
def _device_error_clean():
    yield
    assert sa().device_error() == 0, "a kernel reported a pipeline timeout"


def test_latent_encode_golden():
    g = golden("latent")
    freqs = torch.as_tensor(g["freqs"]).to(DEV)
    xs, qr = sa().latent_encode(b16(g["x"]), b16(g["enc"]), freqs, int(g["pos0"]))
    assert np.mean(f32(xs) != g["xs"]) < 0.01
    assert O.rel_fro(f32(xs), g["xs"]) < 3e-3
    assert np.mean(f32(qr) != g["qr"]) < 0.01
    assert O.rel_fro(f32(qr), g["qr"]) < 3e-3


def test_latent_gate_golden():
    g = golden("latent")
    xy = sa().latent_gate(b16(g["y"]), b16(g["encv"]), b16(g["xs"]))
    assert np.mean(f32(xy) != g["xy"]) < 0.01
    assert O.rel_fro(f32(xy), g["xy"]) < 3e-3


def test_latent_gate_x_golden():
    """The fused gate recomputes xs from x and enc: the reference's xy within the bf16 bound."""
    g = golden("latent")
    xy = sa().latent_gate_x(b16(g["y"]), b16(g["encv"]), b16(g["x"]), b16(g["enc"]))
    assert np.mean(f32(xy) != g["xy"]) < 0.01
    assert O.rel_fro(f32(xy), g["xy"]) < 3e-3


@pytest.mark.parametrize("B,T,D,H,N,kmaj", [(2, 200, 256, 4, 1024, False),
                                             (2, 200, 256, 4, 1024, True),
                                             (1, 130, 32, 3, 136, False),
                                             (3, 77, 96, 2, 520, True),
                                             (1, 1, 64, 1, 64, False)])
def test_latent_gate_x_equals_encode_then_gate(B, T, D, H, N, kmaj):
    """qr-only encode + fused gate give exactly the bits of encode (xs, qr) + gate: the gate's
    x enc product is the encoder's MMA sequence on the same operands."""
    g = torch.Generator().manual_seed(B * 31 + T + D)
    x = F.layer_norm(torch.randn(B, T, D, generator=g), (D,)).to(torch.bfloat16).to(DEV)
    y = F.layer_norm(torch.randn(B, H, T, D, generator=g), (D,)).to(torch.bfloat16).to(DEV)
    enc = (torch.randn(H, D, N, generator=g) * 0.1).to(torch.bfloat16).to(DEV)
    encv = (torch.randn(H, D, N, generator=g) * 0.1).to(torch.bfloat16).to(DEV)
    if kmaj:
        enc, encv = sa().weight_k_major(enc), sa().weight_k_major(encv)
    freqs = torch.as_tensor(O.get_freqs(N)).to(DEV)
    xs, qr = sa().latent_encode(x, enc, freqs, 7)
    none, qr_only = sa().latent_encode(x, enc, freqs, 7, want_xs=False)
    assert none is None and torch.equal(qr_only, qr)
    xy = sa().latent_gate(y, encv, xs)
    xy_x = sa().latent_gate_x(y, encv, x, enc)
    assert torch.equal(xy_x, xy)
    xy_o = O.latent_gate(f32(y), f32(encv), O.latent_encode(f32(x), f32(enc), O.get_freqs(N), 7)[0])
    assert O.rel_fro(f32(xy_x), xy_o) < 3e-3


def test_latent_gate_x_ragged_latent_width():
    """N = 130 (not a multiple of the 8-element store chunk) through padded views: the ragged
    last chunk of every row is written pair by pair and nothing past N is touched."""
    B, T, D, H, N, NP = 2, 100, 64, 2, 130, 136
    g = torch.Generator().manual_seed(130)

    def padded(*shape):
        return torch.empty(*shape[:-1], NP, dtype=torch.bfloat16, device=DEV)[..., :shape[-1]]

    x = torch.randn(B, T, D, generator=g).to(torch.bfloat16).to(DEV)
    y = torch.randn(B, H, T, D, generator=g).to(torch.bfloat16).to(DEV)
    enc, encv = padded(H, D, N), padded(H, D, N)
    enc.copy_((torch.randn(H, D, N, generator=g) * 0.1).to(torch.bfloat16))
    encv.copy_((torch.randn(H, D, N, generator=g) * 0.1).to(torch.bfloat16))
    freqs = torch.as_tensor(O.get_freqs(N)).to(DEV)
    xs = padded(B, T, H, N)
    sa().latent_encode(x, enc, freqs, 0, xs_out=xs, qr_out=padded(B, H, T, N))
    ref = padded(B, T, H, N)
    sa().latent_gate(y, encv, xs, out=ref)
    full = torch.full((B, T, H, NP), 5.0, dtype=torch.bfloat16, device=DEV)
    out = sa().latent_gate_x(y, encv, x, enc, out=full[..., :N])
    assert torch.equal(out, ref)
    assert bool((full[..., N:] == 5.0).all())


def test_latent_gate_x_rejects_mixed_weight_layouts():
    B, T, D, H, N = 1, 64, 64, 2, 128
    x = torch.zeros(B, T, D, dtype=torch.bfloat16, device=DEV)
    y = torch.zeros(B, H, T, D, dtype=torch.bfloat16, device=DEV)
    w = torch.zeros(H, D, N, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(RuntimeError, match="same layout"):
        sa().latent_gate_x(y, w, x, sa().weight_k_major(w))


@pytest.mark.parametrize("B,T,D,H,N,pos0", [(2, 200, 256, 4, 1024, 5), (1, 128, 64, 2, 200, 0),
                                            (3, 77, 96, 1, 520, 4090)])
def test_latent_encode_vs_oracle(B, T, D, H, N, pos0):
    g = torch.Generator().manual_seed(B * 1000 + T)
    x = F.layer_norm(torch.randn(B, T, D, generator=g), (D,)).to(torch.bfloat16)
    enc = (torch.randn(H, D, N, generator=g) * 0.1).to(torch.bfloat16)
    freqs = O.get_freqs(N)
    xs, qr = sa().latent_encode(x.to(DEV), enc.to(DEV), torch.as_tensor(freqs).to(DEV), pos0)
    xs_o, qr_o = O.latent_encode(x.float().numpy(), enc.float().numpy(), freqs, pos0)
    assert np.mean(f32(xs) != xs_o) < 2e-3
    assert O.rel_fro(f32(xs), xs_o) < 3e-3
    assert O.rel_fro(f32(qr), qr_o) < 3e-3
    # the rotation of the kernel's own xs is the library's RoPE, element for element
    qr_r = sa().rope_rotate(xs.permute(0, 2, 1, 3), torch.as_tensor(freqs).to(DEV), pos0)
    assert torch.equal(qr, qr_r)


@pytest.mark.parametrize("B,T,D,H,N", [(2, 200, 256, 4, 1024), (1, 130, 32, 3, 136)])
def test_latent_gate_vs_oracle(B, T, D, H, N):
    g = torch.Generator().manual_seed(B * 77 + T)
    y = F.layer_norm(torch.randn(B, H, T, D, generator=g), (D,)).to(torch.bfloat16)
    encv = (torch.randn(H, D, N, generator=g) * 0.1).to(torch.bfloat16)
    xs = torch.relu(torch.randn(B, T, H, N, generator=g)).to(torch.bfloat16)
    xy = sa().latent_gate(y.to(DEV), encv.to(DEV), xs.to(DEV))
    xy_o = O.latent_gate(y.float().numpy(), encv.float().numpy(), xs.float().numpy())
    assert np.mean(f32(xy) != xy_o) < 2e-3
    assert O.rel_fro(f32(xy), xy_o) < 3e-3


def test_latent_encode_into_strided_cache_slot():
    B, T, D, H, N, cap, pos0 = 2, 150, 256, 4, 512, 400, 100
    g = torch.Generator().manual_seed(11)
    x = torch.randn(B, T, D, generator=g).to(torch.bfloat16).to(DEV)
    enc = (torch.randn(H, D, N, generator=g) * 0.05).to(torch.bfloat16).to(DEV)
    freqs = torch.as_tensor(O.get_freqs(N)).to(DEV)
    buf = torch.full((B, H, cap, N), 7.0, dtype=torch.bfloat16, device=DEV)
    slot = buf.narrow(2, pos0, T)
    xs, qr = sa().latent_encode(x, enc, freqs, pos0, qr_out=slot)
    assert qr.data_ptr() == slot.data_ptr()
    _, qr_ref = sa().latent_encode(x, enc, freqs, pos0)
    assert torch.equal(slot, qr_ref)
    assert bool((buf[:, :, :pos0] == 7.0).all()) and bool((buf[:, :, pos0 + T:] == 7.0).all())


def test_latent_kernels_full_size_vs_cublas():
    """Config-2 layer shapes (B=8 of 32, T=512, D=256, nh=4, N=8192) against torch's bf16
    einsum + ReLU (cuBLAS) and the library's RoPE / gated product on the same operands."""
    B, T, D, H, N = 8, 512, 256, 4, 8192
    g = torch.Generator(device=DEV).manual_seed(5)
    x = F.layer_norm(torch.randn(B, T, D, device=DEV, generator=g), (D,)).to(torch.bfloat16)
    enc = (torch.randn(H, D, N, device=DEV, generator=g) * 0.02).to(torch.bfloat16)
    encv = (torch.randn(H, D, N, device=DEV, generator=g) * 0.02).to(torch.bfloat16)
    y = F.layer_norm(torch.randn(B, H, T, D, device=DEV, generator=g), (D,)).to(torch.bfloat16)
    freqs = torch.as_tensor(O.get_freqs(N)).to(DEV)
    xs, qr = sa().latent_encode(x, enc, freqs, 0)
    xs_ref = torch.relu(torch.einsum("btd,hdn->bthn", x, enc))
    assert (xs != xs_ref).float().mean().item() < 2e-3
    d = (xs.float() - xs_ref.float()).norm() / xs_ref.float().norm()
    assert d.item() < 3e-3
    assert torch.equal(qr, sa().rope_rotate(xs.permute(0, 2, 1, 3), freqs, 0))
    xy = sa().latent_gate(y, encv, xs)
    xy_ref = xs * torch.relu(torch.einsum("bhtd,hdn->bthn", y, encv))
    assert (xy != xy_ref).float().mean().item() < 2e-3
    d = (xy.float() - xy_ref.float()).norm() / xy_ref.float().norm()
    assert d.item() < 3e-3
    # the model's form: qr-only encode + gate with xs recomputed, same bits
    assert torch.equal(sa().latent_encode(x, enc, freqs, 0, want_xs=False)[1], qr)
    assert torch.equal(sa().latent_gate_x(y, encv, x, enc), xy)


def _model(n_layer=2, n_embd=256, n_head=4, mult=128):
    import bdh_model

    cfg = bdh_model.BDHConfig(n_layer=n_layer, n_embd=n_embd, n_head=n_head,
                              mlp_internal_dim_multiplier=mult, vocab_size=256, dropout=0.0)
    torch.manual_seed(3)
    m = bdh_model.BDH(cfg).to(DEV).eval()
    m.attn._attn_impl_override = "cuda_sm100"
    return m


def _launch_counts(fn):
    """Run fn() between the library's profile_begin / profile_end; launches per kernel kind."""
    sa().profile_begin()
    fn()
    return {k: v["launches"] for k, v in sa().profile_end().items()}


def test_model_latent_layer_matches_unfused_and_oracle(monkeypatch):
    """Fused latent layer vs the unfused sm100 layer (the same arithmetic: bf16 GEMM outputs,
    bf16 RoPE and product, scores rounded to bf16 before the value product), and vs the float64
    oracle of the bf16-autocast forward, all within the bf16 bar. One layer: through more
    layers every bf16 rounding point that flips with the accumulation order grows (two faithful
    executions of the reference's own bf16 model differ by about 3e-3 at two layers); the
    multi-layer end-to-end check is against the reference's logits in
    test_gpu_config2_parity.py."""
    m = _model(n_layer=1)
    idx = torch.randint(0, 256, (2, 128), generator=torch.Generator().manual_seed(9)).to(DEV)
    res = {}
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        monkeypatch.setenv("BDH_SM100_LATENT", "1")
        assert m._latent_fusable("cuda_sm100", 128, None, idx.device)
        cnt = _launch_counts(lambda: res.setdefault("fused", m(idx)[0].float()))
        assert cnt["encode"] == 1 and cnt["gate"] == 1 and cnt["rope"] == 0, cnt
        # the same arithmetic as the unfused layers: the gate followed by cuBLAS's decoder
        monkeypatch.setenv("BDH_SM100_GATE_DEC", "0")
        res["fused_cublas_dec"] = m(idx)[0].float()
        monkeypatch.setenv("BDH_SM100_LATENT", "0")
        cnt = _launch_counts(lambda: res.setdefault("plain", m(idx)[0].float()))
        assert cnt["encode"] == 0 and cnt["rope"] == 1, cnt
    fused, plain = res["fused"], res["plain"]
    fc = res["fused_cublas_dec"]
    assert ((fc - plain).norm() / plain.norm()).item() < 1e-3
    assert ((fused - plain).norm() / plain.norm()).item() < 3e-3
    w = {k: getattr(m, k).detach().to(torch.bfloat16).float().cpu().numpy()
         for k in ("encoder", "encoder_v", "decoder", "lm_head")}
    w["embed"] = m.embed.weight.detach().float().cpu().numpy()
    w["freqs"] = m.attn.freqs.reshape(-1).cpu().numpy()
    ref16 = O.bdh_forward_bf16(idx.cpu().numpy(), w, n_layer=1, n_head=4)
    assert O.rel_fro(f32(fused), ref16) < 3e-3


@pytest.mark.parametrize("n_embd,n_head,mult", [(128, 4, 12), (384, 6, 8), (256, 4, 3)])
def test_model_latent_layer_other_widths(monkeypatch, n_embd, n_head, mult):
    """The fused layer's other branches: D = 128 (N = 384) and D = 384 (six heads, N = 512: the
    attention LayerNorm runs after the value pass, D > 256), where the gate runs with cuBLAS's
    decoder GEMM (the fused gate + decoder needs D = 256); and D = 256 with N = 192, a latent
    width that is not a multiple of 128 (gate with ragged latent blocks). Against the unfused
    sm100 layer and the float64 oracle of the bf16-autocast forward, one layer, bf16 bar."""
    m = _model(n_layer=1, n_embd=n_embd, n_head=n_head, mult=mult)
    idx = torch.randint(0, 256, (2, 128), generator=torch.Generator().manual_seed(19)).to(DEV)
    res = {}
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        monkeypatch.setenv("BDH_SM100_LATENT", "1")
        assert m._latent_fusable("cuda_sm100", 128, None, idx.device)
        cnt = _launch_counts(lambda: res.setdefault("fused", m(idx)[0].float()))
        assert cnt["encode"] == 1 and cnt["gate"] == 1 and cnt["rope"] == 0, cnt
        monkeypatch.setenv("BDH_SM100_LATENT", "0")
        res["plain"] = m(idx)[0].float()
    fused, plain = res["fused"], res["plain"]
    assert ((fused - plain).norm() / plain.norm()).item() < 3e-3
    w = {k: getattr(m, k).detach().to(torch.bfloat16).float().cpu().numpy()
         for k in ("encoder", "encoder_v", "decoder", "lm_head")}
    w["embed"] = m.embed.weight.detach().float().cpu().numpy()
    w["freqs"] = m.attn.freqs.reshape(-1).cpu().numpy()
    ref16 = O.bdh_forward_bf16(idx.cpu().numpy(), w, n_layer=1, n_head=n_head)
    assert O.rel_fro(f32(fused), ref16) < 3e-3
    assert sa().device_error() == 0


def test_model_gate_x_matches_stored_xs(monkeypatch):
    """The model's fused layer with xs recomputed in the gate (BDH_SM100_GATE_X=1) and with xs
    stored and re-read (default) give identical logits."""
    m = _model(n_layer=2)
    idx = torch.randint(0, 256, (2, 256), generator=torch.Generator().manual_seed(19)).to(DEV)
    out = {}
    monkeypatch.setenv("BDH_SM100_LATENT", "1")
    monkeypatch.setenv("BDH_SM100_GATE_DEC", "0")  # both forms through cuBLAS's decoder
    for flag in ("1", "0"):
        monkeypatch.setenv("BDH_SM100_GATE_X", flag)
        with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
            out[flag] = m(idx)[0].float()
    assert torch.equal(out["1"], out["0"])


def test_model_latent_layer_stagewise_vs_oracle():
    """One fused layer stage by stage, each stage fed the GPU's own inputs: encode (xs, qr),
    attention output, gate, decoder projection — each within the bf16 bound."""
    m = _model(n_layer=1)
    B, T = 2, 128
    idx = torch.randint(0, 256, (B, T), generator=torch.Generator().manual_seed(9)).to(DEV)
    freqs = m.attn.freqs.reshape(-1).cpu().numpy()
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        x = m._ln(m.embed(idx))
        xb = x.to(torch.bfloat16)
        enc, encv, dec = (m._bf16_param(k) for k in ("encoder", "encoder_v", "decoder"))
        xs, qr = sa().latent_encode(xb, enc, m.attn.freqs, 0)
        v = x.unsqueeze(1).to(torch.bfloat16)
        y = sa().tril_score_v(qr, qr, v)
        yn = m._ln(y.float()).to(torch.bfloat16)
        xy = sa().latent_gate(yn, encv, xs)
        ym = F.linear(xy.view(B, T, -1), dec.t())
    xs_o, qr_o = O.latent_encode(f32(xb), f32(enc), freqs, 0)
    assert O.rel_fro(f32(xs), xs_o) < 3e-3 and O.rel_fro(f32(qr), qr_o) < 3e-3
    q64 = f32(qr).astype(np.float64)
    y_o = O.tril_score_v(q64, q64, f32(v).astype(np.float64))
    assert O.rel_fro(f32(y), y_o) < 3e-3
    assert O.rel_fro(f32(xy), O.latent_gate(f32(yn), f32(encv), f32(xs))) < 3e-3
    ym_o = np.einsum("btk,kd->btd", f32(xy).reshape(B, T, -1).astype(np.float64),
                     f32(dec).astype(np.float64))
    assert O.rel_fro(f32(ym), ym_o) < 3e-3


def test_model_latent_prefill_then_decode(monkeypatch):
    """Cached prefill on the fused kernels (QR written into the cache slot), then T=1 steps;
    logits agree with the unfused path step by step."""
    from bdh_cache import CacheManager

    m = _model(n_layer=2)
    B, P, steps = 2, 192, 4
    idx = torch.randint(0, 256, (B, P + steps), generator=torch.Generator().manual_seed(4)).to(DEV)

    def run(flag, storage):
        monkeypatch.setenv("BDH_SM100_LATENT", flag)
        cache = CacheManager.from_config(m.config, B, P + steps, idx.device, storage_dtype=storage)
        out = []
        with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
            lg, _ = m(idx[:, :P], cache=cache)
            out.append(lg[:, -1].float())
            for t in range(P, P + steps):
                lg, _ = m(idx[:, t:t + 1], cache=cache)
                out.append(lg[:, -1].float())
        return torch.stack(out)

    # the gate followed by cuBLAS's decoder on both sides, so that only the cache-slot path
    # differs (the fused gate + decoder has its own model test in test_gpu_gate_dec.py)
    monkeypatch.setenv("BDH_SM100_GATE_DEC", "0")
    for storage in (None, torch.bfloat16):
        a = run("1", storage)
        b = run("0", storage)
        r = ((a - b).norm() / b.norm()).item()
        assert r < 3e-3, (storage, r)


@pytest.mark.parametrize("D,N", [(256, 1024), (96, 520)])
def test_latent_k_major_weights_match_n_major(D, N):
    """Weights given as a transposed (H, N, D) copy (read K-major) give the same bits as the
    n-contiguous (H, D, N) layout: the MMAs accumulate over the same k order."""
    B, T, H = 2, 150, 3
    g = torch.Generator().manual_seed(D + N)
    x = torch.randn(B, T, D, generator=g).to(torch.bfloat16).to(DEV)
    y = torch.randn(B, H, T, D, generator=g).to(torch.bfloat16).to(DEV)
    enc = (torch.randn(H, D, N, generator=g) * 0.1).to(torch.bfloat16).to(DEV)
    encv = (torch.randn(H, D, N, generator=g) * 0.1).to(torch.bfloat16).to(DEV)
    freqs = torch.as_tensor(O.get_freqs(N)).to(DEV)
    xs_n, qr_n = sa().latent_encode(x, enc, freqs, 3)
    enc_k = sa().weight_k_major(enc)
    assert enc_k.stride(1) == 1 and torch.equal(enc_k, enc)
    xs_k, qr_k = sa().latent_encode(x, enc_k, freqs, 3)
    assert torch.equal(xs_n, xs_k) and torch.equal(qr_n, qr_k)
    xy_n = sa().latent_gate(y, encv, xs_n)
    xy_k = sa().latent_gate(y, sa().weight_k_major(encv), xs_n)
    assert torch.equal(xy_n, xy_k)


@pytest.mark.parametrize("shape", [(2, 4, 300, 256), (3, 200), (5, 7, 520)])
@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
def test_layer_norm_matches_torch(shape, dt):
    g = torch.Generator(device=DEV).manual_seed(len(shape))
    x = (torch.randn(*shape, device=DEV, generator=g) * 3 + 1).to(dt)
    ref = F.layer_norm(x.float(), (shape[-1],), eps=1e-5)
    y32 = sa().layer_norm(x, 1e-5, out_dtype=torch.float32)
    assert ((y32 - ref).norm() / ref.norm()).item() < 1e-6
    y16 = sa().layer_norm(x, 1e-5, out_dtype=torch.bfloat16)
    assert (y16 != ref.to(torch.bfloat16)).float().mean().item() < 1e-2
    assert torch.equal(y16, y32.to(torch.bfloat16))


@pytest.mark.parametrize("D", [256, 200])
@pytest.mark.parametrize("ydt", [torch.float32, torch.bfloat16])
def test_residual_layer_norm_matches_torch(D, ydt):
    g = torch.Generator(device=DEV).manual_seed(D)
    x = torch.randn(4, 150, D, device=DEV, generator=g)
    y = (torch.randn(4, 150, D, device=DEV, generator=g) * 0.1).to(ydt)
    out, out16 = sa().residual_layer_norm(x, y, 1e-5, want_bf16=True)
    ref = F.layer_norm(x + F.layer_norm(y.float(), (D,), eps=1e-5), (D,), eps=1e-5)
    assert ((out - ref).norm() / ref.norm()).item() < 1e-6
    assert torch.equal(out16, out.to(torch.bfloat16))
