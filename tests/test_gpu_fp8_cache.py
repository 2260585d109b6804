"""GPU parity of the fp8 key-cache wire format: bdh_quantize_rows_fp8 against the oracle (bit for
bit), bdh_tril_decode_fp8 against the oracle's decode over the dequantized keys (fp32 tolerance
1e-5), its fused RoPE + slot quantization, and the cached model on an fp8 cache.

The format is lossy by design (3 mantissa bits): the kernels are exact w.r.t. the dequantized
values, and the model's logits on an fp8 cache are compared with the fp32 cache at 3e-2."""

import numpy as np
import pytest
import torch

import tril_oracle as O

pytestmark = pytest.mark.gpu

DEV = "cuda"
FP8 = torch.float8_e4m3fn


def sa():
    from kernels import sm100_attn

    return sm100_attn


@pytest.fixture(autouse=True)
def _device_error_clean():
    yield
    assert sa().device_error() == 0, "a kernel reported a pipeline timeout"


def _f(t):
    return t.detach().float().cpu().numpy()


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("N", [8192, 130, 48])
def test_quantize_rows_matches_oracle(dt, N):
    g = torch.Generator().manual_seed(N)
    x = (torch.randn(2, 3, 7, N, generator=g) * torch.rand(2, 3, 7, 1, generator=g) * 40).to(dt)
    x[1, 2, 3] = 0
    q, sc = sa().quantize_rows_fp8(x.to(DEV))
    q_o, sc_o = O.quantize_rows_fp8(x.float().numpy())
    assert np.array_equal(_f(q), q_o)
    assert np.array_equal(_f(sc), sc_o)


def test_quantize_rows_into_strided_cache_slot():
    B, H, T, N, cap, pos = 2, 4, 5, 512, 40, 17
    x = torch.randn(B, H, T, N, device=DEV) * 3
    buf = torch.full((B, H, cap, N), 1.0, device=DEV).to(FP8)
    sbuf = torch.full((B, H, cap), -1.0, device=DEV)
    sa().quantize_rows_fp8(x, out=buf.narrow(2, pos, T), scale=sbuf.narrow(2, pos, T))
    q, sc = sa().quantize_rows_fp8(x)
    assert torch.equal(buf[:, :, pos:pos + T].float(), q.float())
    assert torch.equal(sbuf[:, :, pos:pos + T], sc)
    assert bool((buf[:, :, :pos].float() == 1).all()) and bool((buf[:, :, pos + T:].float() == 1).all())
    assert bool((sbuf[:, :, :pos] == -1).all())


def _history(B, H, S, N, D, cap, Hv, vdt, seed):
    g = torch.Generator().manual_seed(seed)
    kr = torch.randn(B, H, S, N, generator=g) * torch.rand(B, H, S, 1, generator=g) * 4
    v = torch.randn(B, Hv, S, D, generator=g).to(vdt)
    kbuf = torch.zeros(B, H, cap, N, dtype=FP8, device=DEV)
    sbuf = torch.zeros(B, H, cap, device=DEV)
    vbuf = torch.zeros(B, Hv, cap, D, dtype=vdt, device=DEV)
    k8, ks = kbuf.narrow(2, 0, S), sbuf.narrow(2, 0, S)
    sa().quantize_rows_fp8(kr.to(DEV), out=k8, scale=ks)
    vbuf.narrow(2, 0, S).copy_(v)
    return k8, ks, vbuf.narrow(2, 0, S)


@pytest.mark.parametrize("B,H,S,N,D,Hv,vdt,qdt", [
    (3, 4, 300, 8192, 256, 1, torch.bfloat16, torch.float32),
    (2, 2, 129, 1024, 256, 2, torch.float32, torch.float32),
    (1, 3, 17, 136, 64, 1, torch.bfloat16, torch.bfloat16),
    (2, 1, 1, 512, 128, 1, torch.float32, torch.float32)])
def test_decode_fp8_matches_oracle(B, H, S, N, D, Hv, vdt, qdt):
    k8, ks, v = _history(B, H, S, N, D, S + 9, Hv, vdt, seed=S + N)
    q = (torch.randn(B, H, 1, N, generator=torch.Generator().manual_seed(5)) * 2).to(qdt)
    out = sa().tril_decode_fp8(q.to(DEV), k8, ks, v)
    ref = O.tril_decode_fp8(q.float().numpy(), _f(k8), _f(ks), _f(v))
    tol = 1e-5 if qdt == torch.float32 else 3e-3
    assert O.rel_fro(_f(out), ref) < tol


def test_decode_fp8_empty_past_gives_zeros():
    B, H, N, D = 2, 4, 256, 64
    q = torch.randn(B, H, 1, N, device=DEV)
    k8 = torch.zeros(B, H, 0, N, dtype=FP8, device=DEV)
    out = sa().tril_decode_fp8(q, k8, torch.zeros(B, H, 0, device=DEV),
                               torch.zeros(B, 1, 0, D, device=DEV))
    assert out.shape == (B, H, 1, D) and bool((out == 0).all())


def test_decode_fp8_fused_rope_and_slot():
    """The rotated query is quantized into this step's slot (bytes and scale equal the
    library's RoPE followed by the quantizer) and the output equals the decode with the query
    rotated beforehand."""
    B, H, S, N, D, pos = 2, 4, 200, 8192, 256, 200
    k8, ks, v = _history(B, H, S, N, D, S + 1, 1, torch.bfloat16, seed=11)
    freqs = torch.as_tensor(O.get_freqs(N)).to(DEV)
    q = torch.relu(torch.randn(B, H, 1, N, device=DEV))
    slot = torch.zeros(B, H, 1, N, dtype=FP8, device=DEV)
    slot_sc = torch.zeros(B, H, 1, device=DEV)
    out = sa().tril_decode_fp8(q, k8, ks, v, freqs=freqs, pos=pos, kr_slot=slot, slot_scale=slot_sc)
    qr = sa().rope_rotate(q, freqs, pos)
    q8, sc = sa().quantize_rows_fp8(qr)
    assert torch.equal(slot.float(), q8.float()) and torch.equal(slot_sc, sc)
    assert torch.equal(out, sa().tril_decode_fp8(qr, k8, ks, v))
    ref = O.tril_decode_fp8(_f(qr), _f(k8), _f(ks), _f(v))
    assert O.rel_fro(_f(out), ref) < 1e-5


def _model(n_layer=2):
    import bdh_model

    cfg = bdh_model.BDHConfig(n_layer=n_layer, n_embd=256, n_head=4, mlp_internal_dim_multiplier=128,
                              vocab_size=256, dropout=0.0)
    torch.manual_seed(3)
    m = bdh_model.BDH(cfg).to(DEV).eval()
    m.attn._attn_impl_override = "cuda_sm100"
    return m


def _run_cached(m, idx, P, storage, impl="cuda_sm100"):
    from bdh_cache import CacheManager

    m.attn._attn_impl_override = impl
    cache = CacheManager.from_config(m.config, idx.size(0), idx.size(1), idx.device,
                                     storage_dtype=storage)
    out = []
    with torch.no_grad():
        lg, _ = m(idx[:, :P], cache=cache)
        out.append(lg[:, -1].float())
        for t in range(P, idx.size(1)):
            lg, _ = m(idx[:, t:t + 1], cache=cache)
            out.append(lg[:, -1].float())
    m.attn._attn_impl_override = "cuda_sm100"
    return torch.stack(out), cache


def test_model_fp8_cache_matches_eager_and_fp32_cache(monkeypatch):
    """Cached prefill + decode on an fp8 key cache: the native decode (fp8 stream, fused RoPE and
    slot quantization) matches the eager path over the dequantized cache within the bf16 bound
    (the decode steps read the bf16 value slots; both prefills attend over the fp32 values), and
    stays within 3e-2 of the fp32 cache (the e4m3 rounding of the keys)."""
    m = _model()
    B, P, steps = 2, 160, 6
    idx = torch.randint(0, 256, (B, P + steps), generator=torch.Generator().manual_seed(8)).to(DEV)
    monkeypatch.setenv("BDH_SM100_LATENT", "0")
    native, cache = _run_cached(m, idx, P, FP8)
    assert cache.kr_fp8 and cache.seq_len == P + steps
    eager, _ = _run_cached(m, idx, P, FP8, impl="eager")
    assert ((native - eager).norm() / eager.norm()).item() < 3e-3
    f32, _ = _run_cached(m, idx, P, None)
    assert ((native - f32).norm() / f32.norm()).item() < 3e-2


def test_model_fp8_cache_fused_latent_prefill(monkeypatch):
    """The fused latent prefill quantizes QR into the fp8 cache; decode steps then agree with the
    unfused prefill on the same cache format."""
    m = _model()
    B, P, steps = 2, 128, 4
    idx = torch.randint(0, 256, (B, P + steps), generator=torch.Generator().manual_seed(9)).to(DEV)
    res = {}
    # the gate followed by cuBLAS's decoder on both sides, so that only the QR path differs (the
    # fused gate + decoder has its own model test in test_gpu_gate_dec.py)
    monkeypatch.setenv("BDH_SM100_GATE_DEC", "0")
    for flag in ("1", "0"):
        monkeypatch.setenv("BDH_SM100_LATENT", flag)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            res[flag], _ = _run_cached(m, idx, P, FP8)
    assert ((res["1"] - res["0"]).norm() / res["0"].norm()).item() < 3e-3
