"""GPU parity of the fp32 decoder product of a decode step (bdh_decoder_f32): out = x @ w with K
split into 256-row slices summed in a fixed order. The reference computes y_mlp = xy @ decoder
in fp32 (bdh.py:1050); the bar is the fp32 one (relative Frobenius <= 1e-5) against float64
sums of the same inputs, and against torch's fp32 matmul."""

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def sa():
    from kernels import sm100_attn

    return sm100_attn


def rel(a, b):
    return ((a.double() - b.double()).norm() / b.double().norm()).item()


@pytest.mark.parametrize("M,K,D", [(64, 32768, 256), (1, 256, 256), (130, 1000, 36),
                                   (3, 77, 260), (65, 8192, 128)])
def test_decoder_f32_vs_float64(M, K, D):
    """Ragged K (a partial last slice), M beyond one 64-row block, D not a multiple of 128."""
    g = torch.Generator().manual_seed(M * 7 + K + D)
    x = torch.relu(torch.randn(M, K, generator=g)).to(DEV)
    w = (torch.randn(K, D, generator=g) * 0.02).to(DEV)
    out = sa().decoder_f32(x, w)
    assert out.shape == (M, D) and out.dtype == torch.float32
    assert rel(out, x.double() @ w.double()) < 1e-5
    assert rel(out, x @ w) < 1e-5
    assert torch.equal(out, sa().decoder_f32(x, w))  # fixed summation order


def test_decoder_f32_strided_operands():
    g = torch.Generator().manual_seed(4)
    big_x = torch.randn(40, 3000, generator=g).to(DEV)
    x = big_x[5:37, 100:2148]  # row stride 3000
    w = torch.randn(2048, 64, generator=g).to(DEV)
    big_o = torch.full((32, 100), 9.0, device=DEV)
    out = big_o[:, 20:84]
    r = sa().decoder_f32(x, w, out=out)
    assert r.data_ptr() == out.data_ptr()
    assert rel(out, x.double() @ w.double()) < 1e-5
    assert bool((big_o[:, :20] == 9.0).all()) and bool((big_o[:, 84:] == 9.0).all())


def test_decoder_f32_rejects_bad_shapes():
    x = torch.randn(4, 64, device=DEV)
    with pytest.raises(ValueError):
        sa().decoder_f32(x, torch.randn(32, 8, device=DEV))
    with pytest.raises(RuntimeError, match="multiples of 4"):
        sa().decoder_f32(x, torch.randn(64, 6, device=DEV))


def test_model_fp32_decode_uses_decoder_f32(monkeypatch):
    """The fp32 model's cached decode steps run one bdh_decoder_f32 per layer; the logits match
    torch's linear (BDH_SM100_DEC_F32=0) within the fp32 bar."""
    import bdh_model
    from bdh_cache import CacheManager

    cfg = bdh_model.BDHConfig(n_layer=2, n_embd=256, n_head=4, mlp_internal_dim_multiplier=32,
                              vocab_size=256, dropout=0.0)
    torch.manual_seed(5)
    m = bdh_model.BDH(cfg).to(DEV).eval()
    m.attn._attn_impl_override = "cuda_sm100"
    B, P, steps = 4, 40, 3
    idx = torch.randint(0, 256, (B, P + steps), generator=torch.Generator().manual_seed(6)).to(DEV)
    res = {}
    for flag in ("1", "0"):
        monkeypatch.setenv("BDH_SM100_DEC_F32", flag)
        cache = CacheManager.from_config(m.config, B, P + steps, DEV)
        out = []
        with torch.no_grad():
            m(idx[:, :P], cache=cache)
            sa().profile_begin()
            for t in range(P, P + steps):
                lg, _ = m(idx[:, t:t + 1], cache=cache)
                out.append(lg[:, -1].float())
            cnt = {k: v["launches"] for k, v in sa().profile_end().items()}
        assert cnt["decoder"] == (cfg.n_layer * steps if flag == "1" else 0), cnt
        res[flag] = torch.stack(out)
    assert rel(res["1"], res["0"]) < 1e-5
