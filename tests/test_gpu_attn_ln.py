"""The forward with the attention output's LayerNorm (bdh_tril_score_v_layernorm): folded into
the value pass's epilogue for the quadratic bf16 form, applied to the output rows afterwards for
the fp32 and chunked forms. Against the forward followed by the LayerNorm kernel and against
float64 (LN(bf16(tril(Q Q^T, -1) V)), the reference's bf16 autocast order, bdh.py:1044)."""

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def sa():
    from kernels import sm100_attn

    return sm100_attn


def _inputs(B, H, T, N, D, dt, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    q = torch.relu(torch.randn(B, H, T, N, device=DEV, generator=g)).to(dt)
    v = torch.randn(B, 1, T, D, device=DEV, generator=g).to(dt)
    return q, v


def _ln64(y, eps):
    y = y.double()
    m = y.mean(-1, keepdim=True)
    var = ((y - m) ** 2).mean(-1, keepdim=True)
    return (y - m) / torch.sqrt(var + eps)


@pytest.mark.parametrize("terms", ["bf16", "split"])
@pytest.mark.parametrize("shape", [(2, 4, 512, 8192, 256), (1, 3, 300, 512, 64), (2, 2, 129, 256, 136)])
def test_fused_value_pass_layernorm(shape, terms):
    B, H, T, N, D = shape
    q, v = _inputs(B, H, T, N, D, torch.bfloat16, T + D)
    s = sa()
    fused = s.tril_score_v(q, q, v, score_terms=terms, ln_eps=1e-5)
    plain = s.tril_score_v(q, q, v, score_terms=terms)
    sep = s.layer_norm(plain, 1e-5)
    assert fused.shape == plain.shape and fused.dtype == torch.bfloat16
    # the same bf16 output rows normalised: within one bf16 rounding of the separate kernel's
    # result (the two sum the row statistics in different orders)
    diff = (fused.float() - sep.float()).abs()
    assert diff.max().item() <= 2 ** -7 * sep.float().abs().max().item()
    assert (diff > 0).float().mean().item() < 0.02
    ref = _ln64(plain, 1e-5)
    rel = ((fused.double() - ref).norm() / ref.norm()).item()
    assert rel < 3e-3, rel
    assert torch.equal(fused, s.tril_score_v(q, q, v, score_terms=terms, ln_eps=1e-5))
    assert s.device_error() == 0


@pytest.mark.parametrize("dt,T", [(torch.float32, 200), (torch.bfloat16, 2048)])
def test_layernorm_after_other_forms_equals_separate_kernel(dt, T):
    """fp32 inputs and the chunked bf16 forward (T >= 1536) normalise the rows in place after
    the forward: the same kernels as the forward followed by layer_norm, the same bits."""
    q, v = _inputs(1, 2, T, 512, 64, dt, 7)
    s = sa()
    fused = s.tril_score_v(q, q, v, ln_eps=1e-5)
    sep = s.layer_norm(s.tril_score_v(q, q, v), 1e-5)
    assert torch.equal(fused, sep)


def test_extension_forms_agree():
    from kernels import sm100_ext

    ext = sm100_ext.load_ext()
    q, v = _inputs(2, 4, 384, 2048, 256, torch.bfloat16, 3)
    with sa().score_terms_scope("bf16"):
        a = ext.tril_score_v(q, q, v, 1e-5)
        b = sa().tril_score_v(q, q, v, ln_eps=1e-5)
    assert torch.equal(a, b)
