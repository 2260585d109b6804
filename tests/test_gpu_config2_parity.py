"""The model at config-2 width against the REFERENCE model's own outputs
(golden_config2_bf16.npz, written by tests/golden/make_golden.py from bdh.BDH: n_embd 256,
4 heads, N = 8192 latent columns per head, 2 layers, B = 2, T = 128, weights rebuilt from
tests/golden/config2_case.py), and against the reference's op sequence run by torch on this GPU.

bf16. The reference run is bdh.py's AMP forward (bdh.py:486-500) with CUDA autocast's casts
(layer_norm in fp32), which is how it runs on a GPU.
* Per layer: each fused layer (latent encode + RoPE, tril attention with the scores rounded to
  bf16 as the reference's eager attention rounds them, LayerNorm, gate + decoder, residual
  LayerNorms), fed the reference's own residual stream, is held to the 3e-3 bar.
* End to end, every bf16 rounding point can flip with the order of the fp32 accumulations
  before it, and the flips grow through the layers. The reference's own logits move by up to
  3.1e-3 between two CPU executions of the same run (one thread, or ATen's GEMMs instead of
  oneDNN's: ``reference_bf16_floor``), and by 3.8e-3 when its op sequence runs on this GPU
  (``_reference_ops``, measured in the test): the B200's tensor cores truncate each fp32
  accumulation step. The fused model's logits are held to the larger of 3e-3 and those measured
  floors, with 10% for the order of its own accumulations (its decoder product sums
  K = nh * N = 32768 in one accumulator where cuBLAS splits K at this 256-row shape).
* At the full config-2 batch (B = 32, T = 512, 2 layers), where the reference's GEMMs do not
  split K either, the fused model is held to 3e-3 against the reference's op sequence on this
  GPU.
fp32: the model without autocast against the reference's fp32 logits at 1e-5.
"""

import numpy as np
import pytest
import torch
import torch.nn.functional as F

import tril_oracle as O
from conftest import config2_case, golden, reference_bf16_floor

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _model(impl="cuda_sm100", n_layer=None):
    import bdh_model

    C = config2_case()
    cfg = bdh_model.BDHConfig(n_layer=n_layer or C.N_LAYER, n_embd=C.N_EMBD, n_head=C.N_HEAD,
                              mlp_internal_dim_multiplier=C.MULT, vocab_size=C.VOCAB, dropout=0.0)
    m = bdh_model.BDH(cfg)
    sd = m.state_dict()
    for k, v in C.make_weights().items():
        assert tuple(sd[k].shape) == v.shape, k
        sd[k] = torch.from_numpy(v)
    m.load_state_dict(sd)
    m = m.to(DEV).eval()
    m.attn._attn_impl_override = impl
    return m


def _reference_ops(m, idx):
    """The reference model's eval forward as torch ops, call for call (bdh.py:947-1072 with
    the default eager attention): encoder by F.linear on the (nh*N, D) weight
    (bdh.py:861-889), RoPE with fp32 tables and bf16 products (kernels/rope.py:108-126),
    ``(QR @ QR.mT).tril_(-1) @ V`` (kernels/attention.py:27-40), encoder_v by einsum
    (bdh.py:914-925), the product and decoder F.linear (bdh.py:927-945), the residual double
    LayerNorm (bdh.py:731-750), the lm_head F.linear. Run under the caller's autocast."""
    from kernels.attention_dispatch import rope_tables
    from kernels.rope import eager_rope_rotate

    B, T = idx.shape
    nh, D = m.config.n_head, m.config.n_embd
    N = m.encoder.size(-1)
    wlin = m.encoder.transpose(1, 2).reshape(nh * N, D).contiguous()
    x = F.layer_norm(m.embed(idx), (D,))
    cos, sin = rope_tables(m.attn.freqs, T, 0, idx.device)
    for _ in range(m.config.n_layer):
        xs = F.relu(F.linear(x, wlin).view(B, T, nh, N))
        qr = eager_rope_rotate(xs.permute(0, 2, 1, 3), cos, sin)
        y = (qr @ qr.mT).tril_(-1) @ x.unsqueeze(1)
        y = F.layer_norm(y, (D,))
        ys = F.relu(torch.einsum("bhtd,hdn->bthn", y, m.encoder_v))
        ym = F.linear((xs * ys).view(B, T, nh * N), m.decoder.transpose(-2, -1))
        z = F.layer_norm(ym, (D,))
        z.add_(x)
        x = F.layer_norm(z, (D,))
    return F.linear(x, m.lm_head.transpose(-2, -1))


def _rel(a, ref):
    return O.rel_fro(a.detach().float().cpu().numpy(), np.asarray(ref, np.float32))


def _sa():
    from kernels import sm100_attn

    return sm100_attn


def test_config2_bf16_logits_match_reference(monkeypatch):
    monkeypatch.delenv("BDH_SM100_LATENT", raising=False)
    monkeypatch.delenv("BDH_SM100_GATE_DEC", raising=False)
    C = config2_case()
    g = golden("config2_bf16")
    m = _model()
    idx = torch.from_numpy(g["idx"]).to(DEV)
    _sa().profile_begin()
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        logits = m(idx)[0]
    torch.cuda.synchronize()
    cnt = {k: v["launches"] for k, v in _sa().profile_end().items()}
    # the fused path ran: one encode and one gate + decoder launch per layer, no separate RoPE
    assert cnt["encode"] == C.N_LAYER and cnt["gate"] == C.N_LAYER and cnt["rope"] == 0, cnt
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        ref_gpu = _reference_ops(m, idx)
    ref = g["logits_bf16_cuda_policy"]
    cpu_floor = reference_bf16_floor(g)
    gpu_floor = _rel(ref_gpu, ref)
    err = _rel(logits, ref)
    print(f"config-2 width bf16 logits vs reference: {err:.3e}; reference floors: CPU "
          f"{cpu_floor:.3e}, its op sequence on this GPU {gpu_floor:.3e}")
    assert gpu_floor < 1e-2  # the reference's own chain on this GPU (sanity)
    assert err <= max(3e-3, cpu_floor, 1.1 * gpu_floor)
    assert _sa().device_error() == 0
    # this build's eager model path issues the same calls: the same bits
    m.attn._attn_impl_override = "eager"
    monkeypatch.setenv("BDH_SM100_LATENT", "0")
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        eager = m(idx)[0]
    assert torch.equal(eager, ref_gpu)


def test_config2_bf16_layers_teacher_forced_match_reference(monkeypatch):
    """Each fused layer fed the reference's residual stream: its attention output and its
    output stream against the reference's, within 3e-3."""
    monkeypatch.delenv("BDH_SM100_GATE_DEC", raising=False)
    C = config2_case()
    g = golden("config2_bf16")
    m = _model()
    sa = _sa()
    for layer in range(C.N_LAYER):
        x_in = torch.from_numpy(g[f"layer_in_l{layer}"]).to(DEV)
        with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16), \
                sa.score_terms_scope("bf16"):
            x_out, _ = m._layer_latent(x_in, None, layer, 0, None)
            xb = x_in.to(torch.bfloat16)
            _, qr = sa.latent_encode(xb, m._bf16_param("encoder", True), m.attn.freqs, 0)
            y = sa.tril_score_v(qr, qr, xb.unsqueeze(1))
        y_ref = C.bf16_bits_to_f32(g[f"attn_out_bf16_bits_cuda_policy_l{layer}"])
        ey, ex = _rel(y, y_ref), _rel(x_out, g[f"layer_out_l{layer}"])
        print(f"layer {layer}: attention {ey:.3e}, output stream {ex:.3e}")
        assert ey < 3e-3 and ex < 3e-3


def test_config2_full_batch_bf16_logits_match_reference_ops_on_gpu(monkeypatch):
    """Config 2's batch (B = 32, T = 512) through 2 layers: the fused model against the
    reference's op sequence on this GPU, within 3e-3."""
    monkeypatch.delenv("BDH_SM100_LATENT", raising=False)
    monkeypatch.delenv("BDH_SM100_GATE_DEC", raising=False)
    m = _model()
    idx = torch.randint(0, 256, (32, 512), generator=torch.Generator().manual_seed(1002)).to(DEV)
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        logits = m(idx)[0].float()
        ref = _reference_ops(m, idx).float()
    err = ((logits - ref).norm() / ref.norm()).item()
    print(f"config-2 batch, 2 layers, bf16 logits vs the reference's ops on the GPU: {err:.3e}")
    assert err <= 3e-3


def test_config2_fp32_logits_match_reference():
    g = golden("config2_bf16")
    m = _model()
    idx = torch.from_numpy(g["idx"]).to(DEV)
    with torch.no_grad():
        logits = m(idx)[0]
    err = _rel(logits, g["logits_f32"])
    print(f"config-2 width fp32 logits vs reference: {err:.3e}")
    assert err <= 1e-5
