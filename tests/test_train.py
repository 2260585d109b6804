"""One training step of the model against the reference's upstream model
(tests/golden/golden_train.npz, made by tests/golden/make_golden.py from bdh_baseline.BDH,
bdh_baseline.py:97-139, dropout 0): logits, the cross-entropy loss and the gradient of every
parameter. The eager path runs on the CPU; the native path (the fused RoPE + tril attention
with its analytic sm_100a backward under every layer) on a GPU, both at the fp32 bar 1e-5."""

import numpy as np
import pytest
import torch

import bdh_model


def _rel(a: torch.Tensor, ref: np.ndarray) -> float:
    r = torch.from_numpy(ref).double()
    return ((a.detach().double().cpu() - r).norm() / r.norm()).item()


def _step(device: str):
    from conftest import golden

    g = golden("train")
    cfg = bdh_model.BDHConfig(n_layer=2, n_embd=64, n_head=4, mlp_internal_dim_multiplier=8,
                              dropout=0.0, vocab_size=256)
    m = bdh_model.BDH(cfg)
    sd = {k[2:]: torch.from_numpy(g[k]) for k in g.files if k.startswith("w_")}
    missing, unexpected = m.load_state_dict(sd, strict=False)
    assert not missing and not unexpected, (missing, unexpected)
    m = m.to(device).train()
    idx = torch.from_numpy(g["idx"]).to(device)
    tgt = torch.from_numpy(g["targets"]).to(device)
    logits, loss = m(idx, tgt)
    loss.backward()
    return m, g, logits, loss


def _check(m, g, logits, loss):
    assert abs(loss.item() - float(g["loss"])) <= 1e-5 * abs(float(g["loss"]))
    assert _rel(logits, g["logits"]) < 1e-5
    names = [k[5:] for k in g.files if k.startswith("grad_")]
    assert sorted(names) == sorted(n for n, _ in m.named_parameters())
    for n, p in m.named_parameters():
        assert _rel(p.grad, g[f"grad_{n}"]) < 1e-5, n


def test_train_step_matches_reference_cpu(monkeypatch):
    monkeypatch.setenv("BDH_ATTN_IMPL", "eager")
    _check(*_step("cpu"))


@pytest.mark.gpu
@pytest.mark.parametrize("autograd_fn", ["0", "1"])
def test_train_step_matches_reference_native(monkeypatch, autograd_fn):
    from kernels import sm100_attn

    monkeypatch.setenv("BDH_ATTN_IMPL", "cuda_sm100")
    monkeypatch.setenv("BDH_ATTN_AUTOGRAD", autograd_fn)
    sm100_attn.profile_begin()
    m, g, logits, loss = _step("cuda")
    torch.cuda.synchronize()
    launches = sm100_attn.profile_end()
    assert launches["grad_q"]["launches"] > 0  # the native backward ran
    _check(m, g, logits, loss)
    assert sm100_attn.device_error() == 0
