"""The opt-in recurrent-state cache on the host: bookkeeping, and the model's cached prefill +
decode with a StateCache equal to the key/value history (eager attention, fp32, CPU)."""

import pytest
import torch

import bdh_model
from bdh_cache import CacheManager, StateCache


def _model():
    cfg = bdh_model.BDHConfig(n_layer=2, n_embd=32, n_head=2, mlp_internal_dim_multiplier=4,
                              vocab_size=256, dropout=0.0)
    torch.manual_seed(7)
    m = bdh_model.BDH(cfg).eval()
    m.attn._attn_impl_override = "eager"
    return m


def test_state_cache_bookkeeping():
    c = CacheManager.from_config(_model().config, 2, 10, "cpu", storage_kind="state")
    assert isinstance(c, StateCache) and c.kind == "state"
    assert c.state(1).shape == (2, 2, 64, 32) and c.state(0).dtype == torch.float32
    c.advance(4)
    c.advance(4)
    c.commit()
    assert c.seq_len == 4
    with pytest.raises(RuntimeError):
        c.advance(3)
        c.advance(2)
    c.reset()
    assert c.seq_len == 0 and float(c.state(0).abs().sum()) == 0.0
    c.advance(10)
    c.commit()
    with pytest.raises(RuntimeError):
        c.advance(1)
    with pytest.raises(ValueError):
        CacheManager.from_config(_model().config, 2, 10, "cpu", storage_kind="paged")


def _run(m, idx, kind, P):
    cache = CacheManager.from_config(m.config, idx.size(0), idx.size(1), "cpu", storage_kind=kind)
    out = []
    with torch.no_grad():
        lg, _ = m(idx[:, :P], cache=cache)
        out.append(lg[:, -1])
        for t in range(P, idx.size(1)):
            lg, _ = m(idx[:, t:t + 1], cache=cache)
            out.append(lg[:, -1])
        # a multi-token block continuing a past
    return torch.stack(out), cache


def test_state_cache_decode_equals_history():
    m = _model()
    idx = torch.randint(0, 256, (2, 20), generator=torch.Generator().manual_seed(3))
    kv, ckv = _run(m, idx, "kv", 12)
    st, cst = _run(m, idx, "state", 12)
    assert ckv.seq_len == cst.seq_len == 20
    assert ((st - kv).norm() / kv.norm()).item() < 1e-5
    # the state equals K^T V of the history the kv cache kept
    kr, v = ckv.get_past(0)
    ref = kr.double().transpose(-1, -2) @ v.double().expand(-1, kr.size(1), -1, -1)
    assert ((cst.state(0).double() - ref).norm() / ref.norm()).item() < 1e-6


def test_state_cache_multi_token_blocks():
    m = _model()
    idx = torch.randint(0, 256, (2, 24), generator=torch.Generator().manual_seed(4))
    with torch.no_grad():
        full, _ = m(idx)
        cache = CacheManager.from_config(m.config, 2, 24, "cpu", storage_kind="state")
        a, _ = m(idx[:, :10], cache=cache)
        b, _ = m(idx[:, 10:17], cache=cache)
        c, _ = m(idx[:, 17:], cache=cache)
    got = torch.cat([a, b, c], dim=1)
    assert ((got - full).norm() / full.norm()).item() < 1e-5
