"""The fp8 key-cache wire format on the CPU: the oracle's e4m3 rounding pinned against torch's
float8_e4m3fn cast (an independent implementation of the same OCP E4M3 round-to-nearest-even),
the cache's torch quantizer against the oracle, and the cache bookkeeping of an eager model."""

import numpy as np
import pytest
import torch

import tril_oracle as O


def test_e4m3_rounding_matches_torch_float8():
    rng = np.random.default_rng(7)
    edge = np.array([448, 448.0001, 460, 463.9, 464, 1.0625, 1.1875, 17, 19, 2 ** -9,
                     3 * 2 ** -10, 2 ** -10, -(2 ** -10), -3 * 2 ** -10, 0, -0.0, 2 ** -6,
                     2 ** -6 * 1.0625, 0.015625 * 1.5, 240, 248, 256, 272], np.float32)
    y = np.concatenate([rng.standard_normal(200000).astype(np.float32) * 60,
                        rng.standard_normal(20000).astype(np.float32) * 0.005, edge, -edge])
    y = np.clip(y, -464, 464).astype(np.float32)  # torch's cast is NaN above 464 (no satfinite)
    ours = O.e4m3_rne(y)
    theirs = torch.from_numpy(y).to(torch.float8_e4m3fn).float().numpy()
    assert np.array_equal(ours, theirs)
    # saturation beyond the largest finite value
    assert O.e4m3_rne(np.array([500.0, -1e6], np.float32)).tolist() == [448.0, -448.0]


def test_cache_quantizer_matches_oracle():
    from bdh_cache import quantize_rows_fp8_torch

    g = torch.Generator().manual_seed(3)
    x = torch.randn(2, 3, 5, 130, generator=g) * torch.rand(2, 3, 5, 1, generator=g) * 50
    x[0, 1, 2] = 0.0  # an all-zero row: scale 0, bytes 0
    q, sc = quantize_rows_fp8_torch(x)
    q_o, sc_o = O.quantize_rows_fp8(x.numpy())
    assert np.array_equal(q.float().numpy(), q_o)
    assert np.array_equal(sc.numpy(), sc_o)
    assert float(sc[0, 1, 2]) == 0.0 and bool((q[0, 1, 2].float() == 0).all())
    # the dequantized rows are within e4m3's half-ulp (2^-4 relative at the row maximum)
    deq = q.float() * sc.unsqueeze(-1)
    err = (deq - x).abs().amax(-1) / x.abs().amax(-1).clamp_min(1e-30)
    assert float(err.max()) <= 2 ** -4 + 1e-6


def test_fp8_cache_eager_model_on_cpu():
    import bdh_model
    from bdh_cache import CacheManager

    cfg = bdh_model.BDHConfig(n_layer=2, n_embd=64, n_head=2, mlp_internal_dim_multiplier=16,
                              vocab_size=256, dropout=0.0)
    torch.manual_seed(0)
    m = bdh_model.BDH(cfg).eval()
    m.attn._attn_impl_override = "eager"
    idx = torch.randint(0, 256, (2, 40), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        full, _ = m(idx)
        cache = CacheManager.from_config(cfg, 2, 40, "cpu", storage_dtype=torch.float8_e4m3fn)
        assert cache.kr_fp8 and cache._kr_buf.dtype == torch.float8_e4m3fn
        assert cache._v_buf.dtype == torch.bfloat16 and cache._kr_scale.shape == (2, 2, 2, 40)
        lg, _ = m(idx[:, :32], cache=cache)
        steps = [lg[:, -1]]
        for t in range(32, 40):
            lg, _ = m(idx[:, t:t + 1], cache=cache)
            steps.append(lg[:, -1])
    got = torch.stack(steps, 1)
    ref = full[:, 31:40]
    assert cache.seq_len == 40
    assert ((got - ref).norm() / ref.norm()).item() < 1e-2
    # the cached rows are the quantized rotated keys: dequantization undoes them to e4m3 accuracy
    kr, _ = cache.get_past(0)
    assert kr.dtype == torch.float32 and kr.shape == (2, 2, 40, cfg.mlp_internal_dim_multiplier * 64 // 2)
