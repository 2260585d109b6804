"""CacheManager and cached decode on the CPU (eager path): the reference's packed-cache
contracts (tests/test_cache_pack.py, tests/test_attention_mask.py:56-110), restated for this
package's bdh_cache.CacheManager and bdh_model.BDH. The layout, the reserve / append / stage /
commit bookkeeping, overflow, and the geometric paging are the decode interface the native
kernels read, so they are held to the reference's numbers."""

import pytest
import torch

import bdh_model
from bdh_cache import CacheManager


@pytest.fixture(autouse=True)
def _eager(monkeypatch):
    monkeypatch.setenv("BDH_ATTN_IMPL", "eager")


def _cfg(**kw) -> bdh_model.BDHConfig:
    d = dict(n_layer=2, n_embd=64, n_head=4, mlp_internal_dim_multiplier=8, dropout=0.0,
             vocab_size=256)
    d.update(kw)
    return bdh_model.BDHConfig(**d)


def _model(cfg, seed=0) -> bdh_model.BDH:
    torch.manual_seed(seed)
    return bdh_model.BDH(cfg).eval()


def _N(cfg) -> int:
    return cfg.mlp_internal_dim_multiplier * cfg.n_embd // cfg.n_head


def _fill_tokenwise(cm, cfg, steps, value=0.0):
    for _ in range(steps):
        for level in range(cfg.n_layer):
            cm.append(level, torch.full((1, cfg.n_head, 1, _N(cfg)), value),
                      torch.full((1, 1, 1, cfg.n_embd), value))
        cm.commit()


def test_prealloc_shapes_and_bytes():  # test_cache_pack.py:37-51
    cfg = _cfg()
    B, S = 2, 32
    cm = CacheManager.from_config(cfg, B, S, "cpu")
    assert cm.seq_len == 0 and len(cm._kr) == cfg.n_layer
    assert cm._kr[0].shape == (B, cfg.n_head, S, _N(cfg))
    assert cm._v[0].shape == (B, 1, S, cfg.n_embd)
    assert cm.bytes_allocated == cfg.n_layer * (B * cfg.n_head * S * _N(cfg) * 4 + B * S * cfg.n_embd * 4)


def test_layer_contiguous_packing():  # test_cache_pack.py:235-244
    cm = CacheManager.from_config(_cfg(), 2, 16, "cpu")
    assert cm._kr_buf.ndim == 5 and cm._kr_buf.shape[0] == 2 and cm._v_buf.shape[0] == 2
    assert cm._kr[0].data_ptr() == cm._kr_buf[0].data_ptr()
    assert cm._v[1].untyped_storage().data_ptr() == cm._v_buf.untyped_storage().data_ptr()


def test_append_commit_advances_once():  # test_cache_pack.py:54-69
    cfg = _cfg()
    cm = CacheManager.from_config(cfg, 1, 16, "cpu")
    for level in range(cfg.n_layer):
        cm.append(level, torch.randn(1, cfg.n_head, 3, _N(cfg)), torch.randn(1, 1, 3, cfg.n_embd))
        assert cm.seq_len == 0
    cm.commit()
    kr, v = cm.get_past(0)
    assert cm.seq_len == 3 and kr.shape[2] == 3 and v.shape[2] == 3
    with pytest.raises(RuntimeError, match="inconsistent append T"):
        cm.append(0, torch.randn(1, cfg.n_head, 2, _N(cfg)), torch.randn(1, 1, 2, cfg.n_embd))
        cm.append(1, torch.randn(1, cfg.n_head, 1, _N(cfg)), torch.randn(1, 1, 1, cfg.n_embd))


def test_past_views_share_storage_without_copies():  # test_cache_pack.py:451-480
    cfg = _cfg()
    cm = CacheManager.from_config(cfg, 1, 16, "cpu")
    _fill_tokenwise(cm, cfg, 5, 1.0)
    kr, v = cm.get_past(1)
    assert kr.untyped_storage().data_ptr() == cm._kr_buf.untyped_storage().data_ptr()
    assert not kr.is_contiguous() and kr.stride(2) == _N(cfg)  # capacity-strided view
    dst_kr, dst_v = cm.reserve(1, 1)
    assert dst_kr.untyped_storage().data_ptr() == cm._kr_buf.untyped_storage().data_ptr()


def test_overflow_raises():  # test_cache_pack.py:206-217
    cfg = _cfg()
    cm = CacheManager.from_config(cfg, 1, max_seq=4, device="cpu")
    with pytest.raises(RuntimeError, match="overflow"):
        _model(cfg)(torch.randint(0, 256, (1, 5)), cache=cm)


def test_packed_prefill_and_tokenwise_match_full():  # test_cache_pack.py:72-100
    cfg = _cfg()
    m = _model(cfg, seed=7)
    x = torch.randint(0, 256, (2, 12), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        full, _ = m(x)
        cm = CacheManager.from_config(cfg, 2, 12, "cpu")
        assert torch.allclose(m(x, cache=cm)[0], full, rtol=1e-6, atol=1e-6)
        assert cm.seq_len == 12
        cm = CacheManager.from_config(cfg, 2, 12, "cpu")
        tok = torch.cat([m(x[:, t:t + 1], cache=cm)[0] for t in range(12)], 1)
    assert torch.allclose(full, tok, rtol=1e-5, atol=1e-5) and cm.seq_len == 12


def test_prefill_then_decode_matches_full():  # test_attention_mask.py:56-80
    cfg = _cfg()
    m = _model(cfg, seed=21)
    x = torch.randint(0, 256, (2, 16), generator=torch.Generator().manual_seed(22))
    with torch.no_grad():
        full, _ = m(x)
        cm = CacheManager.from_config(cfg, 2, 16, "cpu")
        parts = [m(x[:, :10], cache=cm)[0]]
        parts += [m(x[:, t:t + 1], cache=cm)[0] for t in range(10, 16)]
    assert torch.allclose(full, torch.cat(parts, 1), rtol=1e-5, atol=1e-5)


def test_rope_phases_continue_across_cache_steps():  # test_attention_mask.py:83-110
    cfg = _cfg()
    attn = _model(cfg).attn
    B, S, Tn, N = 1, 5, 3, _N(cfg)
    g = torch.Generator().manual_seed(3)
    Q = torch.randn(B, cfg.n_head, S + Tn, N, generator=g)
    V = torch.randn(B, 1, S + Tn, cfg.n_embd, generator=g)
    out_full, kr_full, _ = attn(Q, Q, V)
    q_pre, q_new = Q[:, :, :S], Q[:, :, S:]
    out_pre, kr_pre, v_pre = attn(q_pre, q_pre, V[:, :, :S])
    out_inc, kr_new, _ = attn(q_new, q_new, V[:, :, S:], rope_start=S, past_kr=kr_pre,
                              past_v=v_pre)
    assert torch.allclose(kr_new, kr_full[:, :, S:], rtol=0, atol=1e-6)
    assert torch.allclose(out_inc, out_full[:, :, S:], rtol=1e-5, atol=1e-5)


def test_page_growth_then_decode():  # test_cache_pack.py:247-269
    cfg = _cfg()
    m = _model(cfg, seed=5)
    x = torch.randint(0, 256, (1, 6), generator=torch.Generator().manual_seed(4))
    cm = CacheManager.from_config(cfg, 1, max_seq=16, device="cpu", page_size=4)
    assert cm.capacity == 4
    with torch.no_grad():
        full, _ = m(x)
        tok = torch.cat([m(x[:, t:t + 1], cache=cm)[0] for t in range(6)], 1)
    assert torch.allclose(full, tok, rtol=1e-5, atol=1e-5)
    assert cm.seq_len == 6 and 6 <= cm.capacity <= 16 and cm.n_grows >= 1


def test_paged_capacity_matches_packed_footprint():  # test_cache_pack.py:272-296
    cfg = _cfg()
    cm = CacheManager.from_config(cfg, 1, max_seq=16, device="cpu", page_size=4)
    stride = cfg.n_layer * (cfg.n_head * _N(cfg) + cfg.n_embd) * 4
    assert cm.capacity == 4 and cm.bytes_allocated == 4 * stride
    _fill_tokenwise(cm, cfg, 16)
    assert cm.capacity == 16 and cm.bytes_allocated == 16 * stride


def test_geometric_growth_fewer_grows_than_linear():  # test_cache_pack.py:483-513
    cfg = _cfg()
    page, S = 16, 512
    cm = CacheManager.from_config(cfg, 1, max_seq=S, device="cpu", page_size=page)
    _fill_tokenwise(cm, cfg, S)
    assert cm.seq_len == S and cm.capacity == S
    linear = S // page - 1
    assert cm.n_grows < linear // 2 and cm.n_grows <= 6  # 16 -> 32 -> ... -> 512
    stride = cfg.n_layer * (cfg.n_head * _N(cfg) + cfg.n_embd) * 4
    assert cm.bytes_copied_on_grow < stride * page * (linear * (linear + 1) // 2) // 2


def test_ensure_capacity_single_grow():  # test_cache_pack.py:516-537
    cfg = _cfg()
    cm = CacheManager.from_config(cfg, 1, max_seq=256, device="cpu", page_size=8)
    cm.ensure_capacity(200)
    assert cm.n_grows == 1 and 200 <= cm.capacity <= 256
    _fill_tokenwise(cm, cfg, 200)
    assert cm.n_grows == 1 and cm.seq_len == 200


def test_reserve_and_stage_across_page_grow():  # test_cache_pack.py:540-590
    cfg = _cfg()
    N = _N(cfg)
    cm = CacheManager.from_config(cfg, 1, max_seq=64, device="cpu", page_size=4)
    for level in range(cfg.n_layer):
        cm.append(level, torch.full((1, cfg.n_head, 4, N), 1.0), torch.full((1, 1, 4, cfg.n_embd), 2.0))
    cm.commit()
    for level in range(cfg.n_layer):  # needs slot 5: grows
        dst_kr, dst_v = cm.reserve(level, 1)
        dst_kr.fill_(3.0)
        dst_v.fill_(4.0)
    cm.commit()
    assert cm.n_grows >= 1 and cm.capacity >= 5
    kr, v = cm.get_past(0)
    assert kr.shape[2] == 5
    assert torch.all(kr[:, :, :4] == 1.0) and torch.all(kr[:, :, 4:] == 3.0)
    assert torch.all(v[:, :, :4] == 2.0) and torch.all(v[:, :, 4:] == 4.0)
    new_kr = torch.full((1, cfg.n_head, 3, N), 5.0)
    all_kr, all_v = cm.stage(0, new_kr, torch.full((1, 1, 3, cfg.n_embd), 6.0))
    for level in range(1, cfg.n_layer):
        cm.stage(level, torch.full((1, cfg.n_head, 3, N), 5.0), torch.full((1, 1, 3, cfg.n_embd), 6.0))
    assert all_kr.shape[2] == 8 and torch.equal(all_kr[:, :, 5:], new_kr)
    assert torch.all(all_kr[:, :, :4] == 1.0) and torch.all(all_v[:, :, 5:] == 6.0)
    cm.commit()
    assert cm.seq_len == 8


def test_attention_rope_api_matches_reference_golden():
    """Attention's RoPE members of the reference (bdh.py:119-347): phases_cos_sin / rope (static),
    ensure_rope_table, rope_cos_sin narrowing into the table (the same bits as computing them),
    t1_cis_pairs (paired layout, None without a covering table); the rotation reproduces the
    reference's Attention.rope outputs (tests/golden/golden_rope.npz)."""
    from conftest import golden

    g = golden("rope")
    att = bdh_model.Attention(_cfg(n_layer=1, n_embd=32, n_head=2, mlp_internal_dim_multiplier=4))
    x = torch.from_numpy(g["x"])  # (2, 3, 17, 64)
    for pos0 in (0, 37, 4000):
        fresh = att.rope_cos_sin(17, pos0, torch.device("cpu"))
        y = bdh_model.Attention.rope(None, x, cos_sin=fresh)
        assert torch.allclose(y, torch.from_numpy(g[f"y_f32_pos{pos0}"]), rtol=0, atol=2e-6)
        phases = torch.arange(pos0, pos0 + 17, dtype=torch.float32).view(1, 1, -1, 1) * att.freqs
        assert torch.equal(bdh_model.Attention.rope(phases, x), y)
    assert att.t1_cis_pairs(3, "cpu") is None
    att.ensure_rope_table(64, "cpu")
    cached = att.rope_cos_sin(17, 37, torch.device("cpu"))
    fresh = bdh_model.rope_tables(att.freqs, 17, 37, torch.device("cpu"))
    assert torch.equal(cached[0], fresh[0]) and torch.equal(cached[1], fresh[1])
    cp, sp = att.t1_cis_pairs(37, "cpu")
    assert cp.shape == (1, 1, 1, 32, 2) and torch.equal(cp.reshape(1, 1, 1, 64), fresh[0][:, :, :1])
    assert att.t1_cis_pairs(64, "cpu") is None  # past the table
