"""Dispatch / flag semantics of the kernels package (reference kernels/attention_dispatch.py,
kernels/rope_dispatch.py, kernels/attention_bwd.py) on CPU."""

import pytest
import torch

import kernels
from kernels import attention_dispatch as ad
from kernels import sm100_attn as sa


def test_default_is_eager():
    assert ad.resolve_attn_impl() == "eager"


@pytest.mark.parametrize("raw,want", [("eager", "eager"), ("cuda_sm100", "cuda_sm100"),
                                      ("CUDA", "cuda_sm100"), (" cuda_sm100 ", "cuda_sm100")])
def test_resolve_names(monkeypatch, raw, want):
    monkeypatch.setenv("BDH_ATTN_IMPL", raw)
    assert ad.resolve_attn_impl() == want
    assert ad.resolve_attn_impl(raw) == want


@pytest.mark.parametrize("raw", ["blocked", "online", "triton"])
def test_removed_backends_raise(raw):
    with pytest.raises(ValueError, match="not provided"):
        ad.resolve_attn_impl(raw)


def test_unknown_backend_raises():
    with pytest.raises(ValueError, match="BDH_ATTN_IMPL must be"):
        ad.resolve_attn_impl("cuBLAS")


def test_auto_thresholds(monkeypatch):
    assert ad.attn_auto_threshold() == 512
    assert ad.attn_auto_cold_threshold() == 512
    monkeypatch.setenv("BDH_ATTN_AUTO_THRESHOLD", "100")
    assert ad.attn_auto_cold_threshold() == 100
    monkeypatch.setenv("BDH_ATTN_AUTO_COLD_THRESHOLD", "7")
    assert ad.attn_auto_cold_threshold() == 7
    monkeypatch.setenv("BDH_ATTN_AUTO_THRESHOLD", "x")
    with pytest.raises(ValueError, match="must be an int"):
        ad.attn_auto_threshold()
    monkeypatch.setenv("BDH_ATTN_AUTO_THRESHOLD", "-1")
    with pytest.raises(ValueError, match=">= 0"):
        ad.attn_auto_threshold()


def test_auto_keeps_cpu_tensors_on_eager(monkeypatch):
    monkeypatch.setenv("BDH_ATTN_AUTO", "1")
    monkeypatch.setenv("BDH_ATTN_AUTO_THRESHOLD", "4")
    q = torch.zeros(1, 1, 8, 4)
    assert ad.resolve_cold_impl(8, probe=q) == "eager"
    assert ad.resolve_decode_impl(8, probe=q) == "eager"
    monkeypatch.setenv("BDH_ATTN_IMPL", "cuda_sm100")
    assert ad.resolve_cold_impl(8, probe=q) == "cuda_sm100"  # explicit impl never overridden


def _rand(*shape, seed=0):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, generator=g)


def test_eager_forward_semantics():
    q = torch.relu(_rand(2, 3, 9, 8))
    v = _rand(2, 1, 9, 4, seed=1)
    out = ad.bdh_attn(q, q, v)
    ref = torch.einsum("bhij,bjd->bhid", (q @ q.mT).tril(-1), v[:, 0])
    torch.testing.assert_close(out, ref)
    assert torch.all(out[:, :, 0] == 0)


def test_eager_decode_semantics_and_empty_past():
    q = _rand(2, 3, 1, 8)
    k = _rand(2, 3, 5, 8, seed=1)
    v = _rand(2, 1, 5, 4, seed=2)
    torch.testing.assert_close(ad.bdh_attn_decode(q, k, v), (q @ k.mT) @ v)
    z = ad.bdh_attn_decode(q, k[:, :, :0], v[:, :, :0])
    assert z.shape == (2, 3, 1, 4) and torch.all(z == 0)


def test_sm100_never_falls_back_to_cpu(monkeypatch):
    q = torch.relu(_rand(1, 1, 4, 8))
    v = _rand(1, 1, 4, 8)
    with pytest.raises(RuntimeError, match="CUDA tensors|not loadable"):
        ad.bdh_attn(q, q, v, impl="cuda_sm100")
    with pytest.raises(RuntimeError, match="CUDA tensors|not loadable"):
        ad.bdh_attn_decode(q[:, :, :1], q, v, impl="cuda_sm100")


class _Unexpected:
    def __getattr__(self, name):
        raise AssertionError(f"native library touched before validation: {name}")


@pytest.mark.parametrize("args,msg", [
    (((1, 2, 3), (1, 2, 3, 4), (1, 1, 3, 4)), "must be 4D"),
    (((1, 2, 3, 4), (1, 2, 5, 4), (1, 1, 3, 4)), "shapes must match"),
    (((1, 2, 3, 4), (1, 2, 3, 4), (2, 1, 3, 4)), "batch/seq must match"),
    (((1, 2, 3, 4), (1, 2, 3, 4), (1, 3, 3, 4)), "heads must equal"),
])
def test_shape_errors_before_native(monkeypatch, args, msg):
    monkeypatch.setattr(sa, "_lib", _Unexpected())
    q, k, v = (torch.zeros(*s) for s in args)
    with pytest.raises(ValueError, match=msg):
        sa.tril_score_v(q, k, v)


@pytest.mark.parametrize("args,msg", [
    (((1, 2, 1, 4), (1, 2, 3), (1, 1, 3, 4)), "must be 4D"),
    (((1, 2, 1, 4), (1, 3, 3, 4), (1, 1, 3, 4)), "incompatible with q"),
    (((1, 2, 1, 4), (1, 2, 3, 4), (1, 1, 5, 4)), "incompatible with k_past"),
    (((1, 2, 1, 4), (1, 2, 3, 4), (1, 3, 3, 4)), "heads must equal"),
])
def test_decode_shape_errors_before_native(monkeypatch, args, msg):
    monkeypatch.setattr(sa, "_lib", _Unexpected())
    q, k, v = (torch.zeros(*s) for s in args)
    with pytest.raises(ValueError, match=msg):
        sa.tril_decode(q, k, v)


def test_autograd_fn_eager_matches_torch_autograd(monkeypatch):
    monkeypatch.setenv("BDH_ATTN_AUTOGRAD", "1")
    q0 = torch.relu(_rand(1, 2, 7, 5)).double()
    v0 = _rand(1, 1, 7, 3, seed=3).double()
    q = q0.clone().requires_grad_(True)
    v = v0.clone().requires_grad_(True)
    out = ad.bdh_attn(q, q, v)
    g = _rand(1, 2, 7, 3, seed=4).double()
    out.backward(g)
    q2 = q0.clone().requires_grad_(True)
    v2 = v0.clone().requires_grad_(True)
    ((q2 @ q2.mT).tril(-1) @ v2).backward(g)
    torch.testing.assert_close(q.grad, q2.grad)
    torch.testing.assert_close(v.grad, v2.grad)


def test_gradcheck_strict_tril_fn():
    q = torch.randn(1, 2, 5, 3, dtype=torch.float64, requires_grad=True)
    k = torch.randn(1, 2, 5, 3, dtype=torch.float64, requires_grad=True)
    v = torch.randn(1, 1, 5, 2, dtype=torch.float64, requires_grad=True)
    assert torch.autograd.gradcheck(lambda a, b, c: kernels.StrictTrilAttnFn.apply(a, b, c, "eager"), (q, k, v))


def test_rope_dispatch_flags(monkeypatch):
    from kernels import rope_dispatch as rd

    assert rd.resolve_rope_impl() == "eager"
    monkeypatch.setenv("BDH_ROPE_IMPL", "fused")
    assert rd.resolve_rope_impl() == "fused"
    with pytest.raises(ValueError):
        rd.resolve_rope_impl("triton")


def test_rope_out_alias_rejected():
    from kernels.rope import eager_rope_rotate

    x = torch.randn(1, 1, 3, 4)
    c = torch.ones(1, 1, 3, 4)
    with pytest.raises(ValueError, match="alias"):
        eager_rope_rotate(x, c, c, out=x)
    with pytest.raises(ValueError, match="even"):
        eager_rope_rotate(torch.randn(1, 1, 3, 5), torch.ones(1, 1, 3, 5), torch.ones(1, 1, 3, 5))


def test_backend_info_reports_native_status():
    info = ad.backend_info()
    assert info["BDH_ATTN_IMPL"] == "eager" and "ext_status" in info


def test_cuda_attn_module_mirrors_reference_names():
    """kernels.cuda_attn keeps the reference module's public names; its eager references work
    on CPU, and the native entry points refuse CPU tensors (no silent fallback)."""
    import numpy as np
    import pytest
    import torch

    import tril_oracle as O
    from conftest import golden
    from kernels import cuda_attn

    for name in ("tril_score_v", "tril_decode", "tril_score_v_ref", "tril_decode_ref",
                 "tril_score_v_tiled_ref", "tril_decode_tiled_ref", "has_cuda_ext",
                 "has_cuda_kernel", "ext_status", "pick_cuda_cold_tiles", "pick_cuda_decode_tile_n"):
        assert callable(getattr(cuda_attn, name)), name
    g = golden("fwd")
    q, v = torch.tensor(g["shared_v_q"]), torch.tensor(g["shared_v_v"])
    out = cuda_attn.tril_score_v_ref(q, q, v)
    np.testing.assert_allclose(out.numpy(), g["shared_v_out_ref"], rtol=1e-5, atol=1e-5)
    d = golden("decode")
    kb, vb, qd = torch.tensor(d["kbuf"]), torch.tensor(d["vbuf"]), torch.tensor(d["q"])
    assert O.rel_fro(cuda_attn.tril_decode_ref(qd, kb[:, :, :25], vb[:, :, :25]).numpy(),
                     d["out_ext_S25"]) < 1e-6
    assert float(cuda_attn.tril_decode_ref(qd, kb[:, :, :0], vb[:, :, :0]).abs().sum()) == 0.0
    with pytest.raises(RuntimeError):
        cuda_attn.tril_score_v(q, q, v)


def test_package_reexports_reference_names():
    """The kernels package re-exports what the reference's kernels/__init__.py does from its
    cuda_attn module (tile constants, tile pickers, CPU references), besides the dispatch, the
    autograd functions and the RoPE dispatch; the blocked and Triton backends stay removed."""
    import kernels

    for name in ("cuda_attn", "CUDA_TILE_M", "CUDA_TILE_N", "CUDA_TILE_M_MAX", "CUDA_TILE_N_MAX",
                 "CUDA_DECODE_TILE_N", "CUDA_DECODE_TILE_N_MAX", "pick_cuda_cold_tiles",
                 "pick_cuda_decode_tile_n", "tril_score_v_ref", "tril_score_v_tiled_ref",
                 "tril_decode_ref", "tril_decode_tiled_ref", "bdh_attn", "bdh_attn_decode",
                 "StrictTrilAttnFn", "StrictTrilSelfAttnFn", "analytic_tril_attn_backward",
                 "bdh_rope_rotate", "bdh_rope_rotate_paired", "resolve_rope_impl"):
        assert hasattr(kernels, name), name
        assert name in kernels.__all__, name
    for removed in ("blocked_tril_attn", "triton_tril_attn", "triton_decode_attn"):
        assert not hasattr(kernels, removed), removed
