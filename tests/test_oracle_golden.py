"""Pin the numpy oracle to outputs of the reference implementation (tests/golden/*.npz,
generated from the reference sources by tests/golden/make_golden.py)."""

import numpy as np
import pytest

import tril_oracle as O
from conftest import golden


def test_freqs_match_reference():
    g = golden("rope")
    for n in (64, 256, 8192):
        ref = g[f"freqs_{n}"]
        got = O.get_freqs(n)
        # numpy and torch fp32 pow differ by at most one ulp; kernels always receive the
        # model's own freqs buffer, so this only pins the restatement itself.
        np.testing.assert_allclose(got, ref, rtol=3.6e-7, atol=0)


@pytest.mark.parametrize("pos0", [0, 37, 4000])
def test_rope_fp32_matches_reference(pos0):
    g = golden("rope")
    x = g["x"]
    y = O.rope(x, g["freqs_64"], pos0)
    # only the cos/sin implementations differ (numpy vs torch): a few fp32 ulps
    np.testing.assert_allclose(y, g[f"y_f32_pos{pos0}"], rtol=0, atol=2e-6)


@pytest.mark.parametrize("pos0", [0, 37, 4000])
def test_rope_bf16_matches_reference(pos0):
    g = golden("rope")
    xb = O.bf16_round(g["x"])
    y = O.rope(xb, g["freqs_64"], pos0, bf16=True)
    ref = g[f"y_bf16_pos{pos0}"]
    # bit-identical except where a cos/sin ulp flips a bf16 rounding (rare)
    mism = np.mean(y != ref)
    assert mism < 2e-3
    np.testing.assert_allclose(y, ref, rtol=0, atol=2 ** -7 * np.abs(ref).max())


@pytest.mark.parametrize("name", ["shared_v", "per_head_v", "t1", "t2", "distinct_k", "bf16", "tiled"])
def test_forward_matches_reference_extension(name):
    g = golden("fwd")
    q = g[f"{name}_q"]
    k = g[f"{name}_k"] if f"{name}_k" in g else q
    v = g[f"{name}_v"]
    out = O.tril_score_v(q, k, v)
    ext = g[f"{name}_out_ext"]
    tol = 4e-3 if name == "bf16" else 1e-5  # bf16: the extension returns bf16
    assert O.rel_fro(out, ext) <= tol or np.abs(ext).max() == 0
    if name == "t1":
        assert np.all(ext == 0) and np.all(out == 0)
    assert np.all(out[:, :, 0] == 0)  # row 0 attends to nothing
    np.testing.assert_allclose(g[f"{name}_out_ref"], ext, rtol=5e-3 if name == "bf16" else 1e-4, atol=1e-4)


def test_baseline_attention_with_rope():
    g = golden("fwd")
    qr = O.rope(g["baseline_attn_q"], g["baseline_attn_freqs"])
    out = O.tril_score_v(qr, qr, g["baseline_attn_v"])
    assert O.rel_fro(out, g["baseline_attn_out"]) < 1e-5


@pytest.mark.parametrize("S", [0, 1, 25])
def test_decode_matches_reference(S):
    g = golden("decode")
    kp = g["kbuf"][:, :, :S]
    vp = g["vbuf"][:, :, :S]
    out = O.tril_decode(g["q"], kp, vp)
    ref = g[f"out_ext_S{S}"]
    assert out.shape == ref.shape
    if S == 0:
        assert np.all(ref == 0) and np.all(out == 0)
    else:
        assert O.rel_fro(out, ref) < 1e-6


def test_decode_multi_query_rows():
    g = golden("decode")
    out = O.tril_decode(g["q_tq3"], g["kbuf"][:1, :, :25], g["vbuf"][:1, :, :25])
    assert O.rel_fro(out, g["out_ext_tq3"]) < 1e-6


def test_backward_matches_reference_fp64():
    g = golden("bwd")
    dq, dk, dv = O.tril_backward(g["Q"], g["K"], g["V"], g["dO"])
    np.testing.assert_allclose(dq, g["dQ"], rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(dk, g["dK"], rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(dv, g["dV"], rtol=1e-10, atol=1e-12)


def test_self_backward_matches_reference_autograd_fn():
    g = golden("bwd")
    dq, _, dv = O.tril_backward(g["Q"], g["Q"], g["V"], g["dO"], k_is_q=True)
    np.testing.assert_allclose(dq, g["self_dQ"], rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(dv, g["self_dV"], rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(O.tril_score_v(g["Q"], g["Q"], g["V"]), g["self_out"], rtol=1e-10, atol=1e-12)


def test_rope_backward_is_adjoint():
    rng = np.random.default_rng(0)
    f = O.get_freqs(32)
    x = rng.standard_normal((1, 1, 9, 32)).astype(np.float64)
    gy = rng.standard_normal((1, 1, 9, 32))
    c, s = O.rope_cos_sin(f, 9, 3)
    y = np.empty_like(x)
    y[..., 0::2] = x[..., 0::2] * c[:, 0::2] - x[..., 1::2] * s[:, 0::2]
    y[..., 1::2] = x[..., 1::2] * c[:, 1::2] + x[..., 0::2] * s[:, 1::2]
    gx = O.rope_backward(gy, f, 3)
    assert abs(np.sum(gy * y) - np.sum(gx * x)) < 1e-9


def _model_weights(g):
    return dict(embed=g["w_embed.weight"], encoder=g["w_encoder"], encoder_v=g["w_encoder_v"],
                decoder=g["w_decoder"], lm_head=g["w_lm_head"], freqs=g["w_attn.freqs"].reshape(-1))


def test_model_forward_matches_reference_baseline():
    g = golden("model")
    logits = O.bdh_forward(g["idx"], _model_weights(g), n_layer=2, n_head=2)
    assert O.rel_fro(logits, g["logits_baseline"]) < 1e-5
    assert O.rel_fro(g["logits_opt"], g["logits_baseline"]) < 1e-5


def test_latent_encode_matches_reference():
    """Oracle encode (projection, bf16 rounding, ReLU, bf16 RoPE) vs the reference's own
    BDH._encoder_relu + Attention.rope run in bf16 (golden_latent.npz)."""
    g = golden("latent")
    xs, qr = O.latent_encode(g["x"], g["enc"], g["freqs"], int(g["pos0"]))
    # the reference's CPU bf16 GEMM and the float64 oracle may round a few outputs to
    # neighbouring bf16 values; everything else is bit-identical
    assert np.mean(xs != g["xs"]) < 0.01
    assert O.rel_fro(xs, g["xs"]) < 3e-3
    assert np.mean(qr != g["qr"]) < 0.01
    assert O.rel_fro(qr, g["qr"]) < 3e-3
    # given the reference's xs, the rotation is exact
    qr2 = O.rope(np.swapaxes(g["xs"], 1, 2), g["freqs"], int(g["pos0"]), bf16=True)
    assert np.mean(qr2 != g["qr"]) < 1e-3


def test_latent_gate_matches_reference():
    g = golden("latent")
    xy = O.latent_gate(g["y"], g["encv"], g["xs"])
    assert np.mean(xy != g["xy"]) < 0.01
    assert O.rel_fro(xy, g["xy"]) < 3e-3
    # the product itself is one bf16 rounding of an exact fp32 product
    np.testing.assert_array_equal(O.bf16_round(g["xs"] * g["ys"]), g["xy"])


def test_bf16_autocast_oracle_pinned_to_reference_model():
    """The bf16-autocast restatement of the layer has the reference baseline's structure:
    without its bf16 roundings it reproduces the reference logits; with them it stays within
    the bf16 error of those logits."""
    g = golden("model")
    w = _model_weights(g)
    exact = O.bdh_forward_bf16(g["idx"], w, n_layer=2, n_head=2, rounding=False)
    assert O.rel_fro(exact, g["logits_baseline"]) < 1e-5
    rounded = O.bdh_forward_bf16(g["idx"], w, n_layer=2, n_head=2)
    assert O.rel_fro(rounded, g["logits_baseline"]) < 2e-2


def _config2_oracle_weights(g):
    from conftest import config2_case

    w = config2_case().make_weights()
    return {"embed": w["embed.weight"], "encoder": w["encoder"], "encoder_v": w["encoder_v"],
            "decoder": w["decoder"], "lm_head": w["lm_head"], "freqs": g["freqs"]}


def test_bf16_layer_oracle_pinned_to_reference_at_config2_width():
    """Each layer of the bf16-autocast restatement, fed the reference's own residual stream
    (teacher forcing, golden_config2_bf16: bdh.BDH at n_embd 256, 4 heads, N = 8192 under
    autocast with CUDA's layer_norm policy), reproduces that layer's attention output and
    output stream within the bf16 bar. The scores are rounded to bf16 as the reference's eager
    attention rounds them; kept exact, the attention output moves by about the bar."""
    from conftest import config2_case

    C = config2_case()
    g = golden("config2_bf16")
    w = _config2_oracle_weights(g)
    for layer in range(C.N_LAYER):
        x_out, y = O.bdh_layer_bf16(g[f"layer_in_l{layer}"], w, C.N_HEAD)
        y_ref = C.bf16_bits_to_f32(g[f"attn_out_bf16_bits_cuda_policy_l{layer}"])
        assert O.rel_fro(y, y_ref) < 3e-3
        assert O.rel_fro(x_out, g[f"layer_out_l{layer}"]) < 3e-3


def test_bf16_model_oracle_pinned_to_reference_logits_at_config2_width():
    """End to end, every bf16 rounding point of a layer can flip with the fp32 accumulation
    order, and the flips grow through the layers: the reference's own logits move by its
    execution floor (reference_bf16_floor: one thread or ATen's GEMMs instead of oneDNN's;
    about 3e-3 at two layers). The oracle's float64 accumulation is one more such order."""
    from conftest import config2_case, reference_bf16_floor

    C = config2_case()
    g = golden("config2_bf16")
    floor = reference_bf16_floor(g)
    assert 5e-4 < floor < 1e-2
    logits = O.bdh_forward_bf16(g["idx"], _config2_oracle_weights(g), C.N_LAYER, C.N_HEAD)
    assert O.rel_fro(logits, g["logits_bf16_cuda_policy"]) <= max(3e-3, floor)


def test_state_decode_oracle_equals_history_decode():
    """The N x D state form reproduces the reference decode (golden_decode, the reference CPU
    extension's tril_decode_cpu) step by step."""
    g = golden("decode")
    kbuf, vbuf, q = g["kbuf"], g["vbuf"], g["q"]
    # out at past length 25 from a state built over the first 25 keys equals the golden decode
    S25 = O.state_from_history(kbuf[:, :, :25], vbuf[:, :, :25])
    out25, _ = O.state_decode(q, S25, vbuf[:, :, 25:26])
    assert O.rel_fro(out25, g["out_ext_S25"]) < 1e-6
    # stepping the state one key at a time gives the same state as building it at once
    S = O.state_from_history(kbuf[:, :, :1], vbuf[:, :, :1])
    for s in range(1, 25):
        _, S = O.state_decode(kbuf[:, :, s:s + 1], S, vbuf[:, :, s:s + 1])
    assert O.rel_fro(S, S25) < 1e-12


def test_baseline_model_port_pinned_to_reference_logits():
    """The CPU restatement of bdh_baseline.BDH that the timed reference arm runs
    (oracle/baseline_model.py) reproduces the reference's own fp32 logits: the small golden
    model (bdh_baseline.BDH) and the config-2-width model (bdh.BDH without autocast), with the
    attention from the reference's C++ extension where it is built, else in torch."""
    import torch

    import baseline_model as BM
    from conftest import config2_case

    attn = BM.reference_tril_score_v()
    g = golden("model")
    w = {k: torch.from_numpy(np.asarray(v, np.float32)) for k, v in _model_weights(g).items()}
    got = BM.baseline_forward(torch.from_numpy(g["idx"]), w, n_layer=2, n_head=2, attn=attn)
    assert O.rel_fro(got.numpy(), g["logits_baseline"]) < 1e-5
    C = config2_case()
    g2 = golden("config2_bf16")
    w2 = {k: torch.from_numpy(np.asarray(v, np.float32)) for k, v in _config2_oracle_weights(g2).items()}
    got2 = BM.baseline_forward(torch.from_numpy(g2["idx"]), w2, C.N_LAYER, C.N_HEAD, attn=attn)
    assert O.rel_fro(got2.numpy(), g2["logits_f32"]) < 1e-5
