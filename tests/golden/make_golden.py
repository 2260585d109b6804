"""Generate the golden fixtures under tests/golden/ by running the REFERENCE implementation.

Run in the build container (the reference checkout is not available on GPU hosts):

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py <reference checkout>

(default: the ``BDH_REFERENCE`` environment variable, else the ``reference_path`` of
BASELINE.json, as oracle/build_ref.py resolves it; ``--config2-only`` / ``--latent-only`` /
``--generate-only`` / ``--train-only`` rewrite one fixture)

It imports the reference's own Python modules (``bdh``, ``bdh_baseline``, ``bdh_cache``,
``kernels``) and its CPU extension built by ``oracle/build_ref.py`` (``csrc/tril_attn_cpu.cpp``),
runs them on small seeded inputs and stores inputs + outputs as .npz files. The tests pin the
numpy oracle (oracle/tril_oracle.py) and the GPU kernels against these files.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent


def _f32(t):
    return t.detach().to("cpu").float().numpy()


def main(reference: Path) -> None:
    sys.path.insert(0, str(reference))
    sys.path.insert(0, str(REPO / "oracle"))
    import torch

    import bdh  # reference optimized model
    import bdh_baseline  # reference frozen upstream model
    from bdh_cache import CacheManager
    from kernels.attention_bwd import StrictTrilSelfAttnFn, analytic_tril_attn_backward
    from kernels.cuda_attn import tril_decode_ref, tril_score_v_ref

    import build_ref

    ext = build_ref.load_module()
    torch.manual_seed(0)

    # ------------------------------------------------------------------ RoPE
    rope = {}
    for n in (64, 256, 8192):
        rope[f"freqs_{n}"] = bdh.get_freqs(n, theta=2 ** 16, dtype=torch.float32).numpy()
    cfg = bdh.BDHConfig(n_layer=1, n_embd=32, n_head=2, mlp_internal_dim_multiplier=4, dropout=0.0)
    att = bdh.Attention(cfg)  # N = 64
    g = torch.Generator().manual_seed(1)
    x = torch.relu(torch.randn(2, 3, 17, 64, generator=g))
    rope["x"] = x.numpy()
    for pos0 in (0, 37, 4000):
        cs = att.rope_cos_sin(17, pos0, torch.device("cpu"))
        rope[f"y_f32_pos{pos0}"] = _f32(att.rope(None, x, cos_sin=cs))
        xb = x.to(torch.bfloat16)
        rope[f"y_bf16_pos{pos0}"] = _f32(att.rope(None, xb, cos_sin=cs))
    np.savez_compressed(HERE / "golden_rope.npz", **rope)

    # --------------------------------------------------------------- forward
    fwd = {}
    g = torch.Generator().manual_seed(2)

    def case(name, B, H, Hv, T, N, D, dtype=torch.float32, distinct_k=False):
        q = torch.relu(torch.randn(B, H, T, N, generator=g)).to(dtype)
        k = torch.relu(torch.randn(B, H, T, N, generator=g)).to(dtype) if distinct_k else q
        v = torch.randn(B, Hv, T, D, generator=g).to(dtype)
        fwd[f"{name}_q"] = _f32(q)
        if distinct_k:
            fwd[f"{name}_k"] = _f32(k)
        fwd[f"{name}_v"] = _f32(v)
        fwd[f"{name}_out_ext"] = _f32(ext.tril_score_v_cpu(q, k, v))  # csrc/tril_attn_cpu.cpp
        fwd[f"{name}_out_ref"] = _f32(tril_score_v_ref(q.float(), k.float(), v.float()))

    case("shared_v", 2, 3, 1, 130, 64, 32)
    case("per_head_v", 2, 3, 3, 130, 64, 32)
    case("t1", 1, 2, 1, 1, 16, 8)
    case("t2", 1, 2, 1, 2, 16, 8)
    case("distinct_k", 1, 2, 1, 40, 16, 8, distinct_k=True)
    case("bf16", 1, 2, 1, 70, 64, 32, dtype=torch.bfloat16)
    case("tiled", 1, 2, 1, 300, 32, 16)  # T*T > 65536: the extension's tiled path
    # baseline Attention.forward (RoPE + tril) on raw latents
    bcfg = bdh_baseline.BDHConfig(n_layer=1, n_embd=32, n_head=2, mlp_internal_dim_multiplier=4)
    batt = bdh_baseline.Attention(bcfg)
    q = torch.relu(torch.randn(1, 2, 50, 64, generator=g))
    v = torch.randn(1, 1, 50, 32, generator=g)
    fwd["baseline_attn_q"] = q.numpy()
    fwd["baseline_attn_v"] = v.numpy()
    fwd["baseline_attn_out"] = _f32(batt(q, q, v))
    fwd["baseline_attn_freqs"] = batt.freqs.reshape(-1).numpy()
    np.savez_compressed(HERE / "golden_fwd.npz", **fwd)

    # ---------------------------------------------------------------- decode
    dec = {}
    g = torch.Generator().manual_seed(3)
    kbuf = torch.randn(2, 2, 40, 64, generator=g)
    vbuf = torch.randn(2, 1, 40, 32, generator=g)
    q = torch.randn(2, 2, 1, 64, generator=g)
    dec["kbuf"], dec["vbuf"], dec["q"] = kbuf.numpy(), vbuf.numpy(), q.numpy()
    for S in (0, 1, 25):
        kp, vp = kbuf.narrow(2, 0, S), vbuf.narrow(2, 0, S)
        dec[f"out_ext_S{S}"] = _f32(ext.tril_decode_cpu(q, kp, vp))
        dec[f"out_ref_S{S}"] = _f32(tril_decode_ref(q, kp, vp))
    q2 = torch.randn(1, 2, 3, 64, generator=g)  # Tq > 1
    dec["q_tq3"] = q2.numpy()
    dec["out_ext_tq3"] = _f32(ext.tril_decode_cpu(q2, kbuf[:1].narrow(2, 0, 25), vbuf[:1].narrow(2, 0, 25)))
    np.savez_compressed(HERE / "golden_decode.npz", **dec)

    # -------------------------------------------------------------- backward
    bwd = {}
    g = torch.Generator().manual_seed(4)
    Q = torch.randn(1, 2, 24, 16, generator=g, dtype=torch.float64)
    K = torch.randn(1, 2, 24, 16, generator=g, dtype=torch.float64)
    V = torch.randn(1, 1, 24, 8, generator=g, dtype=torch.float64)
    dO = torch.randn(1, 2, 24, 8, generator=g, dtype=torch.float64)
    dQ, dK, dV = analytic_tril_attn_backward(Q, K, V, dO)
    bwd.update(Q=Q.numpy(), K=K.numpy(), V=V.numpy(), dO=dO.numpy(), dQ=dQ.numpy(), dK=dK.numpy(),
               dV=dV.numpy())
    Qs = Q.clone().requires_grad_(True)
    Vs = V.clone().requires_grad_(True)
    out = StrictTrilSelfAttnFn.apply(Qs, Vs, "eager")
    out.backward(dO)
    bwd["self_out"] = out.detach().numpy()
    bwd["self_dQ"] = Qs.grad.numpy()
    bwd["self_dV"] = Vs.grad.numpy()
    np.savez_compressed(HERE / "golden_bwd.npz", **bwd)

    # ----------------------------------------------------------------- model
    mod = {}
    torch.manual_seed(5)
    mcfg = bdh_baseline.BDHConfig(n_layer=2, n_embd=32, n_head=2, mlp_internal_dim_multiplier=4,
                                  dropout=0.0, vocab_size=256)
    base = bdh_baseline.BDH(mcfg).eval()
    for k, v in base.state_dict().items():
        mod[f"w_{k}"] = v.numpy()
    g = torch.Generator().manual_seed(6)
    idx = torch.randint(0, 256, (2, 24), generator=g)
    mod["idx"] = idx.numpy()
    with torch.no_grad():
        mod["logits_baseline"] = _f32(base(idx)[0])
        opt = bdh.BDH(bdh.BDHConfig(**dataclasses_asdict(mcfg))).eval()
        opt.load_state_dict(base.state_dict(), strict=False)
        mod["logits_opt"] = _f32(opt(idx)[0])
        # cached prefill of 16 tokens, then 8 teacher-forced T=1 steps
        cache = CacheManager.from_config(opt.config, batch_size=2, max_seq=24, device="cpu")
        lg, _ = opt(idx[:, :16], cache=cache)
        steps = [_f32(lg[:, -1])]
        for t in range(16, 24):
            lg, _ = opt(idx[:, t:t + 1], cache=cache)
            steps.append(_f32(lg[:, -1]))
        mod["logits_cached_steps"] = np.stack(steps)
    np.savez_compressed(HERE / "golden_model.npz", **mod)
    latent_fixture(bdh, HERE)
    config2_bf16_fixture(bdh, HERE)
    generate_fixture(bdh, HERE)
    train_fixture(bdh_baseline, HERE)
    print("wrote", sorted(p.name for p in HERE.glob("golden_*.npz")))


def latent_fixture(bdh, out_dir: Path) -> None:
    """The two latent projections around the attention, in bf16 as the model runs them:
    BDH._encoder_relu + Attention.rope (bdh.py:861-889, 396-412) and BDH._encoder_v_relu + the
    product of _mlp_merge (bdh.py:914-945)."""
    import torch
    import torch.nn.functional as F

    lat = {}
    cfg = bdh.BDHConfig(n_layer=1, n_embd=32, n_head=2, mlp_internal_dim_multiplier=4, dropout=0.0)
    att = bdh.Attention(cfg)  # N = 64
    g = torch.Generator().manual_seed(7)
    B, T, D, nh, N, pos0 = 2, 20, 32, 2, 64, 37
    x = F.layer_norm(torch.randn(B, T, D, generator=g), (D,)).to(torch.bfloat16)
    enc = (torch.randn(nh, D, N, generator=g) * 0.3).to(torch.bfloat16)
    encv = (torch.randn(nh, D, N, generator=g) * 0.3).to(torch.bfloat16)
    y = F.layer_norm(torch.randn(B, nh, T, D, generator=g), (D,)).to(torch.bfloat16)
    with torch.no_grad():
        xs = bdh.BDH._encoder_relu(x, enc)  # (B,T,nh,N) bf16
        cs = att.rope_cos_sin(T, pos0, torch.device("cpu"))
        qr = att.rope(None, xs.permute(0, 2, 1, 3), cos_sin=cs)  # (B,nh,T,N) bf16
        ys = bdh.BDH._encoder_v_relu(y, encv)  # (B,T,nh,N) bf16
        xy = xs * ys
    lat.update(x=_f32(x), enc=_f32(enc), encv=_f32(encv), y=_f32(y), xs=_f32(xs), qr=_f32(qr),
               ys=_f32(ys), xy=_f32(xy), freqs=att.freqs.reshape(-1).numpy(), pos0=np.int64(pos0))
    np.savez_compressed(out_dir / "golden_latent.npz", **lat)


def config2_bf16_fixture(bdh, out_dir: Path) -> None:
    """The reference model at config-2 width (config2_case.py) under bf16 autocast on the CPU,
    as bdh.py's AMP path runs it (bdh.py:486-500, default eager attention
    ``(QR @ QR.mT).tril_(-1) @ V``, kernels/attention.py:27-40).

    The two autocast device types cast differently: CUDA's autocast runs ``layer_norm`` in fp32
    (fp32 policy) while the CPU's leaves it in its input dtype, so on the CPU the residual stream
    x = LN(x + LN(y_mlp)) (bdh.py:731-750) becomes bf16 after the first layer and on a GPU it
    stays fp32. Two runs are stored: ``*_cpu`` with the stock CPU autocast, and ``*_cuda_policy``
    with CUDA's cast for ``layer_norm`` applied on the CPU (its input cast to fp32 by a
    TorchFunctionMode, what CUDA autocast does for that op); the reference code itself is
    unchanged. For each: logits and the attention output of every layer (bf16, stored as bit
    patterns); for the CUDA policy also the residual stream entering and leaving every layer
    (fp32), and the logits of two other executions of the same run (one thread; ATen's GEMMs),
    whose spread is the reference's own floor. Also the fp32 logits without autocast."""
    import torch
    import torch.nn.functional as F
    from torch.overrides import TorchFunctionMode

    class LayerNormFp32(TorchFunctionMode):
        def __torch_function__(self, func, types, args=(), kwargs=None):
            kwargs = kwargs or {}
            if func is F.layer_norm and args and args[0].dtype in (torch.bfloat16, torch.float16):
                args = (args[0].float(),) + tuple(args[1:])
            return func(*args, **kwargs)

    sys.path.insert(0, str(HERE))
    import config2_case as C

    cfg = bdh.BDHConfig(n_layer=C.N_LAYER, n_embd=C.N_EMBD, n_head=C.N_HEAD,
                        mlp_internal_dim_multiplier=C.MULT, dropout=0.0, vocab_size=C.VOCAB)
    model = bdh.BDH(cfg).eval()
    w = C.make_weights()
    sd = model.state_dict()
    for k, v in w.items():
        assert tuple(sd[k].shape) == v.shape, k
        sd[k] = torch.from_numpy(v)
    model.load_state_dict(sd)
    idx = torch.from_numpy(C.make_idx())
    attn_out = []
    hook = model.attn.register_forward_hook(lambda m, a, o: attn_out.append(o[0].detach().clone()))
    fix = {"idx": idx.numpy()}
    from contextlib import nullcontext

    # the residual stream entering each layer and leaving it (instance-level wrappers of the
    # model's own helpers; the reference code is not changed)
    layer_in, layer_out = [], []
    enc_fwd, res_ln = model._encoder_relu_fwd, model._residual_ln

    def enc_hook(x):
        layer_in.append(x.detach().clone())
        return enc_fwd(x)

    def res_hook(x, y):
        out = res_ln(x, y)
        layer_out.append(out.detach().clone())
        return out

    model._encoder_relu_fwd, model._residual_ln = enc_hook, res_hook
    threads = torch.get_num_threads()
    torch.set_num_threads(8)
    with torch.no_grad():
        for tag, mode in (("cpu", nullcontext()), ("cuda_policy", LayerNormFp32())):
            attn_out.clear()
            layer_in.clear()
            layer_out.clear()
            with mode, torch.autocast(device_type="cpu", dtype=torch.bfloat16):
                logits, _ = model(idx)
            assert len(attn_out) == C.N_LAYER and attn_out[0].dtype == torch.bfloat16
            fix[f"logits_bf16_{tag}"] = _f32(logits)
            for i, a in enumerate(attn_out):
                fix[f"attn_out_bf16_bits_{tag}_l{i}"] = (
                    a.contiguous().view(torch.int16).numpy().view(np.uint16))
            if tag == "cuda_policy":
                for i in range(C.N_LAYER):
                    assert layer_in[i].dtype == torch.float32 and layer_out[i].dtype == torch.float32
                    fix[f"layer_in_l{i}"] = _f32(layer_in[i])
                    fix[f"layer_out_l{i}"] = _f32(layer_out[i])
        # The same reference bf16 run executed differently: one CPU thread, and ATen's own CPU
        # GEMMs instead of oneDNN's. Only the order of the fp32 accumulations inside each GEMM
        # changes; the spread of these logits is the reference's own execution-to-execution floor.
        torch.set_num_threads(1)
        with LayerNormFp32(), torch.autocast(device_type="cpu", dtype=torch.bfloat16):
            fix["logits_bf16_cuda_policy_1thread"] = _f32(model(idx)[0])
        torch.set_num_threads(8)
        with torch.backends.mkldnn.flags(enabled=False), LayerNormFp32(), \
                torch.autocast(device_type="cpu", dtype=torch.bfloat16):
            fix["logits_bf16_cuda_policy_aten_gemm"] = _f32(model(idx)[0])
        hook.remove()
        model._encoder_relu_fwd, model._residual_ln = enc_fwd, res_ln
        logits32, _ = model(idx)
        fix["logits_f32"] = _f32(logits32)
    torch.set_num_threads(threads)
    fix["freqs"] = model.attn.freqs.reshape(-1).numpy()
    np.savez_compressed(out_dir / "golden_config2_bf16.npz", **fix)


GENERATE_CASES = (  # (name, seed, temperature, top_k, cache_dtype, cache_page_size)
    ("plain", 101, 1.0, None, None, None),
    ("temp07", 102, 0.7, None, None, None),
    ("topk5_temp13", 103, 1.3, 5, None, None),
    ("topk300", 104, 1.0, 300, None, None),
    ("fp16_cache", 105, 1.0, None, "float16", None),
    ("paged", 106, 0.9, 20, None, 4),
)


def generate_fixture(bdh, out_dir: Path) -> None:
    """The reference's BDH.generate (bdh.py:1076-1190, sampler :680-728) on a small seeded model:
    for each case torch.manual_seed(seed) and then generate(prompt, 10, ...) on the CPU."""
    import torch

    cfg = bdh.BDHConfig(n_layer=2, n_embd=64, n_head=4, mlp_internal_dim_multiplier=8,
                        dropout=0.0, vocab_size=256)
    torch.manual_seed(41)
    m = bdh.BDH(cfg).eval()
    fix = {f"w_{k}": v.numpy() for k, v in m.state_dict().items()}
    prompt = torch.randint(0, 256, (2, 6), generator=torch.Generator().manual_seed(42))
    fix["prompt"] = prompt.numpy()
    for name, seed, temp, top_k, cdt, page in GENERATE_CASES:
        torch.manual_seed(seed)
        out = m.generate(prompt.clone(), 10, temperature=temp, top_k=top_k,
                         cache_dtype=getattr(torch, cdt) if cdt else None, cache_page_size=page)
        fix[f"tokens_{name}"] = out.numpy()
    np.savez_compressed(out_dir / "golden_generate.npz", **fix)


def train_fixture(bdh_baseline, out_dir: Path) -> None:
    """One training step's numbers from the reference's upstream model (bdh_baseline.BDH,
    bdh_baseline.py:97-139, dropout 0): logits, the cross-entropy loss and the gradient of every
    parameter, on a small seeded model and batch (fp32, CPU)."""
    import torch

    cfg = bdh_baseline.BDHConfig(n_layer=2, n_embd=64, n_head=4, mlp_internal_dim_multiplier=8,
                                 dropout=0.0, vocab_size=256)
    torch.manual_seed(61)
    m = bdh_baseline.BDH(cfg)
    fix = {f"w_{k}": v.detach().numpy().copy() for k, v in m.state_dict().items()}
    g = torch.Generator().manual_seed(62)
    idx = torch.randint(0, 256, (3, 40), generator=g)
    tgt = torch.randint(0, 256, (3, 40), generator=g)
    logits, loss = m(idx, tgt)
    loss.backward()
    fix.update(idx=idx.numpy(), targets=tgt.numpy(), logits=_f32(logits), loss=np.float64(loss.item()))
    for k, p in m.named_parameters():
        fix[f"grad_{k}"] = _f32(p.grad)
    np.savez_compressed(out_dir / "golden_train.npz", **fix)


def dataclasses_asdict(c):
    import dataclasses

    return dataclasses.asdict(c)


if __name__ == "__main__":
    if len(sys.argv) > 1 and not sys.argv[1].startswith("--"):
        ref = Path(sys.argv[1])
    else:
        sys.path.insert(0, str(HERE.parent.parent / "oracle"))
        import build_ref

        ref = build_ref.reference_root()
        if ref is None:
            sys.exit("no reference checkout: pass its path or set BDH_REFERENCE")
    only = [a for a in sys.argv[1:] if a in ("--latent-only", "--config2-only", "--generate-only",
                                             "--train-only")]
    if only:
        sys.path.insert(0, str(ref))
        import bdh as _bdh
        import bdh_baseline as _bdh_baseline

        {"--latent-only": lambda: latent_fixture(_bdh, HERE),
         "--config2-only": lambda: config2_bf16_fixture(_bdh, HERE),
         "--generate-only": lambda: generate_fixture(_bdh, HERE),
         "--train-only": lambda: train_fixture(_bdh_baseline, HERE)}[only[0]]()
    else:
        main(ref)
