"""The model's prefill captured as a CUDA graph (bdh_model.GraphedForward): every native call on
the path is stream-ordered with no host synchronisation, so the captured graph replays the same
kernels and gives the same bits as eager calls, for new inputs on every replay."""

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.mark.parametrize("amp", [torch.bfloat16, None])
def test_graphed_forward_matches_eager_calls(amp):
    import bdh_model

    cfg = bdh_model.BDHConfig(n_layer=2, n_embd=256, n_head=4, mlp_internal_dim_multiplier=128,
                              vocab_size=256, dropout=0.0)
    torch.manual_seed(7)
    m = bdh_model.BDH(cfg).to(DEV).eval()
    m.attn._attn_impl_override = "cuda_sm100"
    B, T = 4, 256
    run = m.graphed_forward(B, T, amp_dtype=amp)
    g = torch.Generator().manual_seed(8)
    for _ in range(2):  # new inputs on each replay
        idx = torch.randint(0, 256, (B, T), generator=g).to(DEV)
        got = run(idx).clone()
        ctx = torch.autocast("cuda", dtype=amp) if amp is not None else torch.autocast("cuda", enabled=False)
        with torch.inference_mode(), ctx:
            want = m(idx)[0]
        torch.cuda.synchronize()
        assert torch.equal(got, want)
    with pytest.raises(ValueError):
        run(torch.zeros(B, T + 1, dtype=torch.long, device=DEV))
    from kernels import sm100_attn

    assert sm100_attn.device_error() == 0


_PLAIN_LAUNCH_SCRIPT = r"""
import os, sys
import torch
sys.path.insert(0, {pkg!r})
import bdh_model
cfg = bdh_model.BDHConfig(n_layer=2, n_embd=256, n_head=4, mlp_internal_dim_multiplier=128,
                          vocab_size=256, dropout=0.0)
torch.manual_seed(7)
m = bdh_model.BDH(cfg).to("cuda").eval()
m.attn._attn_impl_override = "cuda_sm100"
idx = torch.randint(0, 256, (4, 256), generator=torch.Generator().manual_seed(9)).to("cuda")
run = m.graphed_forward(4, 256)
with torch.inference_mode(), torch.autocast("cuda", dtype=torch.bfloat16):
    eager = m(idx)[0]
graphed = run(idx).clone()
torch.save({{"eager": eager.cpu(), "graphed": graphed.cpu()}}, {out!r})
"""


def test_programmatic_launch_gives_the_plain_launch_bits(tmp_path):
    """The tensor-core kernels launch as programmatic dependent launches by default
    (BDH_SM100_PDL): each waits on the device for the previous kernel before touching memory.
    The same model step in a child process with BDH_SM100_PDL=0 (plain launches; the setting is
    read once per process) gives the same logits bit for bit, eager and graphed."""
    import os
    import subprocess
    import sys

    import bdh_model

    pkg = os.path.dirname(bdh_model.__file__)
    out = str(tmp_path / "plain.pt")
    env = dict(os.environ, BDH_SM100_PDL="0")
    subprocess.run([sys.executable, "-c", _PLAIN_LAUNCH_SCRIPT.format(pkg=pkg, out=out)],
                   env=env, check=True, timeout=600)
    plain = torch.load(out)

    cfg = bdh_model.BDHConfig(n_layer=2, n_embd=256, n_head=4, mlp_internal_dim_multiplier=128,
                              vocab_size=256, dropout=0.0)
    torch.manual_seed(7)
    m = bdh_model.BDH(cfg).to(DEV).eval()
    m.attn._attn_impl_override = "cuda_sm100"
    idx = torch.randint(0, 256, (4, 256), generator=torch.Generator().manual_seed(9)).to(DEV)
    run = m.graphed_forward(4, 256)
    with torch.inference_mode(), torch.autocast("cuda", dtype=torch.bfloat16):
        eager = m(idx)[0]
    graphed = run(idx).clone()
    torch.cuda.synchronize()
    assert torch.equal(eager.cpu(), plain["eager"])
    assert torch.equal(graphed.cpu(), plain["graphed"])
    assert torch.equal(eager, graphed)


def test_side_stream_gives_the_default_stream_bits():
    """The native kernels run on the caller's current stream, programmatic launches included:
    the model step issued on a created stream, with the input copied on that stream just before
    it, gives the default stream's logits bit for bit."""
    import bdh_model

    cfg = bdh_model.BDHConfig(n_layer=2, n_embd=256, n_head=4, mlp_internal_dim_multiplier=128,
                              vocab_size=256, dropout=0.0)
    torch.manual_seed(7)
    m = bdh_model.BDH(cfg).to(DEV).eval()
    m.attn._attn_impl_override = "cuda_sm100"
    idx_host = torch.randint(0, 256, (4, 256), generator=torch.Generator().manual_seed(11)).pin_memory()
    with torch.inference_mode(), torch.autocast("cuda", dtype=torch.bfloat16):
        want = m(idx_host.to(DEV))[0]
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    with torch.cuda.stream(s), torch.inference_mode(), torch.autocast("cuda", dtype=torch.bfloat16):
        idx = idx_host.to(DEV, non_blocking=True)
        got = [m(idx)[0] for _ in range(2)]
    s.synchronize()
    assert torch.equal(got[0], want) and torch.equal(got[1], want)
