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
