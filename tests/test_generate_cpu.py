"""BDH.generate against the reference's own generate (tests/golden/golden_generate.npz, made by
tests/golden/make_golden.py running the reference's bdh.BDH.generate, bdh.py:1076-1190): the
same weights, prompt and seed give the same tokens, for plain sampling, a temperature, top-k
below and above the vocabulary size, an fp16-stored cache and a paged cache (eager path, CPU)."""

import numpy as np
import pytest
import torch

import bdh_model

CASES = (  # (name, seed, temperature, top_k, cache_dtype, cache_page_size), as the fixture made
    ("plain", 101, 1.0, None, None, None),
    ("temp07", 102, 0.7, None, None, None),
    ("topk5_temp13", 103, 1.3, 5, None, None),
    ("topk300", 104, 1.0, 300, None, None),
    ("fp16_cache", 105, 1.0, None, torch.float16, None),
    ("paged", 106, 0.9, 20, None, 4),
)


@pytest.fixture(scope="module")
def model_and_golden():
    from conftest import golden

    g = golden("generate")
    cfg = bdh_model.BDHConfig(n_layer=2, n_embd=64, n_head=4, mlp_internal_dim_multiplier=8,
                              dropout=0.0, vocab_size=256)
    m = bdh_model.BDH(cfg)
    sd = {k[2:]: torch.from_numpy(g[k]) for k in g.files if k.startswith("w_")}
    missing, unexpected = m.load_state_dict(sd, strict=False)
    assert not missing and not unexpected, (missing, unexpected)
    return m.eval(), g


@pytest.mark.parametrize("name,seed,temp,top_k,cdt,page", CASES)
def test_generate_matches_reference_tokens(model_and_golden, monkeypatch, name, seed, temp, top_k,
                                           cdt, page):
    monkeypatch.setenv("BDH_ATTN_IMPL", "eager")
    m, g = model_and_golden
    prompt = torch.from_numpy(g["prompt"])
    torch.manual_seed(seed)
    out = m.generate(prompt.clone(), 10, temperature=temp, top_k=top_k, cache_dtype=cdt,
                     cache_page_size=page)
    np.testing.assert_array_equal(out.numpy(), g[f"tokens_{name}"])


def test_generate_restores_training_mode(model_and_golden):
    m, g = model_and_golden
    m.train()
    m.generate(torch.from_numpy(g["prompt"]), 2)
    assert m.training
    m.eval()
