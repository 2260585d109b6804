"""fp16 cache storage with fp32 compute: the reference's CacheManager option
(bdh_cache.py:240-243, get_past upcasts the whole past every step) and its contracts
(tests/test_cache_pack.py:146-200): on a small model the fp16-stored cache keeps the prefill
logits within 1e-4 and the tokenwise decode logits within 2e-4 (max abs) of the fp32-stored
cache. The eager path runs on the CPU; the cuda_sm100 path (the past upcast on the device, then
the native decode kernel, the new keys stored back as fp16) on a GPU."""

import pytest
import torch

import bdh_model
from bdh_cache import CacheManager


def _small_model(seed: int, device) -> bdh_model.BDH:
    cfg = bdh_model.BDHConfig(n_layer=2, n_embd=64, n_head=4, mlp_internal_dim_multiplier=8,
                              dropout=0.0, vocab_size=256)
    torch.manual_seed(seed)
    return bdh_model.BDH(cfg).to(device).eval()


def _fp16_vs_fp32(m, x):
    cfg = m.config
    with torch.inference_mode():
        c32 = CacheManager.from_config(cfg, 1, x.size(1), x.device, storage_dtype=torch.float32)
        c16 = CacheManager.from_config(cfg, 1, x.size(1), x.device, storage_dtype=torch.float16)
        assert c16._kr_buf.dtype == torch.float16 and c16._v_buf.dtype == torch.float16
        prefill = (m(x, cache=c32)[0] - m(x, cache=c16)[0]).abs().max().item()
        c32 = CacheManager.from_config(cfg, 1, x.size(1), x.device, storage_dtype=torch.float32)
        c16 = CacheManager.from_config(cfg, 1, x.size(1), x.device, storage_dtype=torch.float16)
        a, b = [], []
        for s in range(x.size(1)):
            a.append(m(x[:, s:s + 1], cache=c32)[0])
            b.append(m(x[:, s:s + 1], cache=c16)[0])
        tokenwise = (torch.cat(a, 1) - torch.cat(b, 1)).abs().max().item()
    return prefill, tokenwise


def test_fp16_storage_eager_cpu(monkeypatch):
    monkeypatch.setenv("BDH_ATTN_IMPL", "eager")
    m = _small_model(21, "cpu")
    x = torch.randint(0, 256, (1, 16), generator=torch.Generator().manual_seed(5))
    prefill, tokenwise = _fp16_vs_fp32(m, x)
    assert prefill < 1e-4 and tokenwise < 2e-4, (prefill, tokenwise)


@pytest.mark.gpu
def test_fp16_storage_native_decode(monkeypatch):
    from kernels import sm100_attn

    monkeypatch.setenv("BDH_ATTN_IMPL", "cuda_sm100")
    m = _small_model(21, "cuda")
    x = torch.randint(0, 256, (1, 16), generator=torch.Generator().manual_seed(5)).cuda()
    sm100_attn.profile_begin()
    prefill, tokenwise = _fp16_vs_fp32(m, x)
    torch.cuda.synchronize()
    launches = sm100_attn.profile_end()
    assert launches["decode"]["launches"] > 0  # the native decode kernel served the steps
    assert prefill < 1e-4 and tokenwise < 2e-4, (prefill, tokenwise)
    assert sm100_attn.device_error() == 0
