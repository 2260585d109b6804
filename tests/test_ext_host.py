"""bdh_sm100_ext, the PyTorch extension over the C-ABI, on a CPU-only host: it builds in-tree,
imports, carries the reference module's exports (csrc/tril_attn_bind.cpp:25-40: tril_score_v,
tril_decode, has_cuda) and the new ops, binds the library of this ABI, and rejects what the
reference's C++ module rejects with RuntimeError (TORCH_CHECK) before any launch: bad shapes,
CPU tensors (no CPU path), unsupported dtypes."""

import pytest
import torch


@pytest.fixture(scope="module")
def ext():
    import build_lib
    from kernels import sm100_ext

    build_lib.build_ext()
    return sm100_ext.load_ext()


def test_exports_the_reference_module_names(ext):
    for name in ("tril_score_v", "tril_decode", "tril_score_v_bwd", "rope_rotate",
                 "rope_tril_score_v", "rope_tril_decode", "abi_version"):
        assert callable(getattr(ext, name)), name
    assert ext.has_cuda is True
    from kernels import sm100_attn

    assert ext.abi_version() == sm100_attn.ABI_VERSION


def test_shape_errors_raise_runtime_error(ext):
    z = torch.zeros
    with pytest.raises(RuntimeError, match="q and k shapes must match"):
        ext.tril_score_v(z(1, 1, 4, 8), z(1, 1, 5, 8), z(1, 1, 4, 8))
    with pytest.raises(RuntimeError, match="v heads must equal q heads or 1"):
        ext.tril_score_v(z(1, 2, 4, 8), z(1, 2, 4, 8), z(1, 3, 4, 8))
    with pytest.raises(RuntimeError, match="must be 4D"):
        ext.tril_score_v(z(1, 4, 8), z(1, 4, 8), z(1, 4, 8))
    with pytest.raises(RuntimeError, match="incompatible with k_past S=3"):
        ext.tril_decode(z(1, 1, 1, 8), z(1, 1, 3, 8), z(1, 1, 2, 4))
    with pytest.raises(RuntimeError, match="k_past shape"):
        ext.tril_decode(z(1, 1, 1, 8), z(1, 2, 3, 8), z(1, 1, 3, 4))
    with pytest.raises(RuntimeError, match="RoPE last dim must be even, got 7"):
        ext.rope_rotate(z(1, 1, 4, 7), z(7))


def test_cpu_tensors_are_rejected_not_computed(ext):
    z = torch.zeros
    with pytest.raises(RuntimeError, match="requires CUDA tensors"):
        ext.tril_score_v(z(1, 1, 4, 8), z(1, 1, 4, 8), z(1, 1, 4, 8))
    with pytest.raises(RuntimeError, match="requires CUDA tensors"):
        ext.tril_decode(z(1, 1, 1, 8), z(1, 1, 3, 8), z(1, 1, 3, 4))
    with pytest.raises(RuntimeError, match="requires CUDA tensors"):
        ext.tril_score_v_bwd(z(1, 1, 4, 8), z(1, 1, 4, 8), z(1, 1, 4, 8), z(1, 1, 4, 8))
    with pytest.raises(RuntimeError, match="requires CUDA tensors"):
        ext.rope_tril_score_v(z(1, 1, 4, 8), z(1, 1, 4, 8), z(8))


def test_cuda_attn_keeps_the_reference_value_errors(ext):
    """kernels.cuda_attn validates with the reference wrapper's ValueError messages
    (kernels/cuda_attn.py:103-131) before the native call."""
    from kernels import cuda_attn

    z = torch.zeros
    with pytest.raises(ValueError, match="q and k shapes must match"):
        cuda_attn.tril_score_v(z(1, 1, 4, 8), z(1, 1, 5, 8), z(1, 1, 4, 8))
    with pytest.raises(ValueError, match="v_past heads must equal q heads or 1"):
        cuda_attn.tril_decode(z(1, 2, 1, 8), z(1, 2, 3, 8), z(1, 3, 3, 4))
    assert "binding=bdh_sm100_ext" in cuda_attn.ext_status()


def test_fused_layer_ops_exported_and_checked(ext):
    for name in ("latent_encode", "latent_gate_dec", "layer_norm", "residual_layer_norm"):
        assert callable(getattr(ext, name)), name
    z = torch.zeros
    with pytest.raises(RuntimeError, match="latent_encode expects x"):
        ext.latent_encode(z(2, 8, 16), z(4, 32, 64), z(64))
    with pytest.raises(RuntimeError, match="requires CUDA tensors"):
        ext.latent_gate_dec(z(1, 4, 8, 256), z(4, 256, 128), z(1, 8, 4, 128), z(512, 256))
    with pytest.raises(RuntimeError, match="x must be fp32"):
        ext.residual_layer_norm(z(4, 8).bfloat16(), z(4, 8))
    from kernels import sm100_ext

    assert sm100_ext.model_ops() is ext
