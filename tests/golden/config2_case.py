"""The config-2-width model case shared by the golden generator and the GPU parity tests.

BASELINE config 2 is the BDH prefill at n_embd = 256, n_head = 4, N = 8192 latent columns per
head (mlp_internal_dim_multiplier = 128), vocab 256, under bf16 autocast. The fixture
``golden_config2_bf16.npz`` holds what the REFERENCE model (``bdh.BDH``) computes for this
case on the CPU; the weights are not stored (about 100 MB) but rebuilt here from a seeded
numpy generator, which gives the same values on every machine. Parameter names and shapes are
the reference's ``state_dict`` (bdh.py:517-563); every weight is N(0, 0.02) as its
initialisation draws them, the RoPE frequencies are the model's own buffer.
"""

from __future__ import annotations

import numpy as np

N_LAYER = 2
N_EMBD = 256
N_HEAD = 4
MULT = 128
VOCAB = 256
BATCH = 2
SEQ = 128
SEED = 2026


def latent_width() -> int:
    return N_EMBD * MULT // N_HEAD


def make_weights() -> dict:
    """float32 arrays keyed by the reference's parameter names (no RoPE buffer)."""
    rng = np.random.default_rng(SEED)
    N, D, nh = latent_width(), N_EMBD, N_HEAD

    def normal(*shape):
        return (rng.standard_normal(shape, dtype=np.float32) * np.float32(0.02)).astype(np.float32)

    return {
        "decoder": normal(nh * N, D),
        "encoder": normal(nh, D, N),
        "encoder_v": normal(nh, D, N),
        "lm_head": normal(D, VOCAB),
        "embed.weight": normal(VOCAB, D),
    }


def make_idx() -> np.ndarray:
    rng = np.random.default_rng(SEED + 1)
    return rng.integers(0, VOCAB, size=(BATCH, SEQ), dtype=np.int64)


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)
