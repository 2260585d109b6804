"""The C-ABI library loads on a CPU-only host, exports every symbol include/bdh_sm100.h
declares, and rejects bad arguments on the host side (no kernel is launched)."""

import ctypes
import re

import pytest

from conftest import REPO

HEADER = REPO / "include" / "bdh_sm100.h"


def _declared():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:size_t|int|const char\*)\s+(bdh_\w+)\s*\(", text, re.M)))


def test_header_declares_the_boundary():
    names = _declared()
    for n in ("bdh_tril_score_v", "bdh_tril_decode", "bdh_tril_score_v_bwd", "bdh_rope_rotate",
              "bdh_last_error", "bdh_abi_version"):
        assert n in names


def test_library_exports_every_declared_symbol():
    from kernels import sm100_attn as sa

    lib = sa.load_library()
    for name in _declared():
        assert hasattr(lib, name), f"{name} missing from {sa._LIB_PATH}"
    assert lib.bdh_abi_version() == sa.ABI_VERSION == 9


def test_workspace_queries_are_host_only():
    from kernels import sm100_attn as sa

    lib = sa.load_library()
    B, H, T, N, D = 2, 4, 300, 512, 256
    bf = lib.bdh_tril_score_v_workspace_size(1, B, H, 1, T, N, D, 1)
    ldp = (T + 7) // 8 * 8
    assert bf >= 2 * B * H * T * ldp * 2
    f32 = lib.bdh_tril_score_v_workspace_size(0, B, H, 1, T, N, D, 1)
    assert f32 > 2 * B * H * T * N * 4  # tf32 hi/lo operand copies + score pair
    # split partials (at least ceil(S/128) splits) + the rotated fp32 queries
    dws = lib.bdh_tril_decode_workspace_size(64, 4, 1, 1000, 8192, 256)
    assert dws >= 8 * 64 * 4 * 256 * 4 + 64 * 4 * 8192 * 4
    assert lib.bdh_tril_score_v_bwd_workspace_size(1, B, H, 1, T, N, D, 1) > 0


def _i64x4(*v):
    return (ctypes.c_int64 * 4)(*v)


def test_invalid_arguments_rejected_before_launch():
    from kernels import sm100_attn as sa

    lib = sa.load_library()
    s = _i64x4(4096, 1024, 64, 1)
    # bad dtype
    rc = lib.bdh_tril_score_v(None, s, None, s, None, s, 7, None, s, 1, 1, 1, 1, 16, 64, 64, None, 0, None)
    assert rc == 1 and b"dtype" in lib.bdh_last_error()
    # v heads neither 1 nor H
    rc = lib.bdh_tril_score_v(None, s, None, s, None, s, 1, None, s, 1, 1, 4, 2, 16, 64, 64, None, 0, None)
    assert rc == 1 and b"heads" in lib.bdh_last_error()
    # non-unit last stride
    bad = _i64x4(4096, 1024, 64, 2)
    rc = lib.bdh_tril_score_v(None, bad, None, bad, None, s, 1, None, s, 1, 1, 1, 1, 16, 64, 64, None, 0, None)
    assert rc == 1 and b"contiguous" in lib.bdh_last_error()
    # missing workspace
    rc = lib.bdh_tril_score_v(None, s, None, s, None, s, 1, None, s, 1, 1, 1, 1, 16, 64, 64, None, 0, None)
    assert rc == 3 and b"workspace" in lib.bdh_last_error()
    # odd RoPE width
    rc = lib.bdh_rope_rotate(None, 1, s, None, 1, s, None, None, 1, 1, 4, 63, 0, 0, None)
    assert rc == 1 and b"even" in lib.bdh_last_error()
    # empty problems are a no-op success
    rc = lib.bdh_tril_score_v(None, s, None, s, None, s, 1, None, s, 1, 0, 1, 1, 16, 64, 64, None, 0, None)
    assert rc == 0


def test_build_recipe_targets_sm100a():
    import build_lib

    assert "arch=compute_100a,code=sm_100a" in " ".join(build_lib.ARCH)
    assert "-lineinfo" in build_lib.NVCC_FLAGS


def test_profile_kinds_match_header():
    from kernels import sm100_attn as sa

    m = re.search(r"#define BDH_PROF_KINDS (\d+)", HEADER.read_text())
    assert m and int(m.group(1)) == len(sa.PROF_KINDS)


def test_latent_entry_points_validate_on_host():
    from kernels import sm100_attn as sa

    lib = sa.load_library()
    s3 = (ctypes.c_int64 * 3)(512, 256, 1)
    s4 = _i64x4(4096, 1024, 64, 1)
    # odd latent width (RoPE pairs)
    rc = lib.bdh_latent_encode(None, s3, None, s3, None, s4, None, s4, None, 1, 16, 2, 256, 63, 0, None)
    assert rc == 1 and b"even" in lib.bdh_last_error()
    # a non-contiguous last dimension
    bad = _i64x4(4096, 1024, 64, 2)
    rc = lib.bdh_latent_gate(None, bad, None, s3, None, s4, None, s4, 1, 16, 2, 256, 64, None)
    assert rc == 1 and b"stride" in lib.bdh_last_error()
    # empty problems are a no-op
    assert lib.bdh_latent_encode(None, s3, None, s3, None, s4, None, s4, None, 0, 16, 2, 256, 64, 0, None) == 0
    # the fused gate keeps both weight blocks resident: D <= 256, one weight layout
    w_n = (ctypes.c_int64 * 3)(512 * 64, 64, 1)      # (H, D, N) with n contiguous
    w_d = (ctypes.c_int64 * 3)(512 * 64, 1, 512)     # d contiguous (transposed copy)
    rc = lib.bdh_latent_gate_x(None, s4, None, w_n, None, s3, None, w_n, None, s4,
                               1, 16, 2, 512, 64, None)
    assert rc == 1 and b"256" in lib.bdh_last_error()
    rc = lib.bdh_latent_gate_x(None, s4, None, w_n, None, s3, None, w_d, None, s4,
                               1, 16, 2, 256, 64, None)
    assert rc == 1 and b"same layout" in lib.bdh_last_error()
    rc = lib.bdh_latent_gate_x(None, bad, None, w_n, None, s3, None, w_n, None, s4,
                               1, 16, 2, 256, 64, None)
    assert rc == 1 and b"stride" in lib.bdh_last_error()
    assert lib.bdh_latent_gate_x(None, s4, None, w_n, None, s3, None, w_n, None, s4,
                                 1, 0, 2, 256, 64, None) == 0


def test_gate_dec_entry_point_validates_on_host():
    """bdh_latent_gate_dec: D = 256, N a multiple of 128, d-contiguous encv, latent-contiguous
    decoder; all checked before any device work."""
    from kernels import sm100_attn as sa

    lib = sa.load_library()
    H, N, D = 2, 256, 256
    s4 = (ctypes.c_int64 * 4)(16 * H * N, H * N, N, 1)
    y4 = (ctypes.c_int64 * 4)(H * 16 * D, 16 * D, D, 1)
    s3 = (ctypes.c_int64 * 3)(16 * D, D, 1)
    ev_d = (ctypes.c_int64 * 3)(N * D, 1, D)        # d contiguous (transposed copy)
    ev_n = (ctypes.c_int64 * 3)(N * D, N, 1)        # n contiguous
    dec_k = (ctypes.c_int64 * 2)(1, H * N)           # latent contiguous (transposed copy)
    dec_d = (ctypes.c_int64 * 2)(D, 1)               # d contiguous
    call = lambda *a: lib.bdh_latent_gate_dec(*a)
    rc = call(None, y4, None, ev_d, None, s4, None, dec_k, None, s3, 1, 16, H, 128, N, None)
    assert rc == 1 and b"D = 256" in lib.bdh_last_error()
    rc = call(None, y4, None, ev_d, None, s4, None, dec_k, None, s3, 1, 16, H, D, 192, None)
    assert rc == 1 and b"multiple of 128" in lib.bdh_last_error()
    rc = call(None, y4, None, ev_n, None, s4, None, dec_k, None, s3, 1, 16, H, D, N, None)
    assert rc == 1 and b"d contiguous" in lib.bdh_last_error()
    rc = call(None, y4, None, ev_d, None, s4, None, dec_d, None, s3, 1, 16, H, D, N, None)
    assert rc == 1 and b"latent index contiguous" in lib.bdh_last_error()
    assert call(None, y4, None, ev_d, None, s4, None, dec_k, None, s3, 1, 0, H, D, N, None) == 0


def test_layernorm_entry_points_validate_on_host():
    from kernels import sm100_attn as sa

    lib = sa.load_library()
    rc = lib.bdh_layernorm(None, 1, 12, None, 1, 12, 4, 12, 1e-5, None)
    assert rc == 1 and b"multiple of 8" in lib.bdh_last_error()
    rc = lib.bdh_residual_layernorm(None, 256, None, 7, 256, None, 256, None, 256, 4, 256, 1e-5, None)
    assert rc == 1 and b"dtype" in lib.bdh_last_error()
    assert lib.bdh_layernorm(None, 1, 256, None, 1, 256, 0, 256, 1e-5, None) == 0
