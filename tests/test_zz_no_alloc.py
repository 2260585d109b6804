"""GPU test of bdh_tril_decode_noalloc, the decode entry point that allocates nothing.

It serves callers that cannot hand the library a workspace: processes that reserve all of
their device memory up front, host bindings without a device allocator, loops that must not
risk an allocation's implicit synchronisation. Its scratch is a fixed array inside the
library, shared by every call on a device. The test calls it through the C ABI twice in a
row (different inputs each time, so stale scratch contents would show) and compares each
result with the regular workspace entry point, within the decode tolerance used elsewhere
(fp32 1e-5, bf16 3e-3 relative Frobenius). It also checks the size limit is enforced.

The file name sorts last so that a run stopping at the first failure has run every other
test before this one.
"""

import ctypes

import numpy as np
import pytest
import torch

import tril_oracle as O

pytestmark = pytest.mark.gpu

DEV = "cuda"
_P = ctypes.POINTER(ctypes.c_int64)


def _lib():
    from kernels import sm100_attn

    lib = sm100_attn.load_library()
    f = lib.bdh_tril_decode_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p, _P, ctypes.c_int, ctypes.c_void_p, _P, ctypes.c_void_p, _P,
                  ctypes.c_int, ctypes.c_void_p, _P, ctypes.c_int64, ctypes.c_int64,
                  ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                  ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, _P,
                  ctypes.c_void_p]
    return lib


def _s(t):
    return (ctypes.c_int64 * 4)(*t.stride())


def _code(dt):
    return 0 if dt == torch.float32 else 1


def _noalloc(lib, q, kp, vp, freqs=None, pos=0, slot=None):
    B, H, Tq, N = q.shape
    S, D, Hv = kp.size(2), vp.size(-1), vp.size(1)
    out = torch.empty(B, H, Tq, D, dtype=q.dtype, device=q.device)
    rc = lib.bdh_tril_decode_noalloc(
        q.data_ptr(), _s(q), _code(q.dtype), kp.data_ptr(), _s(kp), vp.data_ptr(), _s(vp),
        _code(kp.dtype), out.data_ptr(), _s(out), B, H, Hv, Tq, S, N, D,
        freqs.data_ptr() if freqs is not None else None, pos,
        slot.data_ptr() if slot is not None else None, _s(slot) if slot is not None else None,
        torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.bdh_last_error().decode()
    return out


def _rel(a, b):
    return O.rel_fro(a.double().cpu().numpy(), b.double().cpu().numpy())


@pytest.mark.parametrize("qdt,kvdt", [(torch.float32, torch.float32), (torch.float32, torch.bfloat16),
                                      (torch.bfloat16, torch.bfloat16)])
def test_noalloc_decode_matches_workspace_entry_on_consecutive_calls(qdt, kvdt):
    from kernels import sm100_attn

    lib = _lib()
    tol = 1e-5 if qdt == torch.float32 else 3e-3
    B, H, cap, N, D = 4, 4, 1024, 2048, 256
    for call, S in enumerate((700, 129)):  # two calls in a row, different sizes and data
        g = torch.Generator(device=DEV).manual_seed(100 + call)
        kbuf = torch.randn(B, H, cap, N, device=DEV, generator=g).to(kvdt)
        vbuf = torch.randn(B, 1, cap, D, device=DEV, generator=g).to(kvdt)
        q = torch.randn(B, H, 1, N, device=DEV, generator=g).to(qdt)
        kp, vp = kbuf.narrow(2, 0, S), vbuf.narrow(2, 0, S)
        ref = sm100_attn.tril_decode(q, kp, vp)  # workspace entry point (bdh_tril_decode)
        out = _noalloc(lib, q, kp, vp)
        torch.cuda.synchronize()
        assert _rel(out, ref) <= tol, f"call {call}"
    assert sm100_attn.device_error() == 0


def test_noalloc_decode_fused_rope_slot_write_twice():
    from kernels import sm100_attn

    lib = _lib()
    B, H, cap, N, D = 2, 4, 256, 512, 128
    f = torch.tensor(O.get_freqs(N), device=DEV)
    for call, S in enumerate((200, 37)):
        kbuf = torch.randn(B, H, cap, N, device=DEV)
        vbuf = torch.randn(B, 1, cap, D, device=DEV)
        kbuf2 = kbuf.clone()
        q = torch.relu(torch.randn(B, H, 1, N, device=DEV))
        ref = sm100_attn.tril_decode(q, kbuf[:, :, :S], vbuf[:, :, :S], freqs=f, pos=S,
                                     kr_slot=kbuf[:, :, S:S + 1])
        out = _noalloc(lib, q, kbuf2[:, :, :S], vbuf[:, :, :S], freqs=f, pos=S,
                       slot=kbuf2[:, :, S:S + 1])
        torch.cuda.synchronize()
        assert _rel(out, ref) <= 1e-5, f"call {call}"
        assert torch.equal(kbuf2[:, :, S:S + 1], kbuf[:, :, S:S + 1])
    assert sm100_attn.device_error() == 0


def test_noalloc_rejects_problems_beyond_the_fixed_scratch():
    lib = _lib()
    s = (ctypes.c_int64 * 4)(0, 0, 0, 1)
    # B*H = 256, Tq = 1, D = 256: 8 MiB holds 32 split partials of 256 x 256 floats, i.e.
    # S <= 32 splits x 128 rows = 4096; S = 4097 does not fit.
    rc = lib.bdh_tril_decode_noalloc(None, s, 0, None, s, None, s, 0, None, s, 64, 4, 1, 1, 4097,
                                     8192, 256, None, 0, None, None, None)
    assert rc == 1
    msg = lib.bdh_last_error().decode()
    assert "scratch" in msg and str(8 << 20) in msg


def test_noalloc_decode_at_the_split_cap_and_multi_query():
    """Sizes that push the plan to its limits, both checked against bdh_tril_decode.

    B*H = 256, D = 256, S = 4000: the fixed scratch holds 32 split partials, so the plan must
    lengthen each split to 128 cached rows (the most a CTA takes) to stay within it. Then a
    block of three queries (Tq = 3), whose partials take three times the room per split.
    """
    from kernels import sm100_attn

    lib = _lib()
    for call, (B, H, Tq, S, N, D, kvdt) in enumerate(((64, 4, 1, 4000, 512, 256, torch.bfloat16),
                                                     (2, 4, 3, 300, 1024, 128, torch.float32))):
        g = torch.Generator(device=DEV).manual_seed(300 + call)
        kp = torch.randn(B, H, S, N, device=DEV, generator=g).to(kvdt)
        vp = torch.randn(B, 1, S, D, device=DEV, generator=g).to(kvdt)
        q = torch.randn(B, H, Tq, N, device=DEV, generator=g)
        ref = sm100_attn.tril_decode(q, kp, vp)
        out = _noalloc(lib, q, kp, vp)
        torch.cuda.synchronize()
        assert _rel(out, ref) <= 1e-5, f"case {call}"
    assert sm100_attn.device_error() == 0
