"""The allocation-free flash-attention backward (C symbol dmad_flash_attn_bwd_noalloc).

It exists for host programs that own all device memory through their own pool and
cannot let a library call cudaMalloc (see csrc/flash_bwd_noalloc.h).  The test calls
it through its exported C symbol and compares it with the regular entry point on two
calls in a row (the static work array is reused by the second call).  The file name
makes pytest collect it last.
"""
import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _symbol():
    import dmad_b200._C as C

    lib = ctypes.CDLL(C.__file__)
    fn = lib.dmad_flash_attn_bwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 9 + [ctypes.c_int] * 4 + [ctypes.c_void_p, ctypes.c_float, ctypes.c_void_p]
    return fn


def _status_symbol():
    import dmad_b200._C as C

    lib = ctypes.CDLL(C.__file__)
    fn = lib.dmad_flash_attn_bwd_noalloc_status
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int)]
    return fn


def _read_status(stream):
    st = ctypes.c_int(-1)
    rc = _status_symbol()(stream.cuda_stream, ctypes.byref(st))
    assert rc == 0, rc
    return st.value


def _strides(*ts):
    vals = []
    for t in ts:
        vals += [t.stride(0), t.stride(1), t.stride(2)]
    return (ctypes.c_int64 * len(vals))(*vals)


def _case(B, Lq, Lk, H, seed):
    from dmad_b200 import ops

    e = ops.ext()
    g = torch.Generator(device="cuda").manual_seed(seed)
    mk = lambda L: torch.randn(B, L, H, 128, device="cuda", dtype=torch.bfloat16, generator=g)  # noqa: E731
    q, k, v, dout = mk(Lq), mk(Lk), mk(Lk), mk(Lq)
    scale = 1.0 / math.sqrt(128)
    o = torch.empty_like(q)
    lse = torch.empty(B, H, e.flash_lse_pad(Lq), device="cuda")
    e.flash_fwd(q, k, v, o, lse, scale)
    # regular entry point (caller-provided work buffer)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    e.flash_bwd(q, k, v, o, dout, lse, dq, dk, dv, torch.empty_like(lse), scale)
    return q, k, v, o, dout, lse, scale, (dq, dk, dv)


def test_noalloc_backward_matches_regular_entry_point():
    from dmad_b200 import ops

    fn = _symbol()
    stream = torch.cuda.current_stream()
    for call, (B, Lq, Lk, H) in enumerate([(1, 999, 999, 2), (2, 640, 300, 3)]):
        q, k, v, o, dout, lse, scale, ref = _case(B, Lq, Lk, H, seed=10 + call)
        dq, dk, dv = torch.full_like(q, float("nan")), torch.full_like(k, float("nan")), torch.full_like(v, float("nan"))
        rc = fn(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), dout.data_ptr(), lse.data_ptr(),
                dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), B, Lq, Lk, H,
                ctypes.cast(_strides(q, k, v, o, dout, dq, dk, dv), ctypes.c_void_p), scale, stream.cuda_stream)
        assert rc == 0, rc
        # the entry point's own status word: 0 means every bounded wait of its kernels completed
        assert _read_status(stream) == 0
        torch.cuda.synchronize()
        ops.check_device_status()
        for a, b, name in zip((dq, dk, dv), ref, ("dq", "dk", "dv")):
            assert torch.isfinite(a).all(), name
            rel = ((a.float() - b.float()).norm() / b.float().norm()).item()
            assert rel < 2e-2, (call, name, rel)


def test_noalloc_rejects_oversize():
    fn = _symbol()
    q = torch.zeros(1, 8, 1, 128, device="cuda", dtype=torch.bfloat16)
    st = _strides(*([q] * 8))
    # B * H * round_up(Lq, 256) far beyond the static array: rejected before any launch
    rc = fn(q.data_ptr(), q.data_ptr(), q.data_ptr(), q.data_ptr(), q.data_ptr(), q.data_ptr(), q.data_ptr(),
            q.data_ptr(), q.data_ptr(), 64, 1 << 16, 128, 64, ctypes.cast(st, ctypes.c_void_p), 0.1,
            torch.cuda.current_stream().cuda_stream)
    assert rc == 2


def test_noalloc_rejects_misaligned_pointer():
    fn = _symbol()
    q = torch.zeros(1, 256, 1, 128, device="cuda", dtype=torch.bfloat16)
    lse = torch.zeros(1, 1, 260, device="cuda")
    st = _strides(*([q] * 8))
    p = q.data_ptr()
    # an lse pointer 4 bytes past a 16-byte boundary is rejected before any launch
    rc = fn(p, p, p, p, p, lse.data_ptr() + 4, p, p, p, 1, 256, 256, 1, ctypes.cast(st, ctypes.c_void_p), 0.1,
            torch.cuda.current_stream().cuda_stream)
    assert rc == 1
    assert _read_status(torch.cuda.current_stream()) == 0
