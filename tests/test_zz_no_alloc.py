"""The allocation-free attention backward (``ddb_attn_bwd_noalloc``, declared in
``csrc/attn/attn_noalloc.h``), called through its exported C symbol, matches the
regular backward on two calls in a row.

The entry point exists for callers that cannot allocate device memory while they run
(runtimes that plan all device memory up front, hosts that own the allocator); it keeps
its scratch in fixed device arrays. This file is collected last so that a failure here
leaves every other test already run.
"""
import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


class _Args(ctypes.Structure):
    _fields_ = [
        ("B", ctypes.c_int), ("H", ctypes.c_int), ("Tq", ctypes.c_int), ("S", ctypes.c_int),
        ("q_rows_per_b", ctypes.c_longlong), ("kv_rows_per_b", ctypes.c_longlong),
        ("q", ctypes.c_void_p), ("ldq", ctypes.c_longlong), ("q_col", ctypes.c_int),
        ("k", ctypes.c_void_p), ("ldk", ctypes.c_longlong), ("k_col", ctypes.c_int),
        ("v", ctypes.c_void_p), ("ldv", ctypes.c_longlong), ("v_col", ctypes.c_int),
        ("o", ctypes.c_void_p), ("ldo", ctypes.c_longlong), ("o_col", ctypes.c_int),
        ("dout", ctypes.c_void_p), ("lddo", ctypes.c_longlong), ("do_col", ctypes.c_int),
        ("lse", ctypes.c_void_p),
        ("dq", ctypes.c_void_p), ("lddq", ctypes.c_longlong), ("dq_col", ctypes.c_int),
        ("dk", ctypes.c_void_p), ("lddk", ctypes.c_longlong), ("dk_col", ctypes.c_int),
        ("dv", ctypes.c_void_p), ("lddv", ctypes.c_longlong), ("dv_col", ctypes.c_int),
        ("causal", ctypes.c_int), ("tokens_per_frame", ctypes.c_int),
        ("q_pos_offset", ctypes.c_int), ("kv_pos_offset", ctypes.c_int),
        ("scale", ctypes.c_float),
    ]


def _lib():
    import drivedit_b200._C as C

    lib = ctypes.CDLL(C.__file__)
    lib.ddb_attn_bwd_noalloc.argtypes = [ctypes.POINTER(_Args), ctypes.c_void_p]
    lib.ddb_attn_bwd_noalloc.restype = ctypes.c_int
    lib.ddb_attn_bwd_noalloc_status.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int)]
    lib.ddb_attn_bwd_noalloc_status.restype = ctypes.c_int
    lib.ddb_attn_bwd_noalloc_args_size.restype = ctypes.c_ulonglong
    # the ctypes mirror of the argument struct must match the compiled layout
    assert lib.ddb_attn_bwd_noalloc_args_size() == ctypes.sizeof(_Args)
    return lib


def _entry():
    return _lib().ddb_attn_bwd_noalloc


def _status(stream=None):
    st = ctypes.c_int(-1)
    rc = _lib().ddb_attn_bwd_noalloc_status(stream, ctypes.byref(st))
    return rc, st.value


def _rel(a, b):
    return ((a.float() - b.float()).abs().max() / (b.float().abs().max() + 1e-6)).item()


def test_noalloc_backward_matches_regular_entry_point_twice():
    from drivedit_b200.ops._ext import ext

    torch.manual_seed(0)
    B, H, T, tpf = 2, 3, 512, 128
    d = H * 64
    scale = 1.0 / math.sqrt(64)
    qkv = (torch.randn(B * T, 3 * d, device="cuda") * 0.7).bfloat16()
    o = torch.empty(B * T, d, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(B * H * T, device="cuda")
    ext().attn_fwd(qkv, qkv, qkv, o, lse, 0, d, 2 * d, 0, B, H, T, T, T, T, 1, tpf, 0, 0, scale,
                   None, None, None)
    fn = _entry()
    for call in range(2):
        do = torch.randn(B * T, d, device="cuda").bfloat16()
        # regular entry point (caller-allocated scratch)
        delta = torch.empty(B * H * T, device="cuda")
        ext().attn_delta(o, do, delta, 0, 0, B, H, T, T)
        dq_acc = torch.zeros(B * T, d, device="cuda")
        ref = torch.zeros(B * T, 3 * d, device="cuda", dtype=torch.bfloat16)
        ext().attn_bwd(qkv, qkv, qkv, o, do, lse, delta, dq_acc, ref, ref, 0, d, 2 * d, 0, 0, d,
                       2 * d, B, H, T, T, T, T, 1, tpf, 0, 0, scale, None, None, None, 0)
        ext().attn_dq_finalize(dq_acc, ref, 0, H, None, T, 0)
        # allocation-free entry point
        out = torch.full((B * T, 3 * d), float("nan"), device="cuda", dtype=torch.bfloat16)
        a = _Args(B, H, T, T, T, T,
                  qkv.data_ptr(), qkv.stride(0), 0,
                  qkv.data_ptr(), qkv.stride(0), d,
                  qkv.data_ptr(), qkv.stride(0), 2 * d,
                  o.data_ptr(), o.stride(0), 0,
                  do.data_ptr(), do.stride(0), 0,
                  lse.data_ptr(),
                  out.data_ptr(), out.stride(0), 0,
                  out.data_ptr(), out.stride(0), d,
                  out.data_ptr(), out.stride(0), 2 * d,
                  1, tpf, 0, 0, scale)
        rc = fn(ctypes.byref(a), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        assert rc == 0, f"call {call}: return code {rc}"
        src, st = _status(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        assert (src, st) == (0, 0), f"call {call}: device status {st} (query rc {src})"
        torch.cuda.synchronize()
        assert torch.isfinite(out.float()).all(), f"call {call}: unwritten outputs"
        assert _rel(out, ref) < 2e-2, f"call {call}: differs from the regular entry point"


def test_noalloc_rejects_oversized_problem():
    fn = _entry()
    dummy = torch.zeros(16, device="cuda")
    p = dummy.data_ptr()
    B, H, T = 64, 16, 8192  # rows * heads * 64 far beyond the 16 MiB accumulator
    a = _Args(B, H, T, T, T, T, p, 3 * H * 64, 0, p, 3 * H * 64, 0, p, 3 * H * 64, 0,
              p, H * 64, 0, p, H * 64, 0, p, p, 3 * H * 64, 0, p, 3 * H * 64, 0, p, 3 * H * 64, 0,
              1, 512, 0, 0, 0.125)
    assert fn(ctypes.byref(a), None) == 2


def test_noalloc_leaves_rows_between_samples_untouched():
    """With q_rows_per_b > Tq the caller's rows after each sample's Tq rows keep their
    contents, and the sample rows match the regular entry point."""
    from drivedit_b200.ops._ext import ext

    torch.manual_seed(1)
    B, H, T, tpf, gap = 2, 2, 256, 64, 64
    R = T + gap                                    # rows per sample in every tensor
    d = H * 64
    scale = 1.0 / math.sqrt(64)
    qkv = (torch.randn(B * R, 3 * d, device="cuda") * 0.7).bfloat16()
    o = torch.zeros(B * R, d, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(B * H * T, device="cuda")
    ext().attn_fwd(qkv, qkv, qkv, o, lse, 0, d, 2 * d, 0, B, H, T, T, R, R, 1, tpf, 0, 0, scale,
                   None, None, None)
    do = torch.randn(B * R, d, device="cuda").bfloat16()
    sentinel = 7.0
    out = torch.full((B * R, 3 * d), sentinel, device="cuda", dtype=torch.bfloat16)
    a = _Args(B, H, T, T, R, R,
              qkv.data_ptr(), qkv.stride(0), 0, qkv.data_ptr(), qkv.stride(0), d,
              qkv.data_ptr(), qkv.stride(0), 2 * d, o.data_ptr(), o.stride(0), 0,
              do.data_ptr(), do.stride(0), 0, lse.data_ptr(),
              out.data_ptr(), out.stride(0), 0, out.data_ptr(), out.stride(0), d,
              out.data_ptr(), out.stride(0), 2 * d, 1, tpf, 0, 0, scale)
    assert _entry()(ctypes.byref(a), None) == 0
    assert _status() == (0, 0)
    torch.cuda.synchronize()
    rows = out.view(B, R, 3 * d)
    assert (rows[:, T:].float() == sentinel).all(), "rows between samples were overwritten"
    # the sample rows equal a per-sample run of the regular entry point
    for b in range(B):
        sl = slice(b * R, b * R + T)
        qb, ob, dob = qkv[sl].contiguous(), o[sl].contiguous(), do[sl].contiguous()
        lb = lse.view(B, H * T)[b].contiguous()
        delta = torch.empty(H * T, device="cuda")
        ext().attn_delta(ob, dob, delta, 0, 0, 1, H, T, T)
        acc = torch.zeros(T, d, device="cuda")
        ref = torch.zeros(T, 3 * d, device="cuda", dtype=torch.bfloat16)
        ext().attn_bwd(qb, qb, qb, ob, dob, lb, delta, acc, ref, ref, 0, d, 2 * d, 0, 0, d,
                       2 * d, 1, H, T, T, T, T, 1, tpf, 0, 0, scale, None, None, None, 0)
        ext().attn_dq_finalize(acc, ref, 0, H, None, T, 0)
        assert _rel(rows[b, :T], ref) < 2e-2


def test_noalloc_rejects_bad_query_count_before_launching():
    fn = _entry()
    dummy = torch.zeros(16, device="cuda")
    p = dummy.data_ptr()
    B, H, T = 1, 2, 200  # not a multiple of 128
    a = _Args(B, H, T, T, T, T, p, 3 * H * 64, 0, p, 3 * H * 64, 0, p, 3 * H * 64, 0,
              p, H * 64, 0, p, H * 64, 0, p, p, 3 * H * 64, 0, p, 3 * H * 64, 0, p, 3 * H * 64, 0,
              1, 100, 0, 0, 0.125)
    assert fn(ctypes.byref(a), None) == 1
