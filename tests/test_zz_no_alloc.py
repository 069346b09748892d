"""The allocation-free attention backward (``ddb_attn_bwd_noalloc``), called through its
exported C symbol, matches the regular backward on two calls in a row.

The entry point exists for callers that cannot allocate device memory while they run
(pre-planned memory executors, foreign allocators); it keeps its scratch in fixed
device arrays. This file is collected last so that a failure here leaves every other
test already run.
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


def _entry():
    import drivedit_b200._C as C

    lib = ctypes.CDLL(C.__file__)
    fn = lib.ddb_attn_bwd_noalloc
    fn.argtypes = [ctypes.POINTER(_Args), ctypes.c_void_p]
    fn.restype = ctypes.c_int
    return fn


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
