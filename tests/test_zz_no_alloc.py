"""nsa_fused_attention_noalloc, the entry point for callers that cannot allocate device memory.

Some hosts of this library cannot give it a workspace: their allocator is closed to plugins, or they
must not call cudaMalloc while sharing the GPU with latency-critical work.  For them the fused
attention step runs on a scratch array built into the library.  This test calls that entry point
through the C ABI, twice in a row on different shapes (so the second call runs on the scratch the
first one left behind), and checks each output against the regular workspace entry point: within the
bf16 tolerance the other parity tests use and, since both run the same kernels on the same inputs,
bit for bit (the tail split merges its halves in a fixed order, so this holds for split launches too).  It also checks that a shape above the scratch limit is
refused with NSA_ERR_WORKSPACE and a message, without launching anything.

The file name makes pytest collect it last; it needs nothing from the other tests.
"""

import ctypes

import numpy as np
import pytest
import torch

from tests._helpers import assert_close_bf16, gemma_inputs, joint_inputs

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def _t(x, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(x)).to(device=DEV, dtype=dtype)


def _desc(B, Lq, Lk, Hq, Hkv, D, ld, offs, causal=0, window=0, bias_len=0, bias_start=0, sin_off=0):
    from nanosaur2_web_b200 import _lib
    d = _lib.FusedDesc()
    d.B, d.Lq, d.Lk, d.Hq, d.Hkv, d.D = B, Lq, Lk, Hq, Hkv, D
    d.ld, d.bstride = ld, Lk * ld
    d.qOff, d.kOff, d.vOff = offs
    d.in_dtype, d.out_dtype = _lib.NSA_BF16, _lib.NSA_F32
    d.eps = 1e-6
    d.sinOff = sin_off
    d.causal, d.window = causal, window
    d.biasStart, d.biasLen, d.bias_bstride = bias_start, bias_len, bias_len
    d.ldo, d.o_bstride, d.oOff = Hq * D, Lq * Hq * D, 0
    return d


def _both(d, qkv, qw, kw, cs, kv_len, bias):
    """Run the regular entry point (torch workspace) and the no-alloc one on the same inputs."""
    from nanosaur2_web_b200 import _lib
    from nanosaur2_web_b200.ops import check_device, stream_handle
    L = _lib.lib()
    s = stream_handle(DEV)
    ptr = lambda x: None if x is None else x.data_ptr()  # noqa: E731
    out_ref = torch.empty((d.B, d.Lq, d.Hq * d.D), dtype=torch.float32, device=DEV)
    out_na = torch.full_like(out_ref, float("nan"))
    ws_bytes = L.nsa_fused_attention_workspace_size(ctypes.byref(d))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=DEV)
    _lib.check(L.nsa_fused_attention(ctypes.byref(d), qkv.data_ptr(), qw.data_ptr(), kw.data_ptr(), ptr(cs),
                                     ptr(kv_len), ptr(bias), out_ref.data_ptr(), ws.data_ptr(), ws_bytes, s))
    _lib.check(L.nsa_fused_attention_noalloc(ctypes.byref(d), qkv.data_ptr(), qw.data_ptr(), kw.data_ptr(), ptr(cs),
                                             ptr(kv_len), ptr(bias), out_na.data_ptr(), s))
    check_device(DEV)
    return out_ref.cpu().numpy(), out_na.cpu().numpy()


def test_noalloc_matches_workspace_entry_point_twice():
    from nanosaur2_web_b200.ops import rope2dTable, ropeTable
    torch.cuda.set_device(DEV)
    # call 1: a DiT joint block (image q|k|v rows + text k|v rows, key bias, padding via kv_len)
    h, w, Lt = 20, 30, 64
    L = h * w
    qkv, q_w, k_w, lv, bias = joint_inputs(2024, 1, h, w, Lt, (10, 64))
    cs = rope2dTable(h, w, 96, DEV)
    d = _desc(1, L, L + Lt, 16, 16, 96, 4608, (0, 1536, 3072), bias_len=Lt, bias_start=L, sin_off=cs.sinOff)
    ref, na = _both(d, _t(qkv, torch.bfloat16), _t(q_w), _t(k_w), cs.buf, _t((L + lv).astype(np.int32), torch.int32),
                    _t(bias))
    assert_close_bf16(na, ref, 96, what="no-alloc call 1 (DiT joint)")
    # the same kernels on the same inputs: the outputs must be identical, bit for bit (a stale row
    # of the previous call's scratch would show up here)
    np.testing.assert_array_equal(na, ref)
    # call 2, right after: a causal Gemma layer with a window, on the scratch call 1 left behind
    B, Lg = 2, 384
    qkv2, q_w2, k_w2 = gemma_inputs(2025, B, Lg)
    cs2 = ropeTable(Lg, 256, 1e4, DEV)
    d2 = _desc(B, Lg, Lg, 4, 1, 256, 1536, (0, 1024, 1280), causal=1, window=200, sin_off=cs2.sinOff)
    ref2, na2 = _both(d2, _t(qkv2, torch.bfloat16), _t(q_w2), _t(k_w2), cs2.buf, None, None)
    assert_close_bf16(na2, ref2, 256, what="no-alloc call 2 (Gemma)")
    np.testing.assert_array_equal(na2, ref2)


def test_noalloc_rejects_shapes_above_the_scratch_limit():
    from nanosaur2_web_b200 import _lib
    L = _lib.lib()
    d = _desc(2, 3952, 4208, 16, 16, 96, 4608, (0, 1536, 3072))
    assert L.nsa_fused_attention_workspace_size(ctypes.byref(d)) > (64 << 20)
    fake = 0x10000   # never dereferenced: the size check fails before any launch
    st = L.nsa_fused_attention_noalloc(ctypes.byref(d), fake, fake, fake, None, None, None, fake, None)
    assert st == _lib.NSA_ERR_WORKSPACE
    assert b"scratch" in L.nsa_last_error()
