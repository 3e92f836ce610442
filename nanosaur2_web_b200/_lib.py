"""ctypes binding of libnsattn.so (the C ABI declared in include/nsattn.h).

The library is built in-tree by ``nanosaur2_web_b200.build``; importing this module fails loudly when
it is missing.  There is no CPU fallback anywhere in the package.
"""

from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libnsattn.so")

NSA_OK, NSA_ERR_INVALID_ARGUMENT, NSA_ERR_UNSUPPORTED, NSA_ERR_WORKSPACE, NSA_ERR_CUDA, NSA_ERR_DEVICE = range(6)
NSA_F32, NSA_BF16 = 0, 1
NSA_COMPUTE_BF16, NSA_COMPUTE_TF32 = 0, 1
NSA_W_BF16, NSA_W_I8 = 0, 1
NSA_LINEAR_AUTO, NSA_LINEAR_SINGLE, NSA_LINEAR_PAIR = 0, 1, 2
NSA_IPC_HANDLE_BYTES = 72

_i32, _i64, _f32, _vp, _sz = ctypes.c_int32, ctypes.c_int64, ctypes.c_float, ctypes.c_void_p, ctypes.c_size_t


class AttentionDesc(ctypes.Structure):
    """nsa_attention_desc (include/nsattn.h)."""
    _fields_ = [
        ("Lq", _i32), ("Lk", _i32), ("H", _i32), ("D", _i32),
        ("ldq", _i64), ("ldk", _i64), ("ldv", _i64),
        ("qOff", _i64), ("kOff", _i64), ("vOff", _i64),
        ("group", _i32), ("causal", _i32), ("window", _i32), ("biasStart", _i32), ("biasLen", _i32), ("B", _i32),
        ("q_bstride", _i64), ("k_bstride", _i64), ("v_bstride", _i64), ("bias_bstride", _i64), ("o_bstride", _i64),
        ("ldo", _i64), ("oOff", _i64),
        ("in_dtype", _i32), ("out_dtype", _i32), ("scale", _f32),
        ("b_begin", _i32), ("b_count", _i32), ("h_begin", _i32), ("h_count", _i32),
        ("compute", _i32),
    ]


class FusedDesc(ctypes.Structure):
    """nsa_fused_desc (include/nsattn.h)."""
    _fields_ = [
        ("B", _i32), ("Lq", _i32), ("Lk", _i32), ("Hq", _i32), ("Hkv", _i32), ("D", _i32),
        ("ld", _i64), ("bstride", _i64),
        ("qOff", _i64), ("kOff", _i64), ("vOff", _i64),
        ("in_dtype", _i32), ("out_dtype", _i32), ("eps", _f32),
        ("sinOff", _i64),
        ("causal", _i32), ("window", _i32), ("biasStart", _i32), ("biasLen", _i32),
        ("bias_bstride", _i64),
        ("ldo", _i64), ("o_bstride", _i64), ("oOff", _i64),
        ("scale", _f32),
        ("b_begin", _i32), ("b_count", _i32), ("h_begin", _i32), ("h_count", _i32),
        ("compute", _i32),
    ]


class SeqShard(ctypes.Structure):
    """nsa_seq_shard (include/nsattn.h)."""
    _fields_ = [("q_begin", _i32), ("q_count", _i32), ("qkv_image_row0", _i32), ("qkv_text_row0", _i32)]


class ProjDesc(ctypes.Structure):
    """nsa_proj_desc (include/nsattn.h)."""
    _fields_ = [("K", _i32), ("x", _vp), ("ldx", _i64), ("x_bstride", _i64), ("x_rows", _i32), ("w_qkv", _vp),
                ("b_qkv", _vp), ("x_text", _vp), ("ld_text", _i64), ("text_bstride", _i64), ("text_rows", _i32),
                ("w_kv", _vp), ("b_kv", _vp), ("w_qkv_scale", _vp), ("w_kv_scale", _vp), ("lora_rank_qkv", _i32),
                ("lora_a_qkv", _vp), ("lora_b_qkv", _vp), ("lora_rank_kv", _i32), ("lora_a_kv", _vp),
                ("lora_b_kv", _vp), ("lora_t", _vp)]


class LinearDesc(ctypes.Structure):
    """nsa_linear_desc (include/nsattn.h)."""
    _fields_ = [("M", _i32), ("N", _i32), ("K", _i32), ("lda", _i64), ("ldc", _i64), ("cOff", _i64), ("gOff", _i64),
                ("alpha", _f32), ("resid", _i32), ("act", _i32), ("out_dtype", _i32), ("w_format", _i32),
                ("w_scale", _vp), ("lora_rank", _i32), ("lora_a", _vp), ("lora_b", _vp), ("lora_t", _vp), ("glu", _i32),
                ("schedule", _i32)]


class RotateDesc(ctypes.Structure):
    """nsa_rotate_desc (include/nsattn.h)."""
    _fields_ = [("rows", _i32), ("cols", _i32), ("ldx", _i64), ("ldy", _i64), ("in_dtype", _i32), ("out_dtype", _i32)]


class LoraEntry(ctypes.Structure):
    """nsa_lora_entry (include/nsattn.h)."""
    _fields_ = [("A", _vp), ("B", _vp), ("r", _i32), ("off", _i32), ("n", _i32), ("scale", _f32)]


class RmsnormDesc(ctypes.Structure):
    """nsa_rmsnorm_desc (include/nsattn.h)."""
    _fields_ = [("rows", _i32), ("cols", _i32), ("ldx", _i64), ("ldy", _i64), ("out_dtype", _i32),
                ("accumulate", _i32), ("eps", _f32), ("next_weight", _vp), ("Z", _vp), ("ldz", _i64),
                ("z_dtype", _i32)]


class GluDesc(ctypes.Structure):
    """nsa_glu_desc (include/nsattn.h)."""
    _fields_ = [("rows", _i32), ("I", _i32), ("ldx", _i64), ("ldy", _i64), ("act", _i32), ("out_dtype", _i32)]


class KernelStat(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * 32), ("launches", _i64), ("total_ms", ctypes.c_double),
                ("flops", ctypes.c_double), ("bytes", ctypes.c_double)]


# every entry point of include/nsattn.h: name -> (restype, argtypes)
SIGNATURES = {
    "nsa_version": (ctypes.c_char_p, []),
    "nsa_last_error": (ctypes.c_char_p, []),
    "nsa_status_string": (ctypes.c_char_p, [_i32]),
    "nsa_attention_workspace_size": (_sz, [ctypes.POINTER(AttentionDesc)]),
    "nsa_attention": (_i32, [ctypes.POINTER(AttentionDesc), _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
    "nsa_head_norm": (_i32, [_vp, _i32, _vp, _i32, _i32, _i32, _i64, _i64, _i64, _vp, _i64, _f32, _vp]),
    "nsa_fused_attention_workspace_size": (_sz, [ctypes.POINTER(FusedDesc)]),
    "nsa_fused_attention": (_i32, [ctypes.POINTER(FusedDesc), _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
    "nsa_fused_attention_noalloc": (_i32, [ctypes.POINTER(FusedDesc), _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "nsa_seq_shard_buffer_sizes": (_i32, [ctypes.POINTER(FusedDesc), ctypes.POINTER(SeqShard), ctypes.POINTER(_sz),
                                          ctypes.POINTER(_sz), ctypes.POINTER(_i32)]),
    "nsa_seq_shard_prologue": (_i32, [ctypes.POINTER(FusedDesc), ctypes.POINTER(SeqShard), _vp, _vp, _vp, _vp, _vp,
                                      _vp, _vp, _vp]),
    "nsa_ipc_export": (_i32, [_vp, _vp]),
    "nsa_ipc_import": (_i32, [_vp, ctypes.POINTER(_vp)]),
    "nsa_ipc_close": (_i32, [_vp]),
    "nsa_memcpy_async": (_i32, [_vp, _vp, _sz, _vp]),
    "nsa_seq_shard_prologue_peers": (_i32, [ctypes.POINTER(FusedDesc), ctypes.POINTER(SeqShard), _vp, _vp, _vp, _vp,
                                            _vp, _vp, _vp, ctypes.POINTER(_vp), _i32, _vp]),
    "nsa_seq_shard_attention": (_i32, [ctypes.POINTER(FusedDesc), ctypes.POINTER(SeqShard), _vp, _vp, _vp, _vp, _vp,
                                       _vp]),
    "nsa_seq_shard_projection": (_i32, [ctypes.POINTER(FusedDesc), ctypes.POINTER(SeqShard), ctypes.POINTER(ProjDesc),
                                        _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "nsa_linear": (_i32, [ctypes.POINTER(LinearDesc), _vp, _vp, _vp, _vp, _vp, _vp]),
    "nsa_rotate": (_i32, [ctypes.POINTER(RotateDesc), _vp, _vp, _vp]),
    "nsa_lora_rank": (_i32, [ctypes.POINTER(LoraEntry), _i32]),
    "nsa_expand_i8": (_i32, [_vp, _i64, _vp, _vp]),
    "nsa_lora_pack": (_i32, [ctypes.POINTER(LoraEntry), _i32, _i32, _i32, _vp, _f32, _vp, _vp, _vp]),
    "nsa_rmsnorm": (_i32, [ctypes.POINTER(RmsnormDesc), _vp, _vp, _vp, _vp]),
    "nsa_glu": (_i32, [ctypes.POINTER(GluDesc), _vp, _vp, _vp]),
    "nsa_glu_interleave": (_i32, [_vp, _vp, _i32, _i64, _vp]),
    "nsa_rope2d_table": (_i32, [_i32, _i32, _i32, _vp, _vp]),
    "nsa_rope1d_table": (_i32, [_i32, _i32, _f32, _vp, _vp]),
    "nsa_check_device": (_i32, [_vp]),
    "nsa_selftest_wait_timeout": (_i32, [_i32, _vp]),
    "nsa_profiler_enable": (None, [_i32]),
    "nsa_profiler_reset": (None, []),
    "nsa_profiler_read": (_i32, [ctypes.POINTER(KernelStat), _i32]),
}


class NsaError(RuntimeError):
    """A failing nsa_* call: ``status`` is the nsa_status code, the message comes from nsa_last_error."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{message} (nsa status {status})")
        self.status = status


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build the CUDA library first (python -m nanosaur2_web_b200.build); "
                "this package has no CPU fallback")
        handle = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def check(status: int) -> None:
    if status != NSA_OK:
        raise NsaError(status, lib().nsa_last_error().decode())


def version() -> str:
    return lib().nsa_version().decode()
