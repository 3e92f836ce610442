"""Host-side mirror of the reference's attention operator surface (app/gpu/ops.js), over torch CUDA
tensors, calling the sm_100a kernels of libnsattn.so through the C ABI.

Names, argument meanings and error behaviour follow the JS operators:

* ``attention(q=, k=, v=, Lq=, Lk=, H=, D=, ldq=, ldk=, ldv=, qOff=, kOff=, vOff=, group=, causal=,
  bias=, biasStart=, out=)`` (app/gpu/ops.js:194-242) returns the output tensor ``[Lq, H*D]``;
* ``headNorm(X, weight, L=, H=, D=, ld=, colOff=, rowOff=, cs=, eps=)`` (app/gpu/ops.js:131-138)
  works in place;
* ``rope2dTable(h, w, D)`` / ``ropeTable(L, D, theta)`` (app/models/common.js:18-43) return a table
  object with ``buf`` (cos block then sin block) and ``sinOff``, like the JS tables.

Unsupported shapes raise ``NsaError`` synchronously, as the JS operators throw.  Extensions: a batch
dimension (3-D tensors), per-batch valid key counts ``kv_len``, a sliding ``window`` and a
``shard=(b_begin, b_count, h_begin, h_count)`` for batch x head partitioning across GPUs.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Optional

import torch

from . import _lib
from ._lib import NSA_BF16, NSA_F32, AttentionDesc, NsaError, check, lib

__all__ = ["attention", "headNorm", "linear", "lora_pack", "LoraPack", "rotate", "expand_i8", "rmsnorm", "glu", "glu_interleave", "rope2dTable", "ropeTable", "RopeTable", "NsaError",
           "dtype_code", "stream_handle", "check_device"]


def dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.float32:
        return NSA_F32
    if t.dtype == torch.bfloat16:
        return NSA_BF16
    raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, f"unsupported dtype {t.dtype} (float32 or bfloat16)")


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _require_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, "tensors must live on a CUDA device")


def check_device(device: Optional[torch.device] = None) -> None:
    """Synchronise the current stream and raise NsaError if any kernel reported a device-side error
    (the async-error surfacing of app/gpu/device.js:224-231)."""
    dev = device or torch.device("cuda", torch.cuda.current_device())
    with torch.cuda.device(dev):
        check(lib().nsa_check_device(stream_handle(dev)))


@dataclass
class RopeTable:
    """cos block [L][D/2] followed by the sin block; ``sinOff`` = L*D/2 (app/models/common.js:4-13)."""
    buf: torch.Tensor
    sinOff: int
    L: int
    D: int


def rope2dTable(h: int, w: int, D: int, device=None) -> RopeTable:
    """2D centred-coordinate RoPE table (app/models/common.js:28-43)."""
    device = device or torch.device("cuda", torch.cuda.current_device())
    L = h * w
    buf = torch.empty(L * D, dtype=torch.float32, device=device)
    with torch.cuda.device(buf.device):
        check(lib().nsa_rope2d_table(h, w, D, buf.data_ptr(), stream_handle(buf.device)))
    return RopeTable(buf, L * (D // 2), L, D)


def ropeTable(L: int, D: int, theta: float, device=None) -> RopeTable:
    """1D RoPE table, angle(l, i) = l / theta^(2i/D) (app/models/common.js:18-24)."""
    device = device or torch.device("cuda", torch.cuda.current_device())
    buf = torch.empty(L * D, dtype=torch.float32, device=device)
    with torch.cuda.device(buf.device):
        check(lib().nsa_rope1d_table(L, D, float(theta), buf.data_ptr(), stream_handle(buf.device)))
    return RopeTable(buf, L * (D // 2), L, D)


def headNorm(X: torch.Tensor, weight: torch.Tensor, *, L: int, H: int, D: int, ld: int, colOff: int = 0,
             rowOff: int = 0, cs: Optional[RopeTable] = None, eps: float = 1e-6) -> None:
    """In-place per-head RMSNorm (+ split-half RoPE with ``cs``) on L rows x H heads of D values at
    X[(rowOff + l) * ld + colOff + h * D] (app/gpu/ops.js:131-138)."""
    _require_cuda(X, weight)
    if weight.dtype != torch.float32:
        raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, "norm weight must be float32")
    with torch.cuda.device(X.device):
        check(lib().nsa_head_norm(X.data_ptr(), dtype_code(X), weight.data_ptr(), L, H, D, ld, colOff, rowOff,
                                  _ptr(cs.buf) if cs is not None else None, cs.sinOff if cs is not None else 0,
                                  float(eps), stream_handle(X.device)))


@dataclass
class LoraPack:
    """The LoRA side paths of one linear packed for ``linear`` (nsa_lora_pack): ``a`` bf16 [R, K],
    ``b`` bf16 [R] columns per output row [N, R], ``R`` the padded rank, and the ``alpha`` / weight
    scales ``b`` was divided by."""
    a: torch.Tensor
    b: torch.Tensor
    R: int
    N: int
    K: int
    alpha: float
    w_scale: Optional[torch.Tensor]


def lora_pack(entries, N: int, K: int, *, w_scale: Optional[torch.Tensor] = None, alpha: float = 1.0,
              rotate_a: bool = False) -> Optional[LoraPack]:
    """Pack LoRA entries ``[{"A": [r, K] fp32, "B": [n, r] fp32, "scale": s, "off": o, "n": n}]`` of one
    linear (app/lora.js:143-150: scale = strength * alpha / r, [off, off + n) the output columns).  For
    int8 ConvRot weights pass their ``w_scale``, and ``rotate_a=True`` when A's rows are not rotated yet
    (the reference's loader rotates them, app/lora.js:126).  Returns None for no entries."""
    entries = list(entries)
    if not entries:
        return None
    dev = entries[0]["A"].device
    _require_cuda(w_scale, *[e["A"] for e in entries], *[e["B"] for e in entries])
    keep = []
    arr = (_lib.LoraEntry * len(entries))()
    for i, e in enumerate(entries):
        A, B = e["A"], e["B"]
        if A.dtype != torch.float32 or B.dtype != torch.float32 or A.dim() != 2 or B.dim() != 2:
            raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, "LoRA A and B must be 2-D float32 tensors")
        r = A.shape[0]
        if A.shape[1] != K or B.shape[1] != r:
            raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, f"LoRA entry {i}: A must be [r, {K}] and B [n, r]")
        A = A.contiguous()
        if rotate_a:
            A = rotate(A)
        B = B.contiguous()
        keep += [A, B]
        arr[i].A, arr[i].B, arr[i].r = A.data_ptr(), B.data_ptr(), r
        arr[i].off, arr[i].n, arr[i].scale = int(e.get("off", 0)), int(e.get("n", B.shape[0])), float(e["scale"])
        if B.shape[0] != arr[i].n:
            raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, f"LoRA entry {i}: B has {B.shape[0]} rows, n = {arr[i].n}")
    R = lib().nsa_lora_rank(arr, len(entries))
    a = torch.empty((R, K), dtype=torch.bfloat16, device=dev)
    b = torch.empty((N, R), dtype=torch.bfloat16, device=dev)
    with torch.cuda.device(dev):
        check(lib().nsa_lora_pack(arr, len(entries), N, K, _ptr(w_scale), float(alpha), a.data_ptr(), b.data_ptr(),
                                  stream_handle(dev)))
    return LoraPack(a, b, R, N, K, float(alpha), w_scale)


def expand_i8(W: torch.Tensor) -> torch.Tensor:
    """int8 weights -> their exact bf16 values (nsa_expand_i8), the form the QKV projection takes
    ConvRot weights in (with their row scales passed separately)."""
    _require_cuda(W)
    if W.dtype != torch.int8 or not W.is_contiguous():
        raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, "W must be a contiguous int8 tensor")
    out = torch.empty(W.shape, dtype=torch.bfloat16, device=W.device)
    with torch.cuda.device(W.device):
        check(lib().nsa_expand_i8(W.data_ptr(), W.numel(), out.data_ptr(), stream_handle(W.device)))
    return out


def rotate(x: torch.Tensor, out: Optional[torch.Tensor] = None, *,
           out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    """ConvRot input rotation (app/gpu/ops.js:38-45): every group of 256 columns times the normalised
    regular Hadamard matrix H256.  x fp32 or bf16 [rows, cols] (cols a multiple of 256, unit inner
    stride); out fp32 or bf16 (``out_dtype``, default x's dtype)."""
    _require_cuda(x, out)
    if x.dim() != 2 or x.stride(1) != 1:
        raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, "x must be [rows, cols] with unit inner stride")
    if out is None:
        out = torch.empty(x.shape, dtype=out_dtype or x.dtype, device=x.device)
    if out.dim() != 2 or out.stride(1) != 1 or tuple(out.shape) != tuple(x.shape):
        raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, "out must match x's shape with unit inner stride")
    d = _lib.RotateDesc()
    d.rows, d.cols = x.shape
    d.ldx, d.ldy = x.stride(0), out.stride(0)
    d.in_dtype, d.out_dtype = dtype_code(x), dtype_code(out)
    with torch.cuda.device(x.device):
        check(lib().nsa_rotate(ctypes.byref(d), x.data_ptr(), out.data_ptr(), stream_handle(x.device)))
    return out


def linear(x: torch.Tensor, W: torch.Tensor, *, bias: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
           resid: bool = False, gate: Optional[torch.Tensor] = None, gOff: int = 0, act: Optional[str] = None,
           cOff: int = 0, alpha: float = 1.0, w_scale: Optional[torch.Tensor] = None,
           lora: Optional[LoraPack] = None, out_dtype: Optional[torch.dtype] = None,
           glu: Optional[str] = None, schedule: str = "auto") -> torch.Tensor:
    """y = x @ W^T (* w_scale) (+ bias) (+ LoRA delta) (silu), then out = y, out += y (resid) or
    out += gate[gOff + n] * y (resid + gate) (app/gpu/ops.js:50-66 with the epilogue of
    app/gpu/gemm.js:155-165).  x [M, K] bf16 (row pitch x.stride(0)); W [N, K] contiguous, bf16, or
    int8 with per-row float32 ``w_scale`` [N] (the ConvRot weights: x must then be the rotated input,
    ``rotate``; ``expand_i8(W)`` with the same ``w_scale`` gives the same result at the bf16 rate);
    ``lora`` from ``lora_pack``.  out [M, ldc] float32 (or bfloat16 for the store form)
    written at columns cOff..cOff+N-1, allocated [M, N] (dtype ``out_dtype``) when not given.
    ``glu`` "silu" / "gelu_tanh" fuses ops.glu (ops.js:141-148) into the gate_up linear: W, bias and
    w_scale in ``glu_interleave`` order, out [M, N / 2] = act(gate) * up.  ``schedule`` "auto",
    "single" (one CTA per 128 x 256 tile) or "pair" (two CTAs per 256 x 256 tile; bf16 W, M > 128):
    the same result either way."""
    _require_cuda(x, W, bias, out, gate, w_scale)
    if x.dim() != 2 or x.dtype != torch.bfloat16 or x.stride(1) != 1 or W.dtype not in (torch.bfloat16, torch.int8):
        raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT,
                       "x must be [M, K] bf16 and W [N, K] bf16 or int8, with unit inner stride")
    if not W.is_contiguous():
        raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, "W must be contiguous [N, K]")
    i8 = W.dtype == torch.int8
    if i8 and w_scale is None:
        raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, "int8 weights need a contiguous float32 w_scale of N entries")
    if w_scale is not None and (w_scale.dtype != torch.float32 or w_scale.numel() != W.shape[0]
                                or not w_scale.is_contiguous()):
        raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, "w_scale must be a contiguous float32 tensor of N entries")
    M, K = x.shape
    N = W.shape[0]
    if glu not in (None, "silu", "gelu_tanh"):
        raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, "glu is None, 'silu' or 'gelu_tanh'")
    if out is None:
        if resid:
            raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, "resid needs out")
        out = torch.empty((M, N // 2 if glu else N), dtype=out_dtype or torch.float32, device=x.device)
    if out.dtype not in (torch.float32, torch.bfloat16) or out.dim() != 2 or out.stride(1) != 1:
        raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, "out must be a float32 or bfloat16 [M, ldc] tensor with unit inner stride")
    d = _lib.LinearDesc()
    d.M, d.N, d.K = M, N, K
    d.lda, d.ldc, d.cOff, d.gOff = x.stride(0), out.stride(0), cOff, gOff
    d.alpha, d.resid, d.act = alpha, int(bool(resid)), {None: 0, "none": 0, "silu": 1}[act]
    d.out_dtype = dtype_code(out)
    d.w_format = _lib.NSA_W_I8 if i8 else _lib.NSA_W_BF16
    d.w_scale = _ptr(w_scale)
    d.glu = {None: 0, "silu": 1, "gelu_tanh": 2}[glu]
    if schedule not in ("auto", "single", "pair"):
        raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, "schedule is 'auto', 'single' or 'pair'")
    d.schedule = {"auto": _lib.NSA_LINEAR_AUTO, "single": _lib.NSA_LINEAR_SINGLE, "pair": _lib.NSA_LINEAR_PAIR}[schedule]
    t = None
    if lora is not None:
        if lora.N != N or lora.K != K:
            raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, f"the LoRA pack is for [{lora.N}, {lora.K}], W is [{N}, {K}]")
        if lora.alpha != float(alpha) or (lora.w_scale is None) != (w_scale is None):
            raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, "the LoRA pack was made for another alpha or weight format")
        t = torch.empty((M, lora.R), dtype=torch.bfloat16, device=x.device)
        d.lora_rank, d.lora_a, d.lora_b, d.lora_t = lora.R, lora.a.data_ptr(), lora.b.data_ptr(), t.data_ptr()
    with torch.cuda.device(x.device):
        check(lib().nsa_linear(ctypes.byref(d), x.data_ptr(), W.data_ptr(), _ptr(bias), _ptr(gate), out.data_ptr(),
                               stream_handle(x.device)))
    return out


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, cols: Optional[int] = None, eps: float = 1e-6,
            out: Optional[torch.Tensor] = None, *, accumulate: bool = False,
            out_dtype: Optional[torch.dtype] = None, next_weight: Optional[torch.Tensor] = None,
            next_out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """y = x * rsqrt(mean(x^2) + eps) * weight over rows of ``cols`` values (app/gpu/ops.js:111-116,
    kernels.js:62-80).  x fp32 [..., cols] with unit inner stride; out fp32 or bf16 (the next GEMM's
    operand), allocated like x when not given.  ``accumulate`` adds into ``out`` instead, the
    ops.accumulate that follows the Gemma layer's post-attention norm (app/models/gemma3.js:74-77);
    with ``next_weight`` the same pass also writes ``next_out`` = rmsnorm(out after the add) *
    next_weight (fp32 or bf16, out's shape), the norm the layer runs next (gemma3.js:78-79)."""
    _require_cuda(x, weight, out)
    cols = cols or x.shape[-1]
    if x.dtype != torch.float32 or weight.dtype != torch.float32 or x.stride(-1) != 1 or x.shape[-1] != cols:
        raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, "x and weight must be float32, x [..., cols] with unit inner stride")
    if weight.numel() < cols or not weight.is_contiguous():
        raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, "weight must be a contiguous [cols] tensor")
    if out is None:
        if accumulate:
            raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, "accumulate needs out")
        out = torch.empty(x.shape, dtype=out_dtype or torch.float32, device=x.device)
    if out.shape != x.shape or out.stride(-1) != 1:
        raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, "out must match x's shape with unit inner stride")

    def rows(t):   # [rows, cols] view with a row pitch: 2-D tensors as they are, others contiguous
        if t.dim() == 2:
            return t
        if not t.is_contiguous():
            raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, "x and out of more than two dims must be contiguous")
        return t.view(-1, cols)

    x2, o2 = rows(x), rows(out)
    d = _lib.RmsnormDesc()
    d.rows, d.cols = x2.shape[0], cols
    d.ldx, d.ldy = x2.stride(0), o2.stride(0)
    d.out_dtype, d.accumulate, d.eps = dtype_code(out), int(bool(accumulate)), eps
    if next_weight is not None:
        _require_cuda(next_weight, next_out)
        if next_out is None or next_out.shape != out.shape or next_out.stride(-1) != 1:
            raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, "next_weight needs next_out of out's shape with unit inner stride")
        if next_weight.dtype != torch.float32 or not next_weight.is_contiguous() or next_weight.numel() < cols:
            raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, "next_weight must be a contiguous float32 [cols] tensor")
        z2 = rows(next_out)
        d.next_weight, d.Z, d.ldz, d.z_dtype = next_weight.data_ptr(), z2.data_ptr(), z2.stride(0), dtype_code(next_out)
    with torch.cuda.device(x.device):
        check(lib().nsa_rmsnorm(ctypes.byref(d), x2.data_ptr(), weight.data_ptr(), o2.data_ptr(),
                                stream_handle(x.device)))
    return out


def glu_interleave(t: torch.Tensor) -> torch.Tensor:
    """The row order ``linear(..., glu=)`` reads, from a gate_up tensor whose 2I rows are [gate; up]
    (the weight [2I, K], its bias or its w_scale [2I]): row 256 j + i is gate row 128 j + i for
    i < 128 and up row I + 128 j + i - 128 otherwise.  I a multiple of 128; a new tensor, made once
    at load time (nsa_glu_interleave)."""
    _require_cuda(t)
    if t.dim() not in (1, 2) or t.shape[0] % 256 or not t.is_contiguous():
        raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, "t must be a contiguous [2I] or [2I, K] tensor, I a multiple of 128")
    out = torch.empty_like(t)
    row_bytes = t.element_size() * (t.shape[1] if t.dim() == 2 else 1)
    with torch.cuda.device(t.device):
        check(lib().nsa_glu_interleave(t.data_ptr(), out.data_ptr(), t.shape[0] // 2, row_bytes, stream_handle(t.device)))
    return out


def glu(x: torch.Tensor, act: str = "gelu_tanh", out: Optional[torch.Tensor] = None,
        out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    """ops.glu (app/gpu/ops.js:141-148): x fp32 [rows, 2I] = [gate | up] -> act(gate) * up, [rows, I];
    act "silu" or "gelu_tanh" (Gemma's MLP).  out fp32 or bf16 (the down projection's operand),
    allocated when not given."""
    _require_cuda(x, out)
    if x.dim() != 2 or x.dtype != torch.float32 or x.stride(1) != 1 or x.shape[1] % 2:
        raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, "x must be float32 [rows, 2I] with unit inner stride")
    rows, I = x.shape[0], x.shape[1] // 2
    if act not in ("silu", "gelu_tanh"):
        raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, "act is 'silu' or 'gelu_tanh'")
    if out is None:
        out = torch.empty((rows, I), dtype=out_dtype or torch.float32, device=x.device)
    if out.dim() != 2 or out.shape != (rows, I) or out.stride(1) != 1:
        raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, "out must be [rows, I] with unit inner stride")
    d = _lib.GluDesc()
    d.rows, d.I, d.ldx, d.ldy = rows, I, x.stride(0), out.stride(0)
    d.act, d.out_dtype = (0 if act == "silu" else 1), dtype_code(out)
    with torch.cuda.device(x.device):
        check(lib().nsa_glu(ctypes.byref(d), x.data_ptr(), out.data_ptr(), stream_handle(x.device)))
    return out


def _bstride(t: torch.Tensor, rows_ld: int) -> int:
    return t.stride(0) if t.dim() == 3 else 0


def attention(*, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, Lq: int, Lk: int, H: int, D: int,
              ldq: int, ldk: int, ldv: int, qOff: int = 0, kOff: int = 0, vOff: int = 0, group: int = 1,
              causal: bool = False, bias: Optional[torch.Tensor] = None, biasStart: int = 0,
              out: Optional[torch.Tensor] = None, window: int = 0, kv_len: Optional[torch.Tensor] = None,
              out_dtype: Optional[torch.dtype] = None, scale: float = 0.0, shard=None,
              tf32: bool = False) -> torch.Tensor:
    """Multi-head attention (app/gpu/ops.js:194-242).

    q: [Lq, ldq] (or [B, Lq, ldq]) with head h at column qOff + h*D; k, v: [Lk, ldk] / [Lk, ldv] with kv
    head h // group at kOff / vOff + (h // group) * D; bias: [biasLen] (or [B, biasLen]) additive
    score bias for keys biasStart..; out: [Lq, H*D] (or [B, Lq, H*D]), allocated when not given.
    ``tf32`` (fp32 q/k/v at head dim 96): multiply at tf32 precision instead of rounding to bf16.
    """
    _require_cuda(q, k, v, bias, out, kv_len)
    B = q.shape[0] if q.dim() == 3 else 1
    if out is None:
        odt = out_dtype or (torch.float32 if q.dtype == torch.float32 else torch.bfloat16)
        shape = (B, Lq, H * D) if q.dim() == 3 else (Lq, H * D)
        out = torch.empty(shape, dtype=odt, device=q.device)
    if q.dtype != k.dtype or q.dtype != v.dtype:
        raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, "q, k and v must share a dtype")
    if kv_len is not None and kv_len.dtype != torch.int32:
        raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, "kv_len must be int32")
    if bias is not None and bias.dtype != torch.float32:
        raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, "bias must be float32")
    d = AttentionDesc()
    d.Lq, d.Lk, d.H, d.D = Lq, Lk, H, D
    d.ldq, d.ldk, d.ldv = ldq, ldk, ldv
    d.qOff, d.kOff, d.vOff = qOff, kOff, vOff
    d.group, d.causal, d.window = group, int(bool(causal)), window
    d.biasStart = biasStart
    d.biasLen = 0 if bias is None else bias.shape[-1]
    d.B = B
    d.q_bstride, d.k_bstride, d.v_bstride = _bstride(q, ldq), _bstride(k, ldk), _bstride(v, ldv)
    d.bias_bstride = bias.stride(0) if (bias is not None and bias.dim() == 2) else 0
    d.o_bstride = out.stride(0) if out.dim() == 3 else 0
    d.ldo = out.stride(-2)
    d.oOff = 0
    d.in_dtype, d.out_dtype = dtype_code(q), dtype_code(out)
    d.scale = scale
    d.compute = _lib.NSA_COMPUTE_TF32 if tf32 else _lib.NSA_COMPUTE_BF16
    if shard is not None:
        d.b_begin, d.b_count, d.h_begin, d.h_count = shard
    L = lib()
    ws_bytes = L.nsa_attention_workspace_size(ctypes.byref(d))
    if ws_bytes == 0:
        # re-run through the entry point to surface the validation message
        check(L.nsa_attention(ctypes.byref(d), q.data_ptr(), k.data_ptr(), v.data_ptr(), None, None,
                              out.data_ptr(), None, 0, None))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device)
    with torch.cuda.device(q.device):
        check(L.nsa_attention(ctypes.byref(d), q.data_ptr(), k.data_ptr(), v.data_ptr(), _ptr(bias), _ptr(kv_len),
                              out.data_ptr(), ws.data_ptr(), ws_bytes, stream_handle(q.device)))
    return out
