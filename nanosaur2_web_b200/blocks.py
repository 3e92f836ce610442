"""The model call sites of the attention hot path, as fused single calls into libnsattn.so.

* ``prepare_text_bias(weights)``: the per-text-key log-weight bias and the dropped (w <= 0) tokens of
  ``Nanosaur2DiT.prepareText`` (app/models/nanosaur2.js:97-118; tools/reference.py:296-297).
* ``dit_block_attention(...)``: one DiT block's attention step over the packed qkv buffer,
  headNorm(q, 2D rope) + headNorm(k, 2D rope) + headNorm(text k) + attention(bias, biasStart = L)
  (app/models/nanosaur2.js:196-208; tools/reference.py:272-286).  Also covers the odd, image-only
  blocks (no text rows).
* ``text_refine_attention(...)``: the text-refine blocks' attention (no RoPE, every text row is a
  query, app/models/nanosaur2.js:128-132; tools/reference.py:258-259).
* ``gemma_layer_attention(...)``: one Gemma3 layer's attention, headNorm(q), headNorm(k) with the
  local/global RoPE table + causal GQA 4/1 attention (app/models/gemma3.js:63-70;
  tools/reference.py:186-194), with an optional sliding window.
"""

from __future__ import annotations

import ctypes
import math
from typing import Optional, Sequence, Tuple

import torch

from . import _lib
from ._lib import FusedDesc, NsaError, check, lib
from .ops import RopeTable, dtype_code, stream_handle

DIT_HEADS, DIT_HEAD_DIM = 16, 96
GEMMA_HEADS, GEMMA_KV_HEADS, GEMMA_HEAD_DIM = 4, 1, 256


def gemma_rope_theta(layer: int) -> float:
    """Every 6th layer is global (theta 1e6), the others local (1e4) (app/models/gemma3.js:24)."""
    return 1e6 if (layer + 1) % 6 == 0 else 1e4


def prepare_text_bias(weights: Sequence[float]) -> Tuple[list, Optional[list]]:
    """Kept token indices and the log-weight key bias of the kept tokens, None when every kept weight
    is 1 (app/models/nanosaur2.js:97-118).  Tokens with w <= 0 are dropped (the reference's -inf
    bias, tools/reference.py:297)."""
    keep = [i for i, w in enumerate(weights) if w > 0]
    kept = [float(weights[i]) for i in keep]
    bias = None
    if any(w != 1 for w in kept):
        bias = [math.log(max(w, 1e-4)) for w in kept]
    return keep, bias


def _fused(qkv: torch.Tensor, *, Lq: int, Lk: int, Hq: int, Hkv: int, D: int, qOff: int, kOff: int, vOff: int,
           q_norm: torch.Tensor, k_norm: torch.Tensor, cs: Optional[RopeTable], kv_len: Optional[torch.Tensor],
           bias: Optional[torch.Tensor], biasStart: int, causal: bool, window: int, eps: float,
           out: Optional[torch.Tensor], out_dtype: Optional[torch.dtype], shard, workspace: Optional[torch.Tensor]):
    for t in (qkv, q_norm, k_norm, kv_len, bias, out):
        if t is not None and not t.is_cuda:
            raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, "tensors must live on a CUDA device")
    if qkv.dim() != 3:
        raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, "qkv must be [B, rows, ld]")
    if qkv.stride(-1) != 1:
        raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, "qkv rows must be contiguous")
    B = qkv.shape[0]
    if q_norm.dtype != torch.float32 or k_norm.dtype != torch.float32:
        raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, "norm weights must be float32")
    if kv_len is not None and kv_len.dtype != torch.int32:
        raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, "kv_len must be int32")
    if bias is not None and bias.dtype != torch.float32:
        raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, "bias must be float32")
    if out is None:
        odt = out_dtype or torch.bfloat16
        out = torch.empty((B, Lq, Hq * D), dtype=odt, device=qkv.device)
    d = FusedDesc()
    d.B, d.Lq, d.Lk, d.Hq, d.Hkv, d.D = B, Lq, Lk, Hq, Hkv, D
    d.ld, d.bstride = qkv.stride(1), qkv.stride(0)
    d.qOff, d.kOff, d.vOff = qOff, kOff, vOff
    d.in_dtype, d.out_dtype = dtype_code(qkv), dtype_code(out)
    d.eps = eps
    d.sinOff = cs.sinOff if cs is not None else 0
    d.causal, d.window = int(bool(causal)), window
    d.biasStart = biasStart
    d.biasLen = 0 if bias is None else bias.shape[-1]
    d.bias_bstride = bias.stride(0) if (bias is not None and bias.dim() == 2) else 0
    d.ldo, d.o_bstride, d.oOff = out.stride(1), out.stride(0), 0
    d.scale = 0.0
    if shard is not None:
        d.b_begin, d.b_count, d.h_begin, d.h_count = shard
    L = lib()
    ws_bytes = L.nsa_fused_attention_workspace_size(ctypes.byref(d))
    args = (qkv.data_ptr(), q_norm.data_ptr(), k_norm.data_ptr(), cs.buf.data_ptr() if cs is not None else None,
            None if kv_len is None else kv_len.data_ptr(), None if bias is None else bias.data_ptr(), out.data_ptr())
    if ws_bytes == 0:
        check(L.nsa_fused_attention(ctypes.byref(d), *args, None, 0, None))
    if workspace is None or workspace.numel() < ws_bytes:
        workspace = torch.empty(ws_bytes, dtype=torch.uint8, device=qkv.device)
    with torch.cuda.device(qkv.device):
        check(L.nsa_fused_attention(ctypes.byref(d), *args, workspace.data_ptr(), workspace.numel(),
                                    stream_handle(qkv.device)))
    return out


def fused_workspace_bytes(**kw) -> int:
    """Workspace size of a fused call with the same keyword arguments as ``dit_block_attention`` /
    ``gemma_layer_attention`` shapes (B, Lq, Lk, Hq, Hkv, D, shard)."""
    d = FusedDesc()
    d.B, d.Lq, d.Lk = kw["B"], kw["Lq"], kw["Lk"]
    d.Hq, d.Hkv, d.D = kw["Hq"], kw["Hkv"], kw["D"]
    d.in_dtype, d.out_dtype = kw.get("in_dtype", _lib.NSA_BF16), kw.get("out_dtype", _lib.NSA_BF16)
    d.causal, d.window = int(kw.get("causal", 0)), kw.get("window", 0)
    shard = kw.get("shard")
    if shard is not None:
        d.b_begin, d.b_count, d.h_begin, d.h_count = shard
    return lib().nsa_fused_attention_workspace_size(ctypes.byref(d))


def dit_block_attention(qkv: torch.Tensor, *, L: int, q_norm: torch.Tensor, k_norm: torch.Tensor,
                        cs: Optional[RopeTable], text_rows: int = 0, kv_len: Optional[torch.Tensor] = None,
                        bias: Optional[torch.Tensor] = None, eps: float = 1e-6, out: Optional[torch.Tensor] = None,
                        out_dtype: Optional[torch.dtype] = None, shard=None,
                        workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """qkv: [B, L + text_rows, 3*1536] with rows [0, L) image q|k|v and rows [L, L+text_rows) text k|v
    (app/models/nanosaur2.js:194-202).  kv_len[b] = L + valid text rows; bias: [B, text_rows] log prompt
    weights of the text keys (biasStart = L).  With text_rows = 0 this is an odd, image-only block.
    Returns [B, L, 1536]."""
    C = DIT_HEADS * DIT_HEAD_DIM
    return _fused(qkv, Lq=L, Lk=L + text_rows, Hq=DIT_HEADS, Hkv=DIT_HEADS, D=DIT_HEAD_DIM, qOff=0, kOff=C,
                  vOff=2 * C, q_norm=q_norm, k_norm=k_norm, cs=cs, kv_len=kv_len, bias=bias, biasStart=L,
                  causal=False, window=0, eps=eps, out=out, out_dtype=out_dtype, shard=shard, workspace=workspace)


def text_refine_attention(qkv: torch.Tensor, *, q_norm: torch.Tensor, k_norm: torch.Tensor,
                          keep_bias: Optional[torch.Tensor] = None, kv_len: Optional[torch.Tensor] = None,
                          eps: float = 1e-6, out: Optional[torch.Tensor] = None,
                          out_dtype: Optional[torch.dtype] = None, shard=None,
                          workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Attention of a text-refine block (app/models/nanosaur2.js:128-132; tools/reference.py:258-259):
    qkv [B, Lt, 3*1536], q/k RMSNorm without RoPE, every text row is a query and a key.  Dropped
    tokens are masked either by ``keep_bias`` [B, Lt] (0 / -inf on every key, the reference's
    keep_bias) or by ``kv_len`` (the JS path compacts the kept tokens to the front)."""
    C = DIT_HEADS * DIT_HEAD_DIM
    Lt = qkv.shape[1]
    return _fused(qkv, Lq=Lt, Lk=Lt, Hq=DIT_HEADS, Hkv=DIT_HEADS, D=DIT_HEAD_DIM, qOff=0, kOff=C, vOff=2 * C,
                  q_norm=q_norm, k_norm=k_norm, cs=None, kv_len=kv_len, bias=keep_bias, biasStart=0, causal=False,
                  window=0, eps=eps, out=out, out_dtype=out_dtype, shard=shard, workspace=workspace)


def gemma_layer_attention(qkv: torch.Tensor, *, q_norm: torch.Tensor, k_norm: torch.Tensor, cs: RopeTable,
                          window: int = 0, kv_len: Optional[torch.Tensor] = None, eps: float = 1e-6,
                          out: Optional[torch.Tensor] = None, out_dtype: Optional[torch.dtype] = None, shard=None,
                          workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """qkv: [B, Lt, 1536] = q 1024 | k 256 | v 256 (app/models/gemma3.js:63); q_norm / k_norm: the
    (w - 1) + 1 weights (gemma3.js:22); cs: the layer's 1D table (theta 1e4 local / 1e6 global).
    Causal GQA 4/1 over head dim 256, scale 1/16.  Returns [B, Lt, 1024]."""
    Lt = qkv.shape[1]
    H, KH, D = GEMMA_HEADS, GEMMA_KV_HEADS, GEMMA_HEAD_DIM
    return _fused(qkv, Lq=Lt, Lk=Lt, Hq=H, Hkv=KH, D=D, qOff=0, kOff=H * D, vOff=(H + KH) * D, q_norm=q_norm,
                  k_norm=k_norm, cs=cs, kv_len=kv_len, bias=None, biasStart=0, causal=True, window=window, eps=eps,
                  out=out, out_dtype=out_dtype, shard=shard, workspace=workspace)
