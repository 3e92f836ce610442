"""The model call sites of the attention hot path, as fused single calls into libnsattn.so.

* ``prepare_text_bias(weights)``: the per-text-key log-weight bias and the dropped (w <= 0) tokens of
  ``Nanosaur2DiT.prepareText`` (app/models/nanosaur2.js:97-118; tools/reference.py:296-297).
* ``dit_block_attention(...)``: one DiT block's attention step over the packed qkv buffer,
  headNorm(q, 2D rope) + headNorm(k, 2D rope) + headNorm(text k) + attention(bias, biasStart = L)
  (app/models/nanosaur2.js:196-208; tools/reference.py:272-286).  Also covers the odd, image-only
  blocks (no text rows).
* ``text_refine_attention(...)``: the text-refine blocks' attention (no RoPE, every text row is a
  query, app/models/nanosaur2.js:128-132; tools/reference.py:258-259).
* ``dit_block_attention_projected(...)``: the same DiT step from the block input instead of qkv:
  ops.linear `dit.qkv` + `dit.kv_y` (app/models/nanosaur2.js:197-201; tools/reference.py:208-210,
  272, 282) as one tcgen05 GEMM per row set whose epilogue applies the bias, the q/k RMSNorm and the
  RoPE and writes the attention's inputs (nsa_seq_shard_projection), then the attention
  (nsa_seq_shard_attention).
* ``gemma_layer_attention_projected(...)``: the Gemma layer's attention from its normalised input
  rows: the ``te.qkv`` linear with the q/k norms and RoPE in the GEMM epilogue, then the causal
  attention over the prepared tiles.
* ``gemma_attention_sublayer(...)``: the attention half of a Gemma layer on its fp32 residual stream
  (app/models/gemma3.js:62-77; tools/reference.py:187-196): input RMSNorm to a bf16 operand, the
  projected attention above, the ``te.o`` linear, and the post-attention RMSNorm added into the
  stream, five launches.
* ``gemma_mlp_sublayer(...)`` / ``gemma_layer(...)``: the MLP half (app/models/gemma3.js:78-89: pre-MLP
  RMSNorm, gate_up linear, GELU-tanh GLU, down linear, post-MLP RMSNorm accumulated) and the whole
  layer, attention half then MLP half.
* ``vae_attention(...)``: the VAE decoder's single-head attention over all latent pixels, head dim C
  = 512 (app/models/vae.js:77-88; tools/reference.py:352-357): ``ops.attention`` with H = 1, D = C on
  the packed qkv rows of the group-normed input.
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
from ._lib import FusedDesc, NsaError, ProjDesc, SeqShard, check, lib
from .ops import RopeTable, dtype_code, glu, linear, rmsnorm, stream_handle

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
           out: Optional[torch.Tensor], out_dtype: Optional[torch.dtype], shard, workspace: Optional[torch.Tensor],
           compute: int = _lib.NSA_COMPUTE_BF16):
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
    d.compute = compute
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
    d.compute = kw.get("compute", _lib.NSA_COMPUTE_BF16)
    shard = kw.get("shard")
    if shard is not None:
        d.b_begin, d.b_count, d.h_begin, d.h_count = shard
    return lib().nsa_fused_attention_workspace_size(ctypes.byref(d))


def dit_block_attention(qkv: torch.Tensor, *, L: int, q_norm: torch.Tensor, k_norm: torch.Tensor,
                        cs: Optional[RopeTable], text_rows: int = 0, kv_len: Optional[torch.Tensor] = None,
                        bias: Optional[torch.Tensor] = None, eps: float = 1e-6, out: Optional[torch.Tensor] = None,
                        out_dtype: Optional[torch.dtype] = None, shard=None,
                        workspace: Optional[torch.Tensor] = None, tf32: bool = False) -> torch.Tensor:
    """qkv: [B, L + text_rows, 3*1536] with rows [0, L) image q|k|v and rows [L, L+text_rows) text k|v
    (app/models/nanosaur2.js:194-202).  kv_len[b] = L + valid text rows; bias: [B, text_rows] log prompt
    weights of the text keys (biasStart = L).  With text_rows = 0 this is an odd, image-only block.
    ``tf32`` (fp32 qkv only): keep the prepared q/k/v in fp32 and multiply at tf32 precision, the
    closer match to the reference's fp32 math (NSA_COMPUTE_TF32).  Returns [B, L, 1536]."""
    C = DIT_HEADS * DIT_HEAD_DIM
    return _fused(qkv, Lq=L, Lk=L + text_rows, Hq=DIT_HEADS, Hkv=DIT_HEADS, D=DIT_HEAD_DIM, qOff=0, kOff=C,
                  vOff=2 * C, q_norm=q_norm, k_norm=k_norm, cs=cs, kv_len=kv_len, bias=bias, biasStart=L,
                  causal=False, window=0, eps=eps, out=out, out_dtype=out_dtype, shard=shard, workspace=workspace,
                  compute=_lib.NSA_COMPUTE_TF32 if tf32 else _lib.NSA_COMPUTE_BF16)


def projection_buffers(B: int, L: int, text_rows: int, device) -> Tuple[torch.Tensor, torch.Tensor]:
    """q_prime (uint8, the q' tiles of all B elements then the split scratch) and kv_packed
    [B, kv_rows, 2*1536] (bf16) of a one-GPU DiT block."""
    d = FusedDesc()
    d.B, d.Lq, d.Lk, d.Hq, d.Hkv, d.D = B, L, L + text_rows, DIT_HEADS, DIT_HEADS, DIT_HEAD_DIM
    d.in_dtype = d.out_dtype = _lib.NSA_BF16
    d.b_begin, d.b_count = 0, B
    s = SeqShard(0, L, 0, 0)
    qb, kb, rows = ctypes.c_size_t(), ctypes.c_size_t(), ctypes.c_int32()
    check(lib().nsa_seq_shard_buffer_sizes(ctypes.byref(d), ctypes.byref(s), ctypes.byref(qb), ctypes.byref(kb),
                                           ctypes.byref(rows)))
    q_prime = torch.empty(qb.value, dtype=torch.uint8, device=device)
    kv_packed = torch.empty((B, rows.value, 2 * DIT_HEADS * DIT_HEAD_DIM), dtype=torch.bfloat16, device=device)
    return q_prime, kv_packed


def dit_block_attention_projected(x: torch.Tensor, *, w_qkv: torch.Tensor, b_qkv: Optional[torch.Tensor],
                                  q_norm: torch.Tensor, k_norm: torch.Tensor, cs: Optional[RopeTable],
                                  x_text: Optional[torch.Tensor] = None, w_kv: Optional[torch.Tensor] = None,
                                  b_kv: Optional[torch.Tensor] = None, kv_len: Optional[torch.Tensor] = None,
                                  bias: Optional[torch.Tensor] = None, eps: float = 1e-6,
                                  out: Optional[torch.Tensor] = None, out_dtype: Optional[torch.dtype] = None,
                                  buffers: Optional[Tuple[torch.Tensor, torch.Tensor]] = None,
                                  w_qkv_scale: Optional[torch.Tensor] = None, w_kv_scale: Optional[torch.Tensor] = None,
                                  lora_qkv=None, lora_kv=None) -> torch.Tensor:
    """One DiT block's attention step from its input rows (app/models/nanosaur2.js:196-208):
    x [B, L, K] bf16 (the modulated block input), w_qkv [3*1536, K] bf16 and b_qkv [3*1536] fp32
    (``attn.qkv_x``), x_text [B, text_rows, K] with w_kv [2*1536, K] / b_kv (``attn.kv_y``) for the
    text keys.  kv_len[b] = L + valid text rows; bias [B, text_rows] log prompt weights.
    ``buffers`` = projection_buffers(...) to reuse across calls.  Returns [B, L, 1536].
    int8 ConvRot weights: pass ``ops.expand_i8(W)`` as the weight, its row scales as ``w_*_scale``, and
    rotated inputs (``ops.rotate``).  LoRA side paths: ``ops.lora_pack`` results for either weight
    (packed with the same scales)."""
    tensors = (x, w_qkv, b_qkv, q_norm, k_norm, x_text, w_kv, b_kv, kv_len, bias, out, w_qkv_scale, w_kv_scale)
    if any(t is not None and not t.is_cuda for t in tensors):
        raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, "tensors must live on a CUDA device")
    if x.dim() != 3 or x.stride(-1) != 1 or x.dtype != torch.bfloat16:
        raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, "x must be a bf16 [B, L, K] tensor with contiguous rows")
    if not w_qkv.is_contiguous() or (w_kv is not None and not w_kv.is_contiguous()):
        raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, "weights must be contiguous [out, K]")
    if kv_len is not None and kv_len.dtype != torch.int32:
        raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, "kv_len must be int32")
    B, L, K = x.shape
    text_rows = 0 if x_text is None else x_text.shape[1]
    C = DIT_HEADS * DIT_HEAD_DIM
    if out is None:
        out = torch.empty((B, L, C), dtype=out_dtype or torch.bfloat16, device=x.device)
    q_prime, kv_packed = buffers if buffers is not None else projection_buffers(B, L, text_rows, x.device)
    d = FusedDesc()
    d.B, d.Lq, d.Lk, d.Hq, d.Hkv, d.D = B, L, L + text_rows, DIT_HEADS, DIT_HEADS, DIT_HEAD_DIM
    d.qOff, d.kOff, d.vOff = 0, C, 2 * C
    d.in_dtype, d.out_dtype = _lib.NSA_BF16, dtype_code(out)
    d.ldo, d.o_bstride, d.oOff = out.stride(1), out.stride(0), 0
    d.eps = eps
    d.sinOff = cs.sinOff if cs is not None else 0
    d.biasStart = L
    d.biasLen = 0 if bias is None else bias.shape[-1]
    d.bias_bstride = bias.stride(0) if (bias is not None and bias.dim() == 2) else 0
    s = SeqShard(0, L, 0, 0)
    p = ProjDesc()
    p.K = K
    p.x, p.ldx, p.x_bstride, p.x_rows = x.data_ptr(), x.stride(1), x.stride(0), L
    p.w_qkv, p.b_qkv = w_qkv.data_ptr(), None if b_qkv is None else b_qkv.data_ptr()
    if x_text is not None:
        p.x_text, p.ld_text, p.text_bstride, p.text_rows = x_text.data_ptr(), x_text.stride(1), x_text.stride(0), text_rows
        p.w_kv, p.b_kv = w_kv.data_ptr(), None if b_kv is None else b_kv.data_ptr()
    for sc in (w_qkv_scale, w_kv_scale):
        if sc is not None and (sc.dtype != torch.float32 or not sc.is_contiguous()):
            raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, "weight scales must be contiguous float32")
    p.w_qkv_scale = None if w_qkv_scale is None else w_qkv_scale.data_ptr()
    p.w_kv_scale = None if w_kv_scale is None else w_kv_scale.data_ptr()
    lora_t = None
    if lora_qkv is not None or (lora_kv is not None and x_text is not None):
        rq = lora_qkv.R if lora_qkv is not None else 0
        rk = lora_kv.R if (lora_kv is not None and x_text is not None) else 0
        lora_t = torch.empty(B * L * rq + B * text_rows * rk, dtype=torch.bfloat16, device=x.device)
        if rq:
            p.lora_rank_qkv, p.lora_a_qkv, p.lora_b_qkv = rq, lora_qkv.a.data_ptr(), lora_qkv.b.data_ptr()
        if rk:
            p.lora_rank_kv, p.lora_a_kv, p.lora_b_kv = rk, lora_kv.a.data_ptr(), lora_kv.b.data_ptr()
        p.lora_t = lora_t.data_ptr()
    d.b_begin, d.b_count = 0, B
    L_ = lib()
    with torch.cuda.device(x.device):
        stream = stream_handle(x.device)
        check(L_.nsa_seq_shard_projection(ctypes.byref(d), ctypes.byref(s), ctypes.byref(p), q_norm.data_ptr(),
                                          k_norm.data_ptr(), cs.buf.data_ptr() if cs is not None else None,
                                          None if kv_len is None else kv_len.data_ptr(), q_prime.data_ptr(),
                                          kv_packed.data_ptr(), stream))
        check(L_.nsa_seq_shard_attention(ctypes.byref(d), ctypes.byref(s), q_prime.data_ptr(), kv_packed.data_ptr(),
                                         None if kv_len is None else kv_len.data_ptr(),
                                         None if bias is None else bias.data_ptr(), out.data_ptr(), stream))
    return out


def gemma_projection_buffers(B: int, L: int, device) -> Tuple[torch.Tensor, torch.Tensor]:
    """q_prime (uint8) and kv_packed [B, kv_rows, 2*256] (bf16) of a Gemma layer from its input rows."""
    d = FusedDesc()
    d.B, d.Lq, d.Lk, d.Hq, d.Hkv, d.D = B, L, L, GEMMA_HEADS, GEMMA_KV_HEADS, GEMMA_HEAD_DIM
    d.in_dtype = d.out_dtype = _lib.NSA_BF16
    d.causal = 1
    d.b_begin, d.b_count = 0, B
    s = SeqShard(0, L, 0, 0)
    qb, kb, rows = ctypes.c_size_t(), ctypes.c_size_t(), ctypes.c_int32()
    check(lib().nsa_seq_shard_buffer_sizes(ctypes.byref(d), ctypes.byref(s), ctypes.byref(qb), ctypes.byref(kb),
                                           ctypes.byref(rows)))
    return (torch.empty(qb.value, dtype=torch.uint8, device=device),
            torch.empty((B, rows.value, 2 * GEMMA_KV_HEADS * GEMMA_HEAD_DIM), dtype=torch.bfloat16, device=device))


def gemma_layer_attention_projected(x: torch.Tensor, *, w_qkv: torch.Tensor, q_norm: torch.Tensor,
                                    k_norm: torch.Tensor, cs: RopeTable, window: int = 0, eps: float = 1e-6,
                                    out: Optional[torch.Tensor] = None, out_dtype: Optional[torch.dtype] = None,
                                    buffers: Optional[Tuple[torch.Tensor, torch.Tensor]] = None) -> torch.Tensor:
    """One Gemma3 layer's attention from the layer's normalised input rows (app/models/gemma3.js:62-70):
    qkv = h W_qkv^T (``te.qkv``, no bias; W_qkv [(4 + 2) * 256, K] bf16, rows q heads then k then v)
    as one tcgen05 GEMM whose epilogue applies the q/k RMSNorm and the layer's 1D RoPE
    (nsa_seq_shard_projection), then causal GQA 4/1 attention with an optional sliding window over
    the prepared tiles (nsa_seq_shard_attention with the full-sequence shard).  x [B, L, K] bf16.
    ``buffers`` = gemma_projection_buffers(B, L, device), to reuse.  Returns [B, L, 1024]."""
    tensors = (x, w_qkv, q_norm, k_norm, out)
    if any(t is not None and not t.is_cuda for t in tensors):
        raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, "tensors must live on a CUDA device")
    if x.dim() != 3 or x.stride(-1) != 1 or x.dtype != torch.bfloat16 or not w_qkv.is_contiguous():
        raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, "x must be bf16 [B, L, K] with contiguous rows, w_qkv contiguous")
    B, L, K = x.shape
    H, KH, D = GEMMA_HEADS, GEMMA_KV_HEADS, GEMMA_HEAD_DIM
    if out is None:
        out = torch.empty((B, L, H * D), dtype=out_dtype or torch.bfloat16, device=x.device)
    d = FusedDesc()
    d.B, d.Lq, d.Lk, d.Hq, d.Hkv, d.D = B, L, L, H, KH, D
    d.qOff, d.kOff, d.vOff = 0, H * D, (H + KH) * D
    d.in_dtype, d.out_dtype = _lib.NSA_BF16, dtype_code(out)
    d.ldo, d.o_bstride, d.oOff = out.stride(1), out.stride(0), 0
    d.eps = eps
    d.sinOff = cs.sinOff
    d.causal, d.window = 1, window
    d.b_begin, d.b_count = 0, B
    s = SeqShard(0, L, 0, 0)
    L_ = lib()
    q_prime, kv_packed = buffers if buffers is not None else gemma_projection_buffers(B, L, x.device)
    p = ProjDesc()
    p.K = K
    p.x, p.ldx, p.x_bstride, p.x_rows = x.data_ptr(), x.stride(1), x.stride(0), L
    p.w_qkv = w_qkv.data_ptr()
    with torch.cuda.device(x.device):
        stream = stream_handle(x.device)
        check(L_.nsa_seq_shard_projection(ctypes.byref(d), ctypes.byref(s), ctypes.byref(p), q_norm.data_ptr(),
                                          k_norm.data_ptr(), cs.buf.data_ptr(), None, q_prime.data_ptr(),
                                          kv_packed.data_ptr(), stream))
        check(L_.nsa_seq_shard_attention(ctypes.byref(d), ctypes.byref(s), q_prime.data_ptr(), kv_packed.data_ptr(),
                                         None, None, out.data_ptr(), stream))
    return out


def gemma_sublayer_buffers(B: int, L: int, hidden: int, device) -> dict:
    """Intermediates of ``gemma_attention_sublayer``: the normalised input h (bf16 [B, L, hidden]),
    the projection's q_prime / kv_packed, the attention output a (bf16 [B, L, 1024]) and the te.o
    output o (fp32 [B*L, hidden])."""
    return {"h": torch.empty((B, L, hidden), dtype=torch.bfloat16, device=device),
            "proj": gemma_projection_buffers(B, L, device),
            "a": torch.empty((B, L, GEMMA_HEADS * GEMMA_HEAD_DIM), dtype=torch.bfloat16, device=device),
            "o": torch.empty((B * L, hidden), dtype=torch.float32, device=device)}


def gemma_attention_sublayer(x: torch.Tensor, *, in_norm: torch.Tensor, w_qkv: torch.Tensor, q_norm: torch.Tensor,
                             k_norm: torch.Tensor, w_o: torch.Tensor, post_norm: torch.Tensor, cs: RopeTable,
                             window: int = 0, eps: float = 1e-6, buffers: Optional[dict] = None,
                             h_ready: bool = False, next_norm: Optional[torch.Tensor] = None,
                             next_out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """The attention half of one Gemma3 layer, in place on the residual stream x (fp32 [B, L, hidden])
    (app/models/gemma3.js:62-77; tools/reference.py:187-196):
        h = rmsnorm(x, in_norm)                       nsa_rmsnorm, bf16 output
        a = attention(headNorm(h W_qkv^T))            nsa_seq_shard_projection + nsa_seq_shard_attention
        x += rmsnorm(a W_o^T, post_norm)              nsa_linear (te.o) + nsa_rmsnorm accumulate
    w_qkv [1536, hidden] and w_o [hidden, 1024] bf16; norm weights fp32, lifted by +1 (gemma3.js:22).
    ``buffers`` = gemma_sublayer_buffers(B, L, hidden, device), to reuse.  Chaining (the norms the
    layer runs back to back, in one pass each): ``h_ready`` means buffers["h"] already holds
    rmsnorm(x, in_norm) (written by the previous accumulate); ``next_norm`` makes the final accumulate
    also write next_out = rmsnorm(x after the add, next_norm) (bf16).  Returns x."""
    if x.dim() != 3 or x.dtype != torch.float32 or not x.is_contiguous():
        raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, "x must be a contiguous float32 [B, L, hidden] tensor")
    B, L, hidden = x.shape
    if w_o.shape != (hidden, GEMMA_HEADS * GEMMA_HEAD_DIM):
        raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, "w_o must be [hidden, 1024]")
    buf = buffers if buffers is not None else gemma_sublayer_buffers(B, L, hidden, x.device)
    h, a, o = buf["h"], buf["a"], buf["o"]
    if not h_ready:
        rmsnorm(x, in_norm, hidden, eps, h)
    gemma_layer_attention_projected(h, w_qkv=w_qkv, q_norm=q_norm, k_norm=k_norm, cs=cs, window=window, eps=eps,
                                    out=a, buffers=buf["proj"])
    linear(a.view(B * L, -1), w_o, out=o)
    rmsnorm(o, post_norm, hidden, eps, x.view(B * L, hidden), accumulate=True, next_weight=next_norm,
            next_out=None if next_norm is None else next_out.view(B * L, hidden))
    return x


def gemma_mlp_buffers(B: int, L: int, hidden: int, inter: int, device, gate_up_interleaved: bool = False) -> dict:
    """Intermediates of ``gemma_mlp_sublayer``: h2 (bf16 [B*L, hidden]), gu (fp32 [B*L, 2*inter]; not
    needed when the GLU runs in the gate_up linear's epilogue), g (bf16 [B*L, inter]) and d (fp32
    [B*L, hidden])."""
    M = B * L
    buf = {"h": torch.empty((M, hidden), dtype=torch.bfloat16, device=device),
           "g": torch.empty((M, inter), dtype=torch.bfloat16, device=device),
           "d": torch.empty((M, hidden), dtype=torch.float32, device=device)}
    if not gate_up_interleaved:
        buf["gu"] = torch.empty((M, 2 * inter), dtype=torch.float32, device=device)
    return buf


def gemma_mlp_sublayer(x: torch.Tensor, *, pre_norm: torch.Tensor, w_gate_up: torch.Tensor, w_down: torch.Tensor,
                       post_norm: torch.Tensor, eps: float = 1e-6, buffers: Optional[dict] = None,
                       gate_up_interleaved: bool = False, h_ready: bool = False,
                       next_norm: Optional[torch.Tensor] = None, next_out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """The MLP half of one Gemma3 layer, in place on the residual stream x (fp32 [B, L, hidden])
    (app/models/gemma3.js:78-89; tools/reference.py:197-199):
        h2 = rmsnorm(x, pre_norm)                     nsa_rmsnorm, bf16 output
        g  = gelu_tanh(h2 W_gate^T) * (h2 W_up^T)     nsa_linear (gate_up) + nsa_glu, bf16 output
        x += rmsnorm(g W_down^T, post_norm)           nsa_linear (down) + nsa_rmsnorm accumulate
    w_gate_up [2*inter, hidden] (gate rows, then up rows: the reference's concatLinears, gemma3.js:33)
    and w_down [hidden, inter] bf16; norm weights fp32, lifted by +1.  With ``gate_up_interleaved``
    w_gate_up is in ``glu_interleave`` order (inter a multiple of 128) and the GLU runs in the gate_up
    linear's epilogue: g is written straight from the accumulator, without the fp32 gu.  ``h_ready`` /
    ``next_norm`` / ``next_out`` chain the norms as in ``gemma_attention_sublayer`` (buffers["h"] holds
    rmsnorm(x, pre_norm) already; the final accumulate also writes the next layer's normalised input).
    Returns x."""
    if x.dim() != 3 or x.dtype != torch.float32 or not x.is_contiguous():
        raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, "x must be a contiguous float32 [B, L, hidden] tensor")
    B, L, hidden = x.shape
    if w_gate_up.dim() != 2 or w_gate_up.shape[1] != hidden or w_gate_up.shape[0] % 2:
        raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, "w_gate_up must be [2*inter, hidden]")
    inter = w_gate_up.shape[0] // 2
    if w_down.shape != (hidden, inter):
        raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, "w_down must be [hidden, inter]")
    buf = buffers if buffers is not None else gemma_mlp_buffers(B, L, hidden, inter, x.device, gate_up_interleaved)
    xs = x.view(B * L, hidden)
    if not h_ready:
        rmsnorm(xs, pre_norm, hidden, eps, buf["h"])
    if gate_up_interleaved:
        linear(buf["h"], w_gate_up, out=buf["g"], glu="gelu_tanh")
    else:
        linear(buf["h"], w_gate_up, out=buf["gu"])
        glu(buf["gu"], "gelu_tanh", out=buf["g"])
    linear(buf["g"], w_down, out=buf["d"])
    rmsnorm(buf["d"], post_norm, hidden, eps, xs, accumulate=True, next_weight=next_norm,
            next_out=None if next_norm is None else next_out.view(B * L, hidden))
    return x


def gemma_layer(x: torch.Tensor, *, attn: dict, mlp: dict, cs: RopeTable, window: int = 0, eps: float = 1e-6,
                buffers: Optional[Tuple[dict, dict]] = None, h_ready: bool = False,
                next_norm: Optional[torch.Tensor] = None) -> torch.Tensor:
    """One whole Gemma3 layer in place on x (app/models/gemma3.js:62-89): ``gemma_attention_sublayer(x,
    **attn)`` then ``gemma_mlp_sublayer(x, **mlp)``, with the post-attention accumulate also writing
    the MLP's normalised input (one pass for gemma3.js:74-79).  ``buffers`` = (gemma_sublayer_buffers(...),
    gemma_mlp_buffers(...)), to reuse.  Across layers: ``next_norm`` (the next layer's in_norm) makes
    the post-MLP accumulate write the next layer's normalised input into buffers[0]["h"], and the next
    call passes ``h_ready=True``."""
    B, L, hidden = x.shape
    if buffers is None:
        inter = mlp["w_down"].shape[1]
        buffers = (gemma_sublayer_buffers(B, L, hidden, x.device),
                   gemma_mlp_buffers(B, L, hidden, inter, x.device, mlp.get("gate_up_interleaved", False)))
    ab, mb = buffers
    gemma_attention_sublayer(x, **attn, cs=cs, window=window, eps=eps, buffers=ab, h_ready=h_ready,
                             next_norm=mlp["pre_norm"], next_out=mb["h"])
    return gemma_mlp_sublayer(x, **mlp, eps=eps, buffers=mb, h_ready=True, next_norm=next_norm,
                              next_out=ab["h"] if next_norm is not None else None)


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


def vae_attention(qkv: torch.Tensor, *, C: int = 512, out: Optional[torch.Tensor] = None,
                  out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    """The VAE decoder's attention call (app/models/vae.js:82): one head of dim C over all hw pixels of
    the packed q|k|v rows [hw, 3C] (or [B, hw, 3C]) that the qkv linear of the group-normed input
    writes; scale 1/sqrt(C); returns [hw, C].  Head dim 512 runs on the kernel that splits each query
    tile's output columns over two CTAs."""
    from .ops import attention
    hw = qkv.shape[-2]
    if qkv.shape[-1] != 3 * C:
        raise NsaError(_lib.NSA_ERR_INVALID_ARGUMENT, "qkv rows must hold q | k | v of C channels each")
    return attention(q=qkv, k=qkv, v=qkv, Lq=hw, Lk=hw, H=1, D=C, ldq=3 * C, ldk=3 * C, ldv=3 * C, qOff=0, kOff=C,
                     vOff=2 * C, out=out, out_dtype=out_dtype)
