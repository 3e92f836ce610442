"""PyTorch CPU restatement of the reference's DiT attention step (TEST INFRASTRUCTURE ONLY).

Only ``bench.py``'s CPU legs (the ``cpu_baseline`` sample and the ``--impl reference`` arm) use this
module, as the timed CPU baseline; the CUDA library never calls it.  The reference computes this
step in PyTorch fp32 (``tools/reference.py``), and this file restates the same operator sequence
with the same torch calls, so the CPU figure is the reference's own CPU path rather than a numpy
loop:

  * ``rms_norm`` / ``rope_split_half`` (tools/reference.py:96-104);
  * the block's q/k prologue, per-head RMSNorm then split-half RoPE on the image rows, RMSNorm only on
    the text keys (tools/reference.py:272-282);
  * ``attention``: heads split off, ``F.scaled_dot_product_attention`` with the additive key bias
    broadcast over the query rows (tools/reference.py:230-237).

``tools/reference.py`` itself cannot be imported on the GPU box (the reference tree is not there),
which is why the operator sequence is restated here; ``tests/test_oracle_golden.py`` checks this
restatement against the numpy oracle, which the reference's own outputs pin.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

HEADS, HD = 16, 96   # tools/reference.py:205
D = HEADS * HD


def rms_norm(x, w, eps=1e-6):
    """x * rsqrt(mean(x^2) + eps) * w over the last axis (tools/reference.py:96-97)."""
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


def rope_split_half(x, cos, sin):
    """x [..., L, D]; pair i is (x[i], x[i + D/2]); cos/sin [L, D/2] (tools/reference.py:100-104)."""
    h = x.shape[-1] // 2
    x1, x2 = x[..., :h], x[..., h:]
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1)


def rope_rows(t, w, cos, sin):
    """Per-head RMSNorm then RoPE of rows [L, 1536] (the block's ``rope``, tools/reference.py:276-278)."""
    L = t.shape[0]
    th = rms_norm(t.view(L, HEADS, HD), w).transpose(0, 1)
    return rope_split_half(th, cos, sin).transpose(0, 1).reshape(L, D)


def head_norm(x, w):
    """Per-head RMSNorm without RoPE (tools/reference.py:240-241)."""
    return rms_norm(x.view(x.shape[0], HEADS, HD), w).view(x.shape[0], D)


def attention(q, k, v, bias=None):
    """q [Lq, 1536], k/v [Lk, 1536], bias [Lk] additive -> [Lq, 1536] (tools/reference.py:230-237)."""
    qh = q.view(q.shape[0], HEADS, HD).transpose(0, 1)
    kh = k.view(k.shape[0], HEADS, HD).transpose(0, 1)
    vh = v.view(v.shape[0], HEADS, HD).transpose(0, 1)
    mask = None if bias is None else bias[None, None, :].expand(1, q.shape[0], -1)
    o = F.scaled_dot_product_attention(qh[None], kh[None], vh[None], attn_mask=mask)[0]
    return o.transpose(0, 1).reshape(q.shape[0], D)


@torch.no_grad()
def joint_attention_step(qkv, L, n, q_w, k_w, cos, sin, txt_bias, q_rows=None):
    """One DiT block's attention step on one batch element of the packed buffer the CUDA path takes:
    qkv [L + Lt, 4608] fp32 (image rows q|k|v, text rows -|k|v), n = L + valid text rows, txt_bias
    [n - L].  ``q_rows`` (int) limits the queries to the first rows (a bounded CPU sample); every key
    is still normalised and rotated.  Returns [q_rows or L, 1536]."""
    r = L if q_rows is None else q_rows
    q = rope_rows(qkv[:r, :D], q_w, cos[:r], sin[:r])
    k = rope_rows(qkv[:L, D:2 * D], k_w, cos, sin)
    v = qkv[:n, 2 * D:]
    bias = None
    if n > L:
        k = torch.cat([k, head_norm(qkv[L:n, D:2 * D], k_w)])
        bias = torch.cat([torch.zeros(L, dtype=qkv.dtype), txt_bias[: n - L]])
    return attention(q, k, v, bias)
