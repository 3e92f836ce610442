"""CPU oracle for the Nanosaur2 attention hot path (TEST INFRASTRUCTURE ONLY).

This module is the checker, never the product: only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import it.  The CUDA library under
``nanosaur2_web_b200/`` never calls into it and has no CPU fallback.

It restates, in numpy, the fp32 PyTorch reference of the attention path in the Nanosaur2 web app
(``tools/reference.py``) and the JS conventions the WGSL kernels follow (``app/gpu/kernels.js``,
``app/models/common.js``, ``app/models/nanosaur2.js``, ``app/models/gemma3.js``).  Every function
cites the reference lines it follows.  Parity of this restatement is pinned by
``tests/test_oracle_golden.py`` against fixtures produced by running the reference's own DiT block,
text-refine block and Gemma encoder code (``tests/golden/make_golden.py``).

The one convention the reference never exercises is Gemma's 512-token sliding window (its text is
capped at 256 tokens, ``app/models/gemma3.js:5-7``); this oracle states it as: key j is visible to
query i iff ``i - window < j <= i``.  That case is parity-unpinned.

All functions take and return ``np.ndarray``.  ``acc`` selects the accumulation dtype
(``np.float32`` mirrors the reference, ``np.float64`` gives a tighter truth for kernel checks).
"""

from __future__ import annotations

import math

import numpy as np

DIT_HEADS, DIT_HEAD_DIM = 16, 96          # tools/reference.py:205
GEMMA_HEADS, GEMMA_KV_HEADS, GEMMA_HEAD_DIM = 4, 1, 256   # tools/reference.py:178


# ----------------------------------------------------------------------------- projection

def linear(x, w, b=None, acc=np.float32):
    """The reference's lin / ops.linear (tools/reference.py:208-210; app/gpu/ops.js:50-66 with
    app/gpu/gemm.js:141): y = x @ W^T (+ b), W in the Linear layout [out features][in features]."""
    y = np.asarray(x, acc) @ np.asarray(w, acc).T
    return y + np.asarray(b, acc) if b is not None else y


def linear_epilogue(y, out=None, gate=None, resid=False, act=None, acc=np.float32):
    """The epilogue of the reference's tiled GEMM (app/gpu/gemm.js:155-165) after ``linear``:
    silu when act == "silu", then out = y, out += y (resid) or out += gate * y (resid with a gate, the
    DiT block's gated residual x + m[2] * lin(...), tools/reference.py:285)."""
    y = np.asarray(y, acc)
    if act == "silu":
        y = y / (1.0 + np.exp(-y))
    if not resid:
        return y
    g = 1.0 if gate is None else np.asarray(gate, acc)
    return np.asarray(out, acc) + g * y


# ----------------------------------------------------------------------------- int8 ConvRot and LoRA

CONVROT_GROUP = 256   # tools/quant.py:18


def hadamard(n=CONVROT_GROUP, acc=np.float32):
    """The normalised regular Hadamard matrix of tools/quant.py:21-30: Kronecker powers of
    H4 = [[1,1,1,-1],[1,1,-1,1],[1,-1,1,1],[-1,1,1,1]], divided by sqrt(n) (n a power of 4)."""
    h4 = np.array([[1, 1, 1, -1], [1, 1, -1, 1], [1, -1, 1, 1], [-1, 1, 1, 1]], dtype=acc)
    h = h4
    while h.shape[0] < n:
        h = np.kron(h, h4)
    if h.shape[0] != n:
        raise ValueError(f"size must be a power of 4, got {n}")
    return h / acc(math.sqrt(n))


def rotate(x, group=CONVROT_GROUP, acc=np.float32):
    """ConvRot rotation of the last axis in groups of 256 (ops.rotate, app/gpu/ops.js:38-45, and the
    hadamard kernel, app/gpu/kernels.js:379-407; tools/quant.py:33-37 for weights): y = x @ H^T per
    group, H symmetric."""
    x = np.asarray(x, acc)
    k = x.shape[-1]
    h = hadamard(group, acc)
    return (x.reshape(*x.shape[:-1], k // group, group) @ h.T).reshape(x.shape)


def quantize_int8_convrot(w):
    """tools/quant.py:48-57: per-output-row int8 of the rotated weight; returns (q int8 [N][K],
    scale float32 [N]).  Rounding is to nearest even, as torch.round."""
    rot = rotate(np.asarray(w, np.float32), acc=np.float32)
    scale = np.maximum(np.abs(rot).max(axis=1, keepdims=True) / np.float32(127.0), np.float32(1e-30))
    q = np.clip(np.round(rot / scale), -128, 127).astype(np.int8)
    return q, scale.reshape(-1).astype(np.float32)


def linear_int8(xr, q, scale, b=None, acc=np.float32):
    """The reference's GEMM with an "i8" B (app/gpu/gemm.js:10, 119-130, epilogue 159-160): the int8
    weights are read as exact integers, the row's dot product times scale[n], then the bias.  xr is the
    rotated input (app/gpu/ops.js:54)."""
    y = (np.asarray(xr, acc) @ np.asarray(q, acc).T) * np.asarray(scale, acc)
    return y + np.asarray(b, acc) if b is not None else y


def lora_delta(x, entries, N, acc=np.float32):
    """delta = sum_i scale_i * B_i (A_i x) over output columns [off_i, off_i + n_i)
    (app/gpu/ops.js:70-86; entries as app/lora.js:143-150 builds them: dicts with A [r][K], B [n][r],
    scale, off, n).  For int8 layers A's rows are rotated and x is the rotated input."""
    x = np.asarray(x, acc)
    d = np.zeros((x.shape[0], N), acc)
    for e in entries:
        off = int(e.get("off", 0))
        B = np.asarray(e["B"], acc)
        d[:, off:off + B.shape[0]] += acc(e["scale"]) * ((x @ np.asarray(e["A"], acc).T) @ B.T)
    return d


# ----------------------------------------------------------------------------- prologue pieces

def rms_norm(x, w, eps=1e-6, acc=np.float32):
    """y = x * rsqrt(mean(x^2) + eps) * w over the last axis (tools/reference.py:96-97)."""
    x = np.asarray(x, dtype=acc)
    r = 1.0 / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + acc(eps))
    return x * r * np.asarray(w, dtype=acc)


def rope_split_half(x, cos, sin, acc=np.float32):
    """Split-half rotary embedding: pair i is (x[i], x[i + D/2]); cos/sin [L, D/2]
    (tools/reference.py:100-104; app/gpu/kernels.js:333-339)."""
    x = np.asarray(x, dtype=acc)
    h = x.shape[-1] // 2
    x1, x2 = x[..., :h], x[..., h:]
    c = np.asarray(cos, dtype=acc)
    s = np.asarray(sin, dtype=acc)
    return np.concatenate([x1 * c - x2 * s, x2 * c + x1 * s], axis=-1)


def inv_freq(D, theta):
    """1 / theta^(2i/D) for i < D/2, rounded to fp32 the way app/models/common.js:15 does it: the
    exponent 2i/D is rounded to fp32, the power and reciprocal are taken in double precision and the
    result is rounded to fp32.  (tools/reference.py:170,222 takes the power in fp32; the two differ
    by at most one fp32 ulp.)"""
    e = (np.arange(0, D, 2, dtype=np.float64) / D).astype(np.float32).astype(np.float64)
    return (1.0 / np.power(np.float64(theta), e)).astype(np.float32)


def rope_2d(h, w, head_dim=DIT_HEAD_DIM):
    """2D RoPE over centred token coordinates, theta 1e4.  The first head_dim/4 pairs rotate by the
    column coordinate, the next head_dim/4 by the row coordinate, both with the frequencies of a
    head_dim/2 axis (tools/reference.py:220-227; app/models/common.js:28-43).
    Returns (cos, sin), each [h*w, head_dim/2] fp32, token l = y*w + x."""
    axis = head_dim // 2
    f = inv_freq(axis, 10000.0)
    y = np.arange(h, dtype=np.float32) - np.float32((h - 1) / 2)
    x = np.arange(w, dtype=np.float32) - np.float32((w - 1) / 2)
    yy, xx = np.meshgrid(y, x, indexing="ij")
    a = np.concatenate([np.outer(xx.reshape(-1), f), np.outer(yy.reshape(-1), f)], axis=-1).astype(np.float32)
    return np.cos(a).astype(np.float32), np.sin(a).astype(np.float32)


def rope_1d(L, theta, head_dim=GEMMA_HEAD_DIM):
    """Standard 1D RoPE table, angle(l, i) = l / theta^(2i/D) (tools/reference.py:169-172;
    app/models/common.js:18-24).  Returns (cos, sin), each [L, head_dim/2] fp32."""
    f = inv_freq(head_dim, theta)
    a = (np.arange(L, dtype=np.float32)[:, None] * f[None]).astype(np.float32)
    return np.cos(a).astype(np.float32), np.sin(a).astype(np.float32)


def gemma_rope_theta(layer):
    """Layer i is global (theta 1e6) iff (i + 1) % 6 == 0, else local (theta 1e4)
    (tools/reference.py:186; app/models/gemma3.js:24)."""
    return 1e6 if (layer + 1) % 6 == 0 else 1e4


def head_norm(x, w, H, D, cos=None, sin=None, eps=1e-6, acc=np.float32):
    """Per-head RMSNorm (+ split-half RoPE when cos/sin are given) of rows [L, H*D]
    (tools/reference.py:240-241, 275-277; app/gpu/kernels.js:311-342 / ops.js:133-138)."""
    x = np.asarray(x, dtype=acc)
    L = x.shape[0]
    t = rms_norm(x.reshape(L, H, D), w, eps, acc)
    if cos is not None:
        t = rope_split_half(t.transpose(1, 0, 2), cos, sin, acc).transpose(1, 0, 2)
    return t.reshape(L, H * D)


# ----------------------------------------------------------------------------- attention core

def _softmax_rows(s, acc):
    m = np.max(s, axis=-1, keepdims=True)
    m = np.where(np.isfinite(m), m, acc(0))
    e = np.exp(s - m)
    return e / np.sum(e, axis=-1, keepdims=True)


def attention(q, k, v, H, D, bias=None, group=1, causal=False, window=0, scale=None, acc=np.float32):
    """Multi-head attention on packed rows, the semantics of F.scaled_dot_product_attention with an
    additive float mask as the reference uses it (tools/reference.py:230-237 DiT, :182-194 Gemma):
    q [Lq, H*D]; k, v [Lk, (H/group)*D]; query head h reads kv head h // group
    (``repeat_interleave``, tools/reference.py:193; ``bDiv``, app/gpu/ops.js:226,235).
    ``bias`` [Lk] is added to every row's scores (-inf drops a key).  ``causal`` keeps keys j <= i
    (tools/reference.py:182; app/gpu/kernels.js:44); ``window`` > 0 further keeps only i - window < j.
    Returns [Lq, H*D]."""
    q = np.asarray(q, dtype=acc)
    k = np.asarray(k, dtype=acc)
    v = np.asarray(v, dtype=acc)
    Lq, Lk = q.shape[0], k.shape[0]
    scale = acc(1.0 / math.sqrt(D)) if scale is None else acc(scale)
    qh = q.reshape(Lq, H, D).transpose(1, 0, 2)
    kh = k.reshape(Lk, H // group, D).transpose(1, 0, 2)
    vh = v.reshape(Lk, H // group, D).transpose(1, 0, 2)
    add = np.zeros((Lq, Lk), dtype=acc)
    if bias is not None:
        add = add + np.asarray(bias, dtype=acc)[None, :]
    if causal or window:
        i = np.arange(Lq)[:, None]
        j = np.arange(Lk)[None, :]
        keep = np.ones((Lq, Lk), dtype=bool)
        if causal:
            keep &= j <= i
        if window:
            keep &= j > i - window
        add = np.where(keep, add, acc(-np.inf))
    out = np.empty((H, Lq, D), dtype=acc)
    for h in range(H):
        s = (qh[h] @ kh[h // group].T) * scale + add
        out[h] = _softmax_rows(s, acc) @ vh[h // group]
    return out.transpose(1, 0, 2).reshape(Lq, H * D)


# ----------------------------------------------------------------------------- call-site assemblies

def text_key_bias(weights):
    """Per-text-key additive bias from prompt weights: log(max(w, 1e-4)), -inf where w <= 0
    (tools/reference.py:297; app/models/nanosaur2.js:97-118 drops the w <= 0 tokens instead)."""
    w = np.asarray(weights, dtype=np.float32)
    b = np.log(np.maximum(w, np.float32(1e-4))).astype(np.float32)
    return np.where(w <= 0, np.float32(-np.inf), b).astype(np.float32)


def refine_keep_bias(weights):
    """Key mask of the text-refine attention: 0 for kept tokens, -inf for w <= 0, keeping token 0
    when nothing survives (tools/reference.py:298-301)."""
    keep = np.asarray(weights) > 0
    if not keep.any():
        keep = keep.copy()
        keep[0] = True
    return np.where(keep, np.float32(0), np.float32(-np.inf)).astype(np.float32)


def dit_joint_attention(q_raw, k_raw, v, q_w, k_w, cos, sin, ky_raw=None, vy=None, txt_bias=None,
                        eps=1e-6, acc=np.float32):
    """One DiT block's attention step (tools/reference.py:272-286; app/models/nanosaur2.js:196-208):
    image q/k get per-head RMSNorm + 2D RoPE, text keys (``ky_raw``) get the k norm only, text values
    are appended as is, and the text keys carry ``txt_bias`` (image keys bias 0).
    q_raw, k_raw, v: [L, 1536]; ky_raw, vy: [Lt, 1536]; returns [L, 1536]."""
    H, D = DIT_HEADS, DIT_HEAD_DIM
    q = head_norm(q_raw, q_w, H, D, cos, sin, eps, acc)
    k = head_norm(k_raw, k_w, H, D, cos, sin, eps, acc)
    vv = np.asarray(v, dtype=acc)
    bias = None
    if ky_raw is not None:
        k = np.concatenate([k, head_norm(ky_raw, k_w, H, D, None, None, eps, acc)])
        vv = np.concatenate([vv, np.asarray(vy, dtype=acc)])
        bias = np.concatenate([np.zeros(q.shape[0], dtype=acc), np.asarray(txt_bias, dtype=acc)])
    return attention(q, k, vv, H, D, bias=bias, acc=acc)


def text_refine_attention(q_raw, k_raw, v, q_w, k_w, keep_bias, eps=1e-6, acc=np.float32):
    """Text-refine attention (tools/reference.py:258-259; app/models/nanosaur2.js:128-132):
    per-head q/k RMSNorm without RoPE, all-text queries and keys, ``keep_bias`` on the keys."""
    H, D = DIT_HEADS, DIT_HEAD_DIM
    q = head_norm(q_raw, q_w, H, D, None, None, eps, acc)
    k = head_norm(k_raw, k_w, H, D, None, None, eps, acc)
    return attention(q, k, v, H, D, bias=keep_bias, acc=acc)


def gemma_attention(q_raw, k_raw, v, q_w, k_w, theta, window=0, eps=1e-6, acc=np.float32):
    """Gemma3-270M layer attention (tools/reference.py:186-194; app/models/gemma3.js:58-70):
    q [L, 4*256], k/v [L, 256]; q/k RMSNorm with the stored (w - 1) weights already lifted by +1,
    1D RoPE with ``theta``, causal GQA 4/1 with scale 1/16.  ``window`` > 0 adds the sliding window
    (parity-unpinned: the reference never reaches it).  Returns [L, 1024]."""
    H, KH, D = GEMMA_HEADS, GEMMA_KV_HEADS, GEMMA_HEAD_DIM
    L = q_raw.shape[0]
    cos, sin = rope_1d(L, theta, D)
    q = head_norm(q_raw, q_w, H, D, cos, sin, eps, acc)
    k = head_norm(k_raw, k_w, KH, D, cos, sin, eps, acc)
    return attention(q, k, v, H, D, group=H // KH, causal=True, window=window, acc=acc)


def group_norm(x, groups, w, b, eps=1e-6, acc=np.float32):
    """GroupNorm over x [C, ...]: mean and biased variance per group of C/groups channels, then
    (x - mean) / sqrt(var + eps) * w[c] + b[c] (F.group_norm as tools/reference.py:339 calls it;
    app/models/vae.js:78 ops.groupNorm without SiLU)."""
    x = np.asarray(x, acc)
    C = x.shape[0]
    g = x.reshape(groups, -1)
    mean = g.mean(axis=1, keepdims=True)
    var = ((g - mean) ** 2).mean(axis=1, keepdims=True)
    n = ((g - mean) / np.sqrt(var + acc(eps))).reshape(x.shape)
    shape = (C,) + (1,) * (x.ndim - 1)
    return n * np.asarray(w, acc).reshape(shape) + np.asarray(b, acc).reshape(shape)


def vae_attention(x, gn_w, gn_b, w_q, b_q, w_k, b_k, w_v, b_v, w_o, b_o, groups=32, eps=1e-6, acc=np.float32):
    """The VAE decoder's single-head attention block over all pixels (tools/reference.py:352-357;
    app/models/vae.js:77-88): x [C, h, w]; n = group_norm(x); q/k/v = 1x1 convolutions of n (linears
    over the channels, weights [C, C]); softmax(q k^T / sqrt(C)) v over the h*w pixels with head dim
    C; then x + proj_out(a).  Returns [C, h, w]."""
    x = np.asarray(x, acc)
    C = x.shape[0]
    n = group_norm(x, groups, gn_w, gn_b, eps, acc).reshape(C, -1).T          # [hw, C]
    q, k, v = (linear(n, w, bb, acc) for w, bb in ((w_q, b_q), (w_k, b_k), (w_v, b_v)))
    a = attention(q, k, v, 1, C, acc=acc)                                    # [hw, C]
    return x + linear(a, w_o, b_o, acc).T.reshape(x.shape)


def glu(x, act="gelu_tanh", acc=np.float32):
    """ops.glu (app/gpu/ops.js:141-148, kernels.js:346-360): x [rows, 2I] = [gate | up] ->
    act(gate) * up.  gelu_tanh is PyTorch's approximate="tanh" GELU (tools/reference.py:198),
    0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))); silu is x / (1 + exp(-x))."""
    x = np.asarray(x, acc)
    I = x.shape[-1] // 2
    g, u = x[..., :I], x[..., I:]
    if act == "silu":
        a = g / (acc(1) + np.exp(-g))
    else:
        a = acc(0.5) * g * (acc(1) + np.tanh(acc(math.sqrt(2.0 / math.pi)) * (g + acc(0.044715) * g * g * g)))
    return a * u


def gemma_mlp_sublayer(x, pre_w, w_gate, w_up, w_down, post_w, eps=1e-6, acc=np.float32):
    """The MLP half of one Gemma3 layer on the residual stream x [L, hidden]
    (tools/reference.py:197-199; app/models/gemma3.js:78-89): h = rms_norm(x, pre_w),
    g = gelu_tanh(h W_gate^T) * (h W_up^T), then x + rms_norm(g W_down^T, post_w)."""
    x = np.asarray(x, acc)
    h = rms_norm(x, pre_w, eps, acc)
    g = glu(np.concatenate([linear(h, w_gate, acc=acc), linear(h, w_up, acc=acc)], axis=-1), "gelu_tanh", acc)
    return x + rms_norm(linear(g, w_down, acc=acc), post_w, eps, acc)


def gemma_attention_sublayer(x, in_w, w_q, w_k, w_v, q_w, k_w, w_o, post_w, theta, window=0, eps=1e-6,
                             acc=np.float32):
    """The attention half of one Gemma3 layer on the residual stream x [L, hidden]
    (tools/reference.py:187-196; app/models/gemma3.js:62-77): h = rms_norm(x, in_w), q/k/v = h W^T,
    a = gemma_attention(q, k, v), then x + rms_norm(a W_o^T, post_w).  Norm weights are the lifted
    (w - 1) + 1 values.  Returns the updated residual stream."""
    x = np.asarray(x, acc)
    h = rms_norm(x, in_w, eps, acc)
    a = gemma_attention(linear(h, w_q, acc=acc), linear(h, w_k, acc=acc), linear(h, w_v, acc=acc), q_w, k_w,
                        theta, window, eps, acc)
    return x + rms_norm(linear(a, w_o, acc=acc), post_w, eps, acc)


# ----------------------------------------------------------------------------- batched helpers

def joint_attention_batched(qkv, L, Lt, kv_len, q_w, k_w, cos, sin, bias=None, H=DIT_HEADS,
                            D=DIT_HEAD_DIM, eps=1e-6, acc=np.float32, heads=None, rows=None):
    """Batched form of ``dit_joint_attention`` on the packed buffer the CUDA path takes:
    qkv [B, L + Lt, 3*H*D] with rows [0, L) image q|k|v and rows [L, L+Lt) text k|v (q unused);
    kv_len[b] = L + valid text rows; bias [B, Lt] on the text keys.  ``heads`` restricts the
    computation to a subset of heads (the output keeps zeros elsewhere).  ``rows`` (an index array
    into [0, L)) restricts it to those query rows, every key still taking part: the result is then
    [B, len(rows), H*D], row i being query rows[i].  Returns [B, L, H*D] otherwise."""
    qkv = np.asarray(qkv)
    B = qkv.shape[0]
    C = H * D
    qi = np.arange(L) if rows is None else np.asarray(rows, np.int64)
    out = np.zeros((B, qi.size, C), dtype=acc)
    hs = list(range(H)) if heads is None else list(heads)
    for b in range(B):
        n = int(kv_len[b])
        x = qkv[b]
        q = x[qi, 0:C].astype(acc)
        k_img = x[:L, C:2 * C].astype(acc)
        v_all = x[:n, 2 * C:3 * C].astype(acc)
        k_txt = x[L:n, C:2 * C].astype(acc)
        qn = head_norm(q, q_w, H, D, cos[qi], sin[qi], eps, acc)
        kn = head_norm(k_img, k_w, H, D, cos, sin, eps, acc)
        if n > L:
            kn = np.concatenate([kn, head_norm(k_txt, k_w, H, D, None, None, eps, acc)])
        kb = None
        if bias is not None and n > L:
            kb = np.concatenate([np.zeros(L, dtype=acc), np.asarray(bias[b][: n - L], dtype=acc)])
        for h in hs:
            sl = slice(h * D, (h + 1) * D)
            out[b, :, sl] = attention(qn[:, sl], kn[:, sl], v_all[:, sl], 1, D, bias=kb, acc=acc)
    return out
