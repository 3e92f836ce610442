"""Generate the golden fixtures that pin the CPU oracle (``oracle/attention_oracle.py``).

Run in a container where the reference repository is mounted (it is NOT needed at test time):

    python tests/golden/make_golden.py --reference /path/to/nanosaur2-web

It imports the reference's own fp32 PyTorch implementation (``tools/reference.py``) unchanged and
drives its real code paths with small seeded stand-in weights (no model files exist here):

* ``DiT.forward`` end to end on a tiny latent: every attention call of the two text-refine blocks
  (``tools/reference.py:252-259``) and of the 18 image blocks (``:267-286``) is captured with the raw
  q/k (the inputs of the per-head RMSNorm), the v rows, the norm weights, the 2D RoPE tables, the
  key bias the forward pass derived from the prompt weights (``:296-301``), the post-prologue q/k and
  the attention output.
* ``gemma_encode`` (``:175-200``): the raw q/k of each layer's q/k norm, the SDPA inputs/outputs and
  the causal mask.
* ``rope_2d`` / ``gemma_rope`` tables and ``rms_norm`` / ``rope_split_half`` on seeded inputs.
* ``lin`` (``:208-210``), the q|k|v projection's linear, on small seeded operands with and without a
  bias (``--only linear`` writes just this fixture).
* ``gemma_encode``'s layers 0 and 5 (``:187-199``: input norm, q/k/v linears, head norms, RoPE,
  causal SDPA, o linear, post-attention norm, residual add; then the GELU-tanh MLP with its norms) on
  a 64-wide residual stream with bf16-exact linear weights (``--only gemma_sublayer``).
* an int8 ConvRot linear with two LoRAs (``--only convrot``): a seeded weight quantised by the
  reference's ``quant.quantize_int8_convrot`` (``tools/quant.py:48-57``), written with a bias to a
  temporary safetensors file beside two LoRA files (PEFT names with an alpha, kohya names without),
  loaded through the reference's ``Weights`` (``tools/reference.py:48-67``: dequantise on access, LoRA
  deltas merged, ``lora_deltas`` at ``:70-94``) and applied with its ``lin``; plus ``quant.hadamard``
  and ``quant.rotate`` on seeded inputs (H16 and a rotation by H256).
* ``VAE.attn`` (``:352-357``), the VAE decoder's single-head attention block (group norm, q/k/v 1x1
  convolutions, SDPA with head dim C, proj_out, residual) on a 64 x 6 x 5 activation
  (``--only vae_attention``).

The qkv projection outputs of the DiT are rounded to bf16 inside the reference run (a hook on its
``lin``), so the bf16 CUDA path sees exactly the inputs the fp32 reference saw.  The Gemma inputs
stay fp32.  Fixtures are written as compressed ``.npz`` next to this script.
"""

from __future__ import annotations

import argparse
import os
import re
import sys
import zlib

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def bf16_round(t):
    return t.to(torch.bfloat16).to(torch.float32)


class StandInWeights:
    """Seeded random weights with the shapes the reference reads.  Blocks/layers share one tensor
    per role to keep memory small; ``kv_y`` exists on even DiT blocks only, as in the real model."""

    def __init__(self, shapes, seed, has_fn):
        self.shapes = shapes
        self.seed = seed
        self.has_fn = has_fn
        self.cache = {}

    def _role(self, name):
        return re.sub(r"^(blocks|text_refine_blocks|model\.layers)\.\d+\.", r"\1.#.", name)

    def __call__(self, name):
        role = self._role(name)
        if role not in self.cache:
            shape, kind = self.shapes(role)
            g = torch.Generator().manual_seed(self.seed + (zlib.crc32(role.encode()) & 0xFFFF))
            if kind == "norm":
                t = 1.0 + 0.25 * torch.randn(shape, generator=g)
            elif kind == "gemma_norm":   # stored as (w - 1); the reference adds 1 on read
                t = 0.25 * torch.randn(shape, generator=g)
            elif kind == "small":
                t = 0.05 * torch.randn(shape, generator=g)
            else:
                t = torch.randn(shape, generator=g) / (shape[-1] ** 0.5)
            self.cache[role] = t.float()
        return self.cache[role]

    def has(self, name):
        return self.has_fn(name)


def dit_shapes(role):
    C, I = 1536, 32
    table = {
        "t_embedder.mlp.0.weight": ((C, 256), "lin"), "t_embedder.mlp.2.weight": ((C, C), "lin"),
        "y_embedder.proj.weight": ((C, 640), "lin"), "y_embedder.norm.weight": ((C,), "norm"),
        "y_pool_proj.weight": ((C, C), "lin"), "shared_encoder_adaLN.0.weight": ((6 * C, C), "small"),
        "encoder_adaLN_offsets.#": ((6 * C,), "small"), "s_embedder.proj.weight": ((C, 64), "lin"),
        "sprint_out_proj.weight": ((C, C), "lin"), "final_layer.adaLN_modulation.weight": ((2 * C, C), "small"),
        "final_layer.linear.weight": ((64, C), "lin"),
    }
    if role in table:
        return table[role]
    if role.startswith("encoder_adaLN_offsets."):
        return ((6 * C,), "small")
    suffix = role.split(".#.", 1)[1]
    per_block = {
        "adaLN_modulation.0.weight": ((6 * C, C), "small"), "norm1.weight": ((C,), "norm"),
        "norm2.weight": ((C,), "norm"), "attn.qkv.weight": ((3 * C, C), "lin"),
        "attn.qkv_x.weight": ((3 * C, C), "lin"), "attn.kv_y.weight": ((2 * C, C), "lin"),
        "attn.q_norm.weight": ((96,), "norm"), "attn.k_norm.weight": ((96,), "norm"),
        "attn.proj.weight": ((C, C), "lin"), "mlp.w12.weight": ((2 * I, C), "lin"),
        "mlp.w3.weight": ((C, I), "lin"),
    }
    return per_block[suffix]


def dit_has(name):
    if name.endswith(".bias") or name.endswith("comfy_quant"):
        return False
    if ".attn.kv_y." in name:
        return int(name.split(".")[1]) % 2 == 0
    return True


def gemma_shapes(role, Hd=640):
    I, V = 64, 300
    if role == "model.embed_tokens.weight":
        return ((V, Hd), "emb")
    if role == "model.norm.weight":
        return ((Hd,), "gemma_norm")
    suffix = role.split(".#.", 1)[1]
    per_layer = {
        "input_layernorm.weight": ((Hd,), "gemma_norm"), "post_attention_layernorm.weight": ((Hd,), "gemma_norm"),
        "pre_feedforward_layernorm.weight": ((Hd,), "gemma_norm"), "post_feedforward_layernorm.weight": ((Hd,), "gemma_norm"),
        "self_attn.q_norm.weight": ((256,), "gemma_norm"), "self_attn.k_norm.weight": ((256,), "gemma_norm"),
        "self_attn.q_proj.weight": ((1024, Hd), "lin"), "self_attn.k_proj.weight": ((256, Hd), "lin"),
        "self_attn.v_proj.weight": ((256, Hd), "lin"), "self_attn.o_proj.weight": ((Hd, 1024), "lin"),
        "mlp.gate_proj.weight": ((I, Hd), "lin"), "mlp.up_proj.weight": ((I, Hd), "lin"),
        "mlp.down_proj.weight": ((Hd, I), "lin"),
    }
    return per_layer[suffix]


def capture_dit(R, seed, h, w, txt_weights):
    """Run DiT.forward with stand-in weights; return one record per attention call."""
    W = StandInWeights(dit_shapes, seed, dit_has)
    dit = R.DiT(W)
    records, norms = [], []
    orig_attention, orig_rms, orig_lin = R.attention, R.rms_norm, R.lin

    def lin_hook(Wt, name, x):
        y = orig_lin(Wt, name, x)
        if name.endswith("attn.qkv_x") or name.endswith("attn.kv_y") or name.endswith("attn.qkv"):
            y = bf16_round(y)
        return y

    def rms_hook(x, wt, eps=1e-6):
        if x.dim() == 3 and x.shape[-1] == 96:
            norms.append((x.detach().clone(), wt.detach().clone()))
        return orig_rms(x, wt, eps)

    def attn_hook(q, k, v, bias=None):
        out = orig_attention(q, k, v, bias)
        records.append({"q_post": q.clone(), "k_post": k.clone(), "v": v.clone(),
                        "bias": None if bias is None else bias.clone(), "out": out.clone(),
                        "norms": list(norms)})
        norms.clear()
        return out

    R.attention, R.rms_norm, R.lin = attn_hook, rms_hook, lin_hook
    try:
        g = torch.Generator().manual_seed(seed)
        latent = torch.randn((64, h, w), generator=g)
        context = torch.randn((len(txt_weights), 640), generator=g)
        wts = torch.tensor(txt_weights, dtype=torch.float32)
        dit.forward(latent, 0.7, context, wts)
    finally:
        R.attention, R.rms_norm, R.lin = orig_attention, orig_rms, orig_lin
    cos, sin = R.rope_2d(h, w)
    return records, cos, sin, wts


def capture_gemma(R, seed, L):
    W = StandInWeights(gemma_shapes, seed, lambda n: True)
    F = R.F
    records, norms = [], []
    orig_sdpa, orig_rms = F.scaled_dot_product_attention, R.rms_norm

    def rms_hook(x, wt, eps=1e-6):
        if x.dim() == 3 and x.shape[-1] == 256:
            norms.append((x.detach().clone(), wt.detach().clone()))
        return orig_rms(x, wt, eps)

    def sdpa_hook(q, k, v, attn_mask=None, **kw):
        out = orig_sdpa(q, k, v, attn_mask=attn_mask, **kw)
        records.append({"q_post": q[0].clone(), "k_post": k[0].clone(), "v": v[0].clone(),
                        "mask": attn_mask.clone(), "out": out[0].clone(), "norms": list(norms)})
        norms.clear()
        return out

    F.scaled_dot_product_attention, R.rms_norm = sdpa_hook, rms_hook
    try:
        ids = [2] + [int(i) for i in torch.randint(3, 300, (L - 1,), generator=torch.Generator().manual_seed(seed))]
        R.gemma_encode(W, ids)
    finally:
        F.scaled_dot_product_attention, R.rms_norm = orig_sdpa, orig_rms
    return records


class Bf16LinearWeights(StandInWeights):
    """Stand-in weights whose matrices are bf16-exact, so a bf16 GEMM sees the reference's values."""

    def __call__(self, name):
        t = super().__call__(name)
        return bf16_round(t) if t.dim() == 2 and not name.endswith("embed_tokens.weight") else t


def write_gemma_sublayer(R, out, L=40, hidden=64):
    """gemma_encode's layers 0 (local) and 5 (global) (tools/reference.py:187-199) on a 64-wide residual
    stream (the attention shapes are the model's: 4 + 1 heads of 256; MLP width 64): the layer input
    x, x after the attention half ``x + rms_norm(a @ W_o^T, post)``, the layer output after the MLP
    half, and the weights, with the linear weights bf16-exact.  The reference's 2-D rms_norm calls
    give, per layer, the input norm (its x is the layer input), the post-attention norm, the pre-MLP
    norm (its x is the stream after attention), the post-MLP norm, and then the next layer's input
    norm (its x is the layer output)."""
    W = Bf16LinearWeights(lambda role: gemma_shapes(role, hidden), 4321, lambda n: True)
    calls = []
    orig_rms = R.rms_norm

    def rms_hook(x, wt, eps=1e-6):
        if x.dim() == 2:
            calls.append((x.detach().clone(), wt.detach().clone()))
        return orig_rms(x, wt, eps)

    R.rms_norm = rms_hook
    try:
        ids = [2] + [int(i) for i in torch.randint(3, 300, (L - 1,), generator=torch.Generator().manual_seed(4321))]
        R.gemma_encode(W, ids)
    finally:
        R.rms_norm = orig_rms
    assert len(calls) == 4 * 17 + 1, len(calls)
    p = "model.layers.0."
    rec = {}
    for layer in (0, 5):
        (x_in, w_in), (_, w_post), (x_mid, pre_ff_w), (_, post_ff_w) = calls[4 * layer:4 * layer + 4]
        x_out = calls[4 * layer + 4][0]   # the next layer's input norm sees the layer's output
        rec[f"x_in{layer}"], rec[f"x_mid{layer}"], rec[f"x_out{layer}"] = np32(x_in), np32(x_mid), np32(x_out)
    np.savez_compressed(
        os.path.join(out, "gemma_sublayer.npz"), **rec, layers=np.array([0, 5]),
        in_w=np32(w_in), post_w=np32(w_post), pre_ff_w=np32(pre_ff_w), post_ff_w=np32(post_ff_w),
        w_gate=np32(W(p + "mlp.gate_proj.weight")), w_up=np32(W(p + "mlp.up_proj.weight")),
        w_down=np32(W(p + "mlp.down_proj.weight")),
        q_w=np32(W(p + "self_attn.q_norm.weight") + 1.0), k_w=np32(W(p + "self_attn.k_norm.weight") + 1.0),
        w_q=np32(W(p + "self_attn.q_proj.weight")), w_k=np32(W(p + "self_attn.k_proj.weight")),
        w_v=np32(W(p + "self_attn.v_proj.weight")), w_o=np32(W(p + "self_attn.o_proj.weight")))


def write_vae_attention(R, out, C=64, h=6, w=5):
    """VAE.attn (tools/reference.py:352-357) on a [1, C, h, w] activation with seeded stand-in weights:
    group norm (32 groups), q/k/v 1x1 convolutions, single-head SDPA over the h*w pixels with head dim
    C, proj_out and the residual."""

    class Params:
        def __init__(self, d):
            self.d = d

        def __call__(self, name):
            return self.d[name]

        def has(self, name):
            return name in self.d

    gen = torch.Generator().manual_seed(55)
    p = "decoder.mid.attn_1"
    d = {p + ".norm.weight": 1.0 + 0.25 * torch.randn(C, generator=gen), p + ".norm.bias": 0.1 * torch.randn(C, generator=gen)}
    for part in (".q", ".k", ".v", ".proj_out"):
        d[p + part + ".weight"] = torch.randn(C, C, 1, 1, generator=gen) / C ** 0.5
        d[p + part + ".bias"] = 0.1 * torch.randn(C, generator=gen)
    x = 2.0 * torch.randn(1, C, h, w, generator=gen)
    y = R.VAE(Params(d)).attn(x, p)
    np.savez_compressed(
        os.path.join(out, "vae_attention.npz"), x=np32(x[0]), y=np32(y[0]),
        gn_w=np32(d[p + ".norm.weight"]), gn_b=np32(d[p + ".norm.bias"]),
        **{f"w_{k}": np32(d[f"{p}.{n}.weight"].reshape(C, C)) for k, n in (("q", "q"), ("k", "k"), ("v", "v"), ("o", "proj_out"))},
        **{f"b_{k}": np32(d[f"{p}.{n}.bias"]) for k, n in (("q", "q"), ("k", "k"), ("v", "v"), ("o", "proj_out"))})


def np32(t):
    return t.detach().float().cpu().numpy().astype(np.float32)


def write_linear(R, out):
    """The reference's lin (y = x @ W^T + b) on a 7 x 64 input and a 96 x 64 weight."""

    class Params:
        def __init__(self, d):
            self.d = d

        def __call__(self, name):
            return self.d[name]

        def has(self, name):
            return name in self.d

    gen = torch.Generator().manual_seed(77)
    x = torch.randn(7, 64, generator=gen)
    w = torch.randn(96, 64, generator=gen) / 8
    b = torch.randn(96, generator=gen)
    y = R.lin(Params({"attn.qkv_x.weight": w, "attn.qkv_x.bias": b}), "attn.qkv_x", x)
    y_nobias = R.lin(Params({"attn.kv_y.weight": w}), "attn.kv_y", x)
    np.savez_compressed(os.path.join(out, "linear.npz"), x=np32(x), w=np32(w), b=np32(b), y=np32(y),
                        y_nobias=np32(y_nobias))


def write_convrot(R, out, N=32, K=512, M=9):
    """int8 ConvRot weights and LoRAs through the reference's own loader and lin."""
    import tempfile

    import quant  # the reference's tools/quant.py (on sys.path beside reference.py)
    from safetensors.torch import save_file

    gen = torch.Generator().manual_seed(505)
    w = torch.randn(N, K, generator=gen) / 16
    b = torch.randn(N, generator=gen)
    x = torch.randn(M, K, generator=gen)
    a1 = torch.randn(8, K, generator=gen) / 16
    b1 = torch.randn(N, 8, generator=gen) / 8
    a2 = torch.randn(4, K, generator=gen) / 16
    b2 = torch.randn(N, 4, generator=gen) / 8
    alpha1, s1, s2 = 4.0, 0.8, -0.5
    qt = quant.quantize_int8_convrot(w)
    with tempfile.TemporaryDirectory() as d:
        base, l1, l2 = (os.path.join(d, f) for f in ("base.safetensors", "l1.safetensors", "l2.safetensors"))
        save_file({"blk.lin.weight": qt["weight"], "blk.lin.weight_scale": qt["weight_scale"],
                   "blk.lin.comfy_quant": qt["comfy_quant"], "blk.lin.bias": b}, base)
        save_file({"diffusion_model.blk.lin.lora_A.weight": a1, "diffusion_model.blk.lin.lora_B.weight": b1,
                   "diffusion_model.blk.lin.alpha": torch.tensor(alpha1)}, l1)
        save_file({"lora_unet_blk_lin.lora_down.weight": a2, "lora_unet_blk_lin.lora_up.weight": b2}, l2)
        y_base = R.lin(R.Weights(base), "blk.lin", x)
        y_lora = R.lin(R.Weights(base, loras=[(l1, s1), (l2, s2)]), "blk.lin", x)
    hx = torch.randn(3, 512, generator=gen)
    np.savez_compressed(
        os.path.join(out, "convrot.npz"), x=np32(x), w=np32(w), b=np32(b), q=qt["weight"].numpy(),
        scale=np32(qt["weight_scale"].reshape(-1)), a1=np32(a1), b1=np32(b1), a2=np32(a2), b2=np32(b2),
        alpha1=alpha1, s1=s1, s2=s2, y_base=np32(y_base), y_lora=np32(y_lora), h16=np32(quant.hadamard(16, "cpu")),
        hx=np32(hx), hx_rot=np32(quant.rotate(hx)))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("NANOSAUR2_REFERENCE"),
                    help="checkout of the reference repository (or NANOSAUR2_REFERENCE)")
    ap.add_argument("--out", default=HERE)
    ap.add_argument("--only", choices=["linear", "gemma_sublayer", "vae_attention", "convrot"],
                    help="write one fixture only")
    args = ap.parse_args()
    if not args.reference:
        ap.error("pass --reference <checkout of the reference> or set NANOSAUR2_REFERENCE")
    sys.path.insert(0, os.path.join(args.reference, "tools"))
    import reference as R  # noqa: E402  (the unmodified reference module)
    torch.set_num_threads(min(8, os.cpu_count() or 1))
    if args.only in (None, "linear"):
        write_linear(R, args.out)
    if args.only in (None, "gemma_sublayer"):
        write_gemma_sublayer(R, args.out)
    if args.only in (None, "vae_attention"):
        write_vae_attention(R, args.out)
    if args.only in (None, "convrot"):
        write_convrot(R, args.out)
    if args.only:
        return

    # ---- DiT: 4x5 latent (20 image tokens), 10 text slots with emphasis weights and dropped tokens
    h, w = 4, 5
    txt_w = [1.0, 1.3, 0.7, 1.0, 1.0, 0.7, 1.3, 1.0, 0.0, 0.0]
    recs, cos, sin, wts = capture_dit(R, 1234, h, w, txt_w)
    L = h * w
    refine = [r for r in recs if r["q_post"].shape[0] == len(txt_w)]
    blocks = [r for r in recs if r["q_post"].shape[0] == L]
    assert len(refine) == 2 and len(blocks) == 18, (len(refine), len(blocks))
    even, odd = blocks[0], blocks[1]
    assert even["bias"] is not None and odd["bias"] is None
    (q_raw, q_w), (k_raw, k_w), (ky_raw, k_w2) = even["norms"]
    assert torch.equal(k_w, k_w2)
    np.savez_compressed(
        os.path.join(args.out, "dit_joint_block.npz"),
        h=h, w=w, q_raw=np32(q_raw.reshape(L, -1)), k_raw=np32(k_raw.reshape(L, -1)),
        ky_raw=np32(ky_raw.reshape(len(txt_w), -1)), v=np32(even["v"][:L]), vy=np32(even["v"][L:]),
        q_w=np32(q_w), k_w=np32(k_w), cos=np32(cos), sin=np32(sin), txt_weights=np32(wts),
        txt_bias=np32(even["bias"][L:]), q_post=np32(even["q_post"]), k_post=np32(even["k_post"]),
        out=np32(even["out"]))
    (q_raw, q_w), (k_raw, k_w) = odd["norms"]
    np.savez_compressed(
        os.path.join(args.out, "dit_image_block.npz"),
        h=h, w=w, q_raw=np32(q_raw.reshape(L, -1)), k_raw=np32(k_raw.reshape(L, -1)), v=np32(odd["v"]),
        q_w=np32(q_w), k_w=np32(k_w), cos=np32(cos), sin=np32(sin), q_post=np32(odd["q_post"]),
        k_post=np32(odd["k_post"]), out=np32(odd["out"]))
    r0 = refine[0]
    (q_raw, q_w), (k_raw, k_w) = r0["norms"]
    Lt = len(txt_w)
    np.savez_compressed(
        os.path.join(args.out, "dit_text_refine.npz"),
        q_raw=np32(q_raw.reshape(Lt, -1)), k_raw=np32(k_raw.reshape(Lt, -1)), v=np32(r0["v"]),
        q_w=np32(q_w), k_w=np32(k_w), txt_weights=np32(wts), keep_bias=np32(r0["bias"]),
        q_post=np32(r0["q_post"]), k_post=np32(r0["k_post"]), out=np32(r0["out"]))

    # ---- Gemma: 40 tokens, layer 0 (local, theta 1e4) and layer 5 (global, theta 1e6)
    grecs = capture_gemma(R, 4321, 40)
    assert len(grecs) == 17
    for layer in (0, 5):
        g = grecs[layer]
        (q_raw, q_w), (k_raw, k_w) = g["norms"]
        Lg = q_raw.shape[1]
        np.savez_compressed(
            os.path.join(args.out, f"gemma_layer{layer}.npz"),
            layer=layer, theta=(1e6 if (layer + 1) % 6 == 0 else 1e4),
            q_raw=np32(q_raw.transpose(0, 1).reshape(Lg, -1)), k_raw=np32(k_raw.transpose(0, 1).reshape(Lg, -1)),
            v=np32(g["v"][0]), q_w=np32(q_w), k_w=np32(k_w), mask=np32(g["mask"]),
            q_post=np32(g["q_post"].transpose(0, 1).reshape(Lg, -1)),
            k_post=np32(g["k_post"][0]), out=np32(g["out"].transpose(0, 1).reshape(Lg, -1)))

    # ---- tables and elementwise pieces
    c2, s2 = R.rope_2d(7, 5)
    c1l, s1l = R.gemma_rope(40, 1e4)
    c1g, s1g = R.gemma_rope(40, 1e6)
    gen = torch.Generator().manual_seed(99)
    x = torch.randn(6, 3, 96, generator=gen) * 3.0
    wn = torch.randn(96, generator=gen)
    cs_c, cs_s = R.rope_2d(2, 3)
    rn = R.rms_norm(x, wn)
    rs = R.rope_split_half(rn.transpose(0, 1), cs_c, cs_s).transpose(0, 1)
    np.savez_compressed(
        os.path.join(args.out, "tables.npz"),
        rope2d_h=7, rope2d_w=5, rope2d_cos=np32(c2), rope2d_sin=np32(s2),
        rope1d_L=40, rope1d_local_cos=np32(c1l), rope1d_local_sin=np32(s1l),
        rope1d_global_cos=np32(c1g), rope1d_global_sin=np32(s1g),
        rms_x=np32(x), rms_w=np32(wn), rms_out=np32(rn), rope_cos=np32(cs_c), rope_sin=np32(cs_s),
        rope_out=np32(rs))
    print("wrote fixtures to", args.out)


if __name__ == "__main__":
    main()
