"""The CPU oracle against golden vectors captured from the reference's own fp32 code paths
(``tests/golden/make_golden.py`` drives ``tools/reference.py``'s ``DiT.forward`` and
``gemma_encode``).  These pin the restatement before any CUDA result is compared with it."""

import numpy as np
import pytest

from oracle import attention_oracle as O

TOL = dict(rtol=2e-5, atol=2e-5)


def test_rope_tables(golden):
    t = golden("tables")
    c, s = O.rope_2d(int(t["rope2d_h"]), int(t["rope2d_w"]))
    np.testing.assert_allclose(c, t["rope2d_cos"], **TOL)
    np.testing.assert_allclose(s, t["rope2d_sin"], **TOL)
    L = int(t["rope1d_L"])
    for name, theta in (("local", 1e4), ("global", 1e6)):
        c, s = O.rope_1d(L, theta)
        np.testing.assert_allclose(c, t[f"rope1d_{name}_cos"], rtol=1e-5, atol=5e-5)
        np.testing.assert_allclose(s, t[f"rope1d_{name}_sin"], rtol=1e-5, atol=5e-5)


def test_rms_norm_and_rope(golden):
    t = golden("tables")
    rn = O.rms_norm(t["rms_x"], t["rms_w"])
    np.testing.assert_allclose(rn, t["rms_out"], **TOL)
    rs = O.rope_split_half(rn.transpose(1, 0, 2), t["rope_cos"], t["rope_sin"]).transpose(1, 0, 2)
    np.testing.assert_allclose(rs, t["rope_out"], **TOL)


def test_linear(golden):
    t = golden("linear")
    np.testing.assert_allclose(O.linear(t["x"], t["w"], t["b"]), t["y"], **TOL)
    np.testing.assert_allclose(O.linear(t["x"], t["w"]), t["y_nobias"], **TOL)


def convrot_lora_entries(t, rotated=True):
    """The two LoRAs of the convrot fixture as app/lora.js:120-150 builds them: A rows rotated for the
    int8 layer, scale = strength * alpha / r (the kohya file has no alpha: scale = strength)."""
    r1 = t["a1"].shape[0]
    rot = (lambda a: O.rotate(a, acc=np.float64)) if rotated else (lambda a: a)
    return [dict(A=rot(t["a1"]), B=t["b1"], scale=float(t["s1"]) * float(t["alpha1"]) / r1),
            dict(A=rot(t["a2"]), B=t["b2"], scale=float(t["s2"]))]


def test_convrot_hadamard_and_rotation(golden):
    t = golden("convrot")
    np.testing.assert_array_equal(O.hadamard(16), t["h16"])
    np.testing.assert_allclose(O.rotate(t["hx"]), t["hx_rot"], rtol=1e-5, atol=2e-6)
    # H256 is symmetric and orthogonal: rotating twice is the identity (tools/quant.py:67)
    np.testing.assert_allclose(O.rotate(O.rotate(t["hx"], acc=np.float64), acc=np.float64), t["hx"], atol=1e-12)


def test_convrot_quantizer(golden):
    """tools/quant.py:48-57 restated: the same int8 weights except where fp32 summation order moves a
    value across a rounding tie, and there by one step."""
    t = golden("convrot")
    q, scale = O.quantize_int8_convrot(t["w"])
    np.testing.assert_allclose(scale, t["scale"], rtol=1e-6)
    diff = q.astype(np.int32) - t["q"].astype(np.int32)
    assert np.abs(diff).max() <= 1
    pre = O.rotate(t["w"], acc=np.float64) / t["scale"][:, None].astype(np.float64)
    ties = np.abs(np.abs(pre - np.floor(pre)) - 0.5) < 1e-4
    assert not (diff != 0)[~ties].any()


def test_convrot_int8_linear_with_loras(golden):
    """The JS side path (rotated input, int8 GEMM with row scales, bias, LoRA delta from rotated A rows:
    app/gpu/ops.js:50-86, gemm.js:159-160) equals the reference's merged, dequantised weight through
    its own loader and lin (tools/reference.py:48-94, 208-210)."""
    t = golden("convrot")
    xr = O.rotate(t["x"], acc=np.float64)
    y = O.linear_int8(xr, t["q"], t["scale"], t["b"], acc=np.float64)
    np.testing.assert_allclose(y, t["y_base"], rtol=1e-5, atol=2e-5)
    y = y + O.lora_delta(xr, convrot_lora_entries(t), t["q"].shape[0], acc=np.float64)
    np.testing.assert_allclose(y, t["y_lora"], rtol=1e-5, atol=2e-5)


def test_gemma_theta_schedule():
    assert [O.gemma_rope_theta(i) for i in range(12)] == [1e4] * 5 + [1e6] + [1e4] * 5 + [1e6]


def test_dit_joint_block(golden):
    g = golden("dit_joint_block")
    L = g["q_raw"].shape[0]
    # prologue: q/k norm + 2D rope on image rows, k norm only on text rows
    qp = O.head_norm(g["q_raw"], g["q_w"], 16, 96, g["cos"], g["sin"])
    kp = np.concatenate([O.head_norm(g["k_raw"], g["k_w"], 16, 96, g["cos"], g["sin"]),
                         O.head_norm(g["ky_raw"], g["k_w"], 16, 96)])
    np.testing.assert_allclose(qp, g["q_post"], **TOL)
    np.testing.assert_allclose(kp, g["k_post"], **TOL)
    # key bias derived from the prompt weights by the reference's forward pass
    tb = O.text_key_bias(g["txt_weights"])
    np.testing.assert_array_equal(np.isneginf(tb), np.isneginf(g["txt_bias"]))
    np.testing.assert_allclose(tb, g["txt_bias"], rtol=1e-6, atol=0)   # numpy vs torch logf: 1 ulp
    out = O.dit_joint_attention(g["q_raw"], g["k_raw"], g["v"], g["q_w"], g["k_w"], g["cos"], g["sin"],
                                g["ky_raw"], g["vy"], g["txt_bias"])
    np.testing.assert_allclose(out, g["out"], rtol=1e-4, atol=1e-5)
    assert out.shape == (L, 1536)


def test_dit_image_block(golden):
    g = golden("dit_image_block")
    out = O.dit_joint_attention(g["q_raw"], g["k_raw"], g["v"], g["q_w"], g["k_w"], g["cos"], g["sin"])
    np.testing.assert_allclose(out, g["out"], rtol=1e-4, atol=1e-5)


def test_dit_text_refine(golden):
    g = golden("dit_text_refine")
    np.testing.assert_array_equal(O.refine_keep_bias(g["txt_weights"]), g["keep_bias"])
    out = O.text_refine_attention(g["q_raw"], g["k_raw"], g["v"], g["q_w"], g["k_w"], g["keep_bias"])
    np.testing.assert_allclose(out, g["out"], rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("layer", [0, 5])
def test_gemma_layer(golden, layer):
    g = golden(f"gemma_layer{layer}")
    assert float(g["theta"]) == O.gemma_rope_theta(layer)
    L = g["q_raw"].shape[0]
    cos, sin = O.rope_1d(L, float(g["theta"]))
    np.testing.assert_allclose(O.head_norm(g["q_raw"], g["q_w"], 4, 256, cos, sin), g["q_post"], rtol=1e-4, atol=1e-4)
    np.testing.assert_allclose(O.head_norm(g["k_raw"], g["k_w"], 1, 256, cos, sin), g["k_post"], rtol=1e-4, atol=1e-4)
    # the reference's mask is the causal triangle
    m = g["mask"]
    assert np.all(np.isneginf(m[np.triu_indices(L, 1)])) and np.all(m[np.tril_indices(L)] == 0)
    out = O.gemma_attention(g["q_raw"], g["k_raw"], g["v"], g["q_w"], g["k_w"], float(g["theta"]))
    np.testing.assert_allclose(out, g["out"], rtol=1e-4, atol=2e-5)


@pytest.mark.parametrize("layer", [0, 5])
def test_gemma_attention_sublayer(golden, layer):
    """Input norm -> q/k/v linears -> head norms + RoPE -> causal attention -> o linear ->
    post-attention norm -> residual add, against gemma_encode's own layers (64-wide stream)."""
    g = golden("gemma_sublayer")
    x, want = g[f"x_in{layer}"], g[f"x_mid{layer}"]
    got = O.gemma_attention_sublayer(x, g["in_w"], g["w_q"], g["w_k"], g["w_v"], g["q_w"], g["k_w"], g["w_o"],
                                     g["post_w"], O.gemma_rope_theta(layer))
    assert got.shape == x.shape == (40, 64)
    np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-4)
    assert np.abs(want - x).max() > 0.1   # the sublayer changed the stream


def test_batched_joint_matches_unbatched(golden):
    g = golden("dit_joint_block")
    L, Lt = g["q_raw"].shape[0], g["ky_raw"].shape[0]
    C = 1536
    qkv = np.zeros((1, L + Lt, 3 * C), np.float32)
    qkv[0, :L, :C], qkv[0, :L, C:2 * C], qkv[0, :L, 2 * C:] = g["q_raw"], g["k_raw"], g["v"]
    qkv[0, L:, C:2 * C], qkv[0, L:, 2 * C:] = g["ky_raw"], g["vy"]
    out = O.joint_attention_batched(qkv, L, Lt, [L + Lt], g["q_w"], g["k_w"], g["cos"], g["sin"],
                                    bias=g["txt_bias"][None])
    np.testing.assert_allclose(out[0], g["out"], rtol=1e-4, atol=1e-5)
    # dropping the masked (w <= 0) text rows through kv_len gives the same result
    valid = int(np.sum(g["txt_weights"] > 0))
    assert np.all(g["txt_weights"][valid:] <= 0)
    out2 = O.joint_attention_batched(qkv, L, Lt, [L + valid], g["q_w"], g["k_w"], g["cos"], g["sin"],
                                     bias=g["txt_bias"][None])
    np.testing.assert_allclose(out2[0], g["out"], rtol=1e-4, atol=1e-5)


def test_vae_attention(golden):
    """The VAE decoder's attention block (tools/reference.py:352-357; app/models/vae.js:77-88): group
    norm, q/k/v 1x1 convolutions, single-head attention with head dim C over the pixels, proj_out,
    residual, against the reference's own VAE.attn (C = 64, 6 x 5 pixels)."""
    g = golden("vae_attention")
    got = O.vae_attention(g["x"], g["gn_w"], g["gn_b"], g["w_q"], g["b_q"], g["w_k"], g["b_k"], g["w_v"], g["b_v"],
                          g["w_o"], g["b_o"])
    assert got.shape == g["x"].shape == (64, 6, 5)
    np.testing.assert_allclose(got, g["y"], rtol=1e-4, atol=1e-4)
    assert np.abs(g["y"] - g["x"]).max() > 0.05   # the block changed the activation


@pytest.mark.parametrize("layer", [0, 5])
def test_gemma_mlp_sublayer(golden, layer):
    """Pre-MLP norm -> gate / up linears -> GELU-tanh GLU -> down linear -> post-MLP norm -> residual
    add, against gemma_encode's own layers: the stream after attention to the layer's output."""
    g = golden("gemma_sublayer")
    x, want = g[f"x_mid{layer}"], g[f"x_out{layer}"]
    got = O.gemma_mlp_sublayer(x, g["pre_ff_w"], g["w_gate"], g["w_up"], g["w_down"], g["post_ff_w"])
    np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-4)
    assert np.abs(want - x).max() > 0.1
    # the whole layer: attention half, then MLP half
    xin = g[f"x_in{layer}"]
    mid = O.gemma_attention_sublayer(xin, g["in_w"], g["w_q"], g["w_k"], g["w_v"], g["q_w"], g["k_w"], g["w_o"],
                                     g["post_w"], O.gemma_rope_theta(layer))
    np.testing.assert_allclose(O.gemma_mlp_sublayer(mid, g["pre_ff_w"], g["w_gate"], g["w_up"], g["w_down"],
                                                    g["post_ff_w"]), want, rtol=2e-4, atol=2e-4)


def test_torch_restatement_matches_reference_block(golden):
    """The PyTorch CPU restatement that bench.py times as the CPU baseline (oracle/torch_reference.py)
    reproduces the reference's own joint block output, and a row-limited sample gives the same rows."""
    import torch

    from oracle import torch_reference as TR
    g = golden("dit_joint_block")
    L, Lt = g["q_raw"].shape[0], g["ky_raw"].shape[0]
    qkv = np.zeros((L + Lt, 4608), np.float32)
    qkv[:L, :1536], qkv[:L, 1536:3072], qkv[:L, 3072:] = g["q_raw"], g["k_raw"], g["v"]
    qkv[L:, 1536:3072], qkv[L:, 3072:] = g["ky_raw"], g["vy"]
    T = torch.from_numpy
    out = TR.joint_attention_step(T(qkv), L, L + Lt, T(g["q_w"]), T(g["k_w"]), T(g["cos"]), T(g["sin"]),
                                  T(g["txt_bias"].astype(np.float32)))
    np.testing.assert_allclose(out.numpy(), g["out"], rtol=1e-4, atol=1e-5)
    part = TR.joint_attention_step(T(qkv), L, L + Lt, T(g["q_w"]), T(g["k_w"]), T(g["cos"]), T(g["sin"]),
                                   T(g["txt_bias"].astype(np.float32)), q_rows=7)
    np.testing.assert_allclose(part.numpy(), out.numpy()[:7], rtol=1e-5, atol=1e-6)
