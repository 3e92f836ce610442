"""nsa_rmsnorm and the Gemma layer's attention half built on it, against the CPU oracle.

* ops.rmsnorm (app/gpu/ops.js:111-116, kernels.js:62-80): fp32 and bf16 outputs, the fused
  accumulate (gemma3.js:74-77), the vector and the scalar paths, rows longer than the register cache.
* blocks.gemma_attention_sublayer (app/models/gemma3.js:62-77; tools/reference.py:187-196) against
  the reference's own layers 0 and 5 (tests/golden/gemma_sublayer.npz, a 64-wide residual stream)
  and against the oracle at the model's width (640) on a batch of two 1024-token sequences.

* ops.glu (app/gpu/ops.js:141-148): SiLU and GELU-tanh, fp32 and bf16 outputs, vector and scalar
  paths; blocks.gemma_mlp_sublayer and blocks.gemma_layer (app/models/gemma3.js:62-89) against the
  reference's layers 0 and 5 (attention half, then MLP half) and the oracle at the model's width.

Tolerances.  rmsnorm: fp32 in, fp32 math; only the order of the sum of squares differs, so 1e-5
relative.  glu: fp32 math with CUDA's tanhf / expf, 1e-5 relative (bf16 output: 2^-8).  The sublayer computes its GEMM operands in bf16 (h, q', k', v, P, a: about 2^-9 relative
each); the post-attention RMSNorm rescales o to unit RMS, so those roundings show as absolute error
on the O(1) update.  Emulating the bf16 roundings on the CPU gives 0.021 max-abs on an update of
|x| <= 3.8; the test allows 6e-2 max-abs and asks for a cosine >= 0.9999 between the updates.  The
MLP half rounds h2 and g to bf16: emulated 0.020 max-abs on an update of |x| <= 7.9; the same bounds,
and 1e-1 for a whole layer (both halves)."""

import ctypes

import numpy as np
import pytest
import torch

from oracle import attention_oracle as O

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


@pytest.fixture(scope="module", autouse=True)
def _lib_loaded():
    torch.cuda.set_device(DEV)
    from nanosaur2_web_b200 import _lib
    _lib.lib()
    yield
    torch.cuda.synchronize()


def t(x, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(x)).to(device=DEV, dtype=dtype)


def check_device():
    from nanosaur2_web_b200.ops import check_device as chk
    chk(DEV)


@pytest.mark.parametrize("rows,cols,ldx,ldy", [(1000, 640, 640, 640), (37, 100, 100, 104), (19, 101, 103, 101),
                                               (9, 2000, 2000, 2000), (1, 4, 4, 4)])
def test_rmsnorm_f32_bf16_accumulate(rows, cols, ldx, ldy):
    from nanosaur2_web_b200.ops import rmsnorm
    rng = np.random.default_rng(rows * 7 + cols)
    xs = (3.0 * rng.standard_normal((rows, ldx))).astype(np.float32)
    w = (1.0 + 0.25 * rng.standard_normal(cols)).astype(np.float32)
    x = t(xs)[:, :cols]
    want = O.rms_norm(xs[:, :cols], w, 1e-6, acc=np.float64)
    # fp32 output into a wider buffer whose other columns stay untouched
    y = torch.full((rows, ldy), 5.0, device=DEV)
    rmsnorm(x, t(w), cols, 1e-6, y[:, :cols])
    check_device()
    got = y.cpu().numpy()
    np.testing.assert_allclose(got[:, :cols], want, rtol=1e-5, atol=1e-6)
    assert (got[:, cols:] == 5.0).all()
    # bf16 output (the next GEMM's operand)
    yb = torch.empty((rows, ldy), dtype=torch.bfloat16, device=DEV)[:, :cols]
    rmsnorm(x, t(w), cols, 1e-6, yb)
    check_device()
    np.testing.assert_allclose(yb.float().cpu().numpy(), want, rtol=2 ** -8, atol=1e-6)
    # accumulate: Y += norm(X)
    base = rng.standard_normal((rows, ldy)).astype(np.float32)
    ya = t(base)
    rmsnorm(x, t(w), cols, 1e-6, ya[:, :cols], accumulate=True)
    check_device()
    got = ya.cpu().numpy()
    np.testing.assert_allclose(got[:, :cols], base[:, :cols] + want, rtol=1e-5, atol=1e-5)
    np.testing.assert_array_equal(got[:, cols:], base[:, cols:])


def test_rmsnorm_zero_rows_is_a_no_op():
    from nanosaur2_web_b200.ops import rmsnorm
    x = torch.empty((0, 640), device=DEV)
    y = rmsnorm(x, torch.ones(640, device=DEV))
    check_device()
    assert y.shape == (0, 640)


def _sublayer_inputs(g):
    w_qkv = np.concatenate([g["w_q"], g["w_k"], g["w_v"]])
    return dict(in_norm=t(g["in_w"]), w_qkv=t(w_qkv, torch.bfloat16), q_norm=t(g["q_w"]), k_norm=t(g["k_w"]),
                w_o=t(g["w_o"], torch.bfloat16), post_norm=t(g["post_w"]))


def _check_update(got, x, want, tol=6e-2):
    d, dw = got - x, want - x
    assert np.abs(got - want).max() <= tol, np.abs(got - want).max()
    cos = float(np.sum(d * dw) / (np.linalg.norm(d) * np.linalg.norm(dw)))
    assert cos >= 0.9999, cos


@pytest.mark.parametrize("layer", [0, 5])
def test_gemma_sublayer_matches_reference_layers(golden, layer):
    """The reference's gemma_encode layers 0 (local, theta 1e4) and 5 (global, 1e6), 40 tokens."""
    from nanosaur2_web_b200.blocks import GEMMA_HEAD_DIM, gemma_attention_sublayer
    from nanosaur2_web_b200.ops import ropeTable
    g = golden("gemma_sublayer")
    x_in, want = g[f"x_in{layer}"], g[f"x_mid{layer}"]
    L = x_in.shape[0]
    x = t(x_in[None])
    gemma_attention_sublayer(x, **_sublayer_inputs(g), cs=ropeTable(L, GEMMA_HEAD_DIM, O.gemma_rope_theta(layer), DEV))
    check_device()
    _check_update(x[0].cpu().numpy(), x_in, want)


def test_gemma_sublayer_model_width_batch():
    """hidden 640, B = 2 x 1024 tokens, a local layer with the 512-key window, against the oracle."""
    from nanosaur2_web_b200.blocks import GEMMA_HEAD_DIM, gemma_attention_sublayer, gemma_sublayer_buffers
    from nanosaur2_web_b200.ops import ropeTable
    from tests._helpers import bf16_round
    B, L, Hd, window = 2, 1024, 640, 512
    rng = np.random.default_rng(11)
    g = {"in_w": (1.0 + 0.25 * rng.standard_normal(Hd)).astype(np.float32),
         "post_w": (1.0 + 0.25 * rng.standard_normal(Hd)).astype(np.float32),
         "q_w": (1.0 + 0.25 * rng.standard_normal(256)).astype(np.float32),
         "k_w": (1.0 + 0.25 * rng.standard_normal(256)).astype(np.float32),
         "w_q": bf16_round(rng.standard_normal((1024, Hd), dtype=np.float32) / np.sqrt(Hd)),
         "w_k": bf16_round(rng.standard_normal((256, Hd), dtype=np.float32) / np.sqrt(Hd)),
         "w_v": bf16_round(rng.standard_normal((256, Hd), dtype=np.float32) / np.sqrt(Hd)),
         "w_o": bf16_round(rng.standard_normal((Hd, 1024), dtype=np.float32) / 32.0)}
    x_in = (8.0 * rng.standard_normal((B, L, Hd))).astype(np.float32)
    x = t(x_in)
    bufs = gemma_sublayer_buffers(B, L, Hd, DEV)
    gemma_attention_sublayer(x, **_sublayer_inputs(g), cs=ropeTable(L, GEMMA_HEAD_DIM, 1e4, DEV), window=window,
                             buffers=bufs)
    check_device()
    got = x.cpu().numpy()
    for b in range(B):
        want = O.gemma_attention_sublayer(x_in[b], g["in_w"], g["w_q"], g["w_k"], g["w_v"], g["q_w"], g["k_w"],
                                          g["w_o"], g["post_w"], 1e4, window=window)
        _check_update(got[b], x_in[b], want)


@pytest.mark.parametrize("rows,I,ldx,ldy", [(1000, 2048, 4096, 2048), (17, 101, 210, 103), (3, 4, 8, 4)])
@pytest.mark.parametrize("act", ["silu", "gelu_tanh"])
def test_glu(rows, I, ldx, ldy, act):
    from nanosaur2_web_b200.ops import glu
    rng = np.random.default_rng(rows + I)
    xs = (3.0 * rng.standard_normal((rows, ldx))).astype(np.float32)
    x = t(xs)[:, :2 * I]
    want = O.glu(xs[:, :2 * I], act, acc=np.float64)
    y = torch.full((rows, ldy), 9.0, device=DEV)
    glu(x, act, out=y[:, :I])
    check_device()
    got = y.cpu().numpy()
    np.testing.assert_allclose(got[:, :I], want, rtol=1e-5, atol=1e-5)
    assert (got[:, I:] == 9.0).all()
    yb = glu(x, act, out_dtype=torch.bfloat16)
    check_device()
    np.testing.assert_allclose(yb.float().cpu().numpy(), want, rtol=2 ** -8, atol=1e-5)


def _mlp_inputs(g):
    return dict(pre_norm=t(g["pre_ff_w"]), w_gate_up=t(np.concatenate([g["w_gate"], g["w_up"]]), torch.bfloat16),
                w_down=t(g["w_down"], torch.bfloat16), post_norm=t(g["post_ff_w"]))


@pytest.mark.parametrize("layer", [0, 5])
def test_gemma_layer_matches_reference_layers(golden, layer):
    """The reference's gemma_encode layers 0 and 5, 40 tokens: the MLP half from the stream after
    attention, and the whole layer (attention half, then MLP half) from the layer input."""
    from nanosaur2_web_b200.blocks import GEMMA_HEAD_DIM, gemma_layer, gemma_mlp_sublayer
    from nanosaur2_web_b200.ops import ropeTable
    g = golden("gemma_sublayer")
    x_mid, x_out, x_in = g[f"x_mid{layer}"], g[f"x_out{layer}"], g[f"x_in{layer}"]
    x = t(x_mid[None])
    gemma_mlp_sublayer(x, **_mlp_inputs(g))
    check_device()
    _check_update(x[0].cpu().numpy(), x_mid, x_out)
    x = t(x_in[None])
    gemma_layer(x, attn=_sublayer_inputs(g), mlp=_mlp_inputs(g),
                cs=ropeTable(x_in.shape[0], GEMMA_HEAD_DIM, O.gemma_rope_theta(layer), DEV))
    check_device()
    _check_update(x[0].cpu().numpy(), x_in, x_out, tol=1e-1)


@pytest.mark.parametrize("fused", [False, True])
def test_gemma_mlp_model_width(fused):
    """hidden 640, MLP width 2048 (Gemma3-270M), B = 2 x 256 tokens, against the oracle; ``fused``
    runs the GLU in the gate_up linear's epilogue (interleaved weight), which gives the same bits."""
    from nanosaur2_web_b200.blocks import gemma_mlp_buffers, gemma_mlp_sublayer
    from nanosaur2_web_b200.ops import glu_interleave
    from tests._helpers import bf16_round
    B, L, Hd, I = 2, 256, 640, 2048
    rng = np.random.default_rng(12)
    pre = (1.0 + 0.25 * rng.standard_normal(Hd)).astype(np.float32)
    post = (1.0 + 0.25 * rng.standard_normal(Hd)).astype(np.float32)
    wg = bf16_round(rng.standard_normal((I, Hd), dtype=np.float32) / np.sqrt(Hd))
    wu = bf16_round(rng.standard_normal((I, Hd), dtype=np.float32) / np.sqrt(Hd))
    wd = bf16_round(rng.standard_normal((Hd, I), dtype=np.float32) / np.sqrt(I))
    x_in = (8.0 * rng.standard_normal((B, L, Hd))).astype(np.float32)
    x = t(x_in)
    wgu = t(np.concatenate([wg, wu]), torch.bfloat16)
    gemma_mlp_sublayer(x, pre_norm=t(pre), w_gate_up=glu_interleave(wgu) if fused else wgu,
                       w_down=t(wd, torch.bfloat16), post_norm=t(post), buffers=gemma_mlp_buffers(B, L, Hd, I, DEV, fused),
                       gate_up_interleaved=fused)
    check_device()
    got = x.cpu().numpy()
    if fused:
        x2 = t(x_in)
        gemma_mlp_sublayer(x2, pre_norm=t(pre), w_gate_up=wgu, w_down=t(wd, torch.bfloat16), post_norm=t(post))
        check_device()
        np.testing.assert_array_equal(got, x2.cpu().numpy())
    for b in range(B):
        _check_update(got[b], x_in[b], O.gemma_mlp_sublayer(x_in[b], pre, wg, wu, wd, post, acc=np.float64))


@pytest.mark.parametrize("cols,z_dtype", [(640, torch.bfloat16), (640, torch.float32), (1000, torch.bfloat16)])
def test_rmsnorm_chained_next_norm_matches_two_passes(cols, z_dtype):
    """Y += rmsnorm(X) * w with the next norm Z = rmsnorm(new Y) * w2 in the same pass (gemma3.js:74-79)
    gives the bits of the accumulate followed by a separate rmsnorm; 640 columns stay in registers,
    1000 also re-read the rest of the row."""
    from nanosaur2_web_b200.ops import NsaError, rmsnorm
    rng = np.random.default_rng(70 + cols)
    rows = 333
    xs = rng.standard_normal((rows, cols), dtype=np.float32) * 3
    ys = rng.standard_normal((rows, cols), dtype=np.float32) * 5
    w = (1 + 0.2 * rng.standard_normal(cols)).astype(np.float32)
    w2 = (1 + 0.2 * rng.standard_normal(cols)).astype(np.float32)
    y1, y2 = t(ys), t(ys)
    z1 = torch.empty((rows, cols), dtype=z_dtype, device=DEV)
    rmsnorm(t(xs), t(w), cols, 1e-6, y1, accumulate=True)
    rmsnorm(y1, t(w2), cols, 1e-6, z1)
    z2 = torch.full((rows, cols), 7.0, dtype=z_dtype, device=DEV)
    rmsnorm(t(xs), t(w), cols, 1e-6, y2, accumulate=True, next_weight=t(w2), next_out=z2)
    check_device()
    np.testing.assert_array_equal(y2.cpu().numpy(), y1.cpu().numpy())
    np.testing.assert_array_equal(z2.float().cpu().numpy(), z1.float().cpu().numpy())
    want_y = ys.astype(np.float64) + O.rms_norm(xs, w, acc=np.float64)
    np.testing.assert_allclose(y2.cpu().numpy(), want_y, rtol=1e-5, atol=1e-4)
    np.testing.assert_allclose(z2.float().cpu().numpy(), O.rms_norm(want_y, w2, acc=np.float64),
                               rtol=2 ** -7 if z_dtype == torch.bfloat16 else 1e-4, atol=1e-3)
    with pytest.raises(NsaError, match="next_weight needs accumulate"):
        from nanosaur2_web_b200 import _lib
        d = _lib.RmsnormDesc()
        d.rows, d.cols, d.eps, d.out_dtype = rows, cols, 1e-6, _lib.NSA_F32
        d.next_weight, d.Z, d.z_dtype = t(w2).data_ptr(), z2.data_ptr(), _lib.NSA_BF16
        _lib.check(_lib.lib().nsa_rmsnorm(ctypes.byref(d), t(xs).data_ptr(), t(w).data_ptr(), y2.data_ptr(), None))


def test_gemma_layers_chained_norms_match_separate():
    """Two whole Gemma layers with the norms chained (post-attention accumulate -> pre-MLP norm,
    post-MLP accumulate -> the next layer's input norm, four fewer passes over x) give the bits of
    the same layers with every norm its own pass."""
    from nanosaur2_web_b200.blocks import (GEMMA_HEAD_DIM, gemma_attention_sublayer, gemma_layer,
                                           gemma_mlp_buffers, gemma_mlp_sublayer, gemma_sublayer_buffers)
    from nanosaur2_web_b200.ops import glu_interleave, ropeTable
    B, L, Hd, I = 2, 256, 640, 2048
    rng = np.random.default_rng(71)

    def norm(n):
        return t((1.0 + 0.2 * rng.standard_normal(n)).astype(np.float32))

    def lin(o, i):
        return t(rng.standard_normal((o, i), dtype=np.float32) / np.sqrt(i), torch.bfloat16)

    layers = []
    for _ in range(2):
        layers.append(({"in_norm": norm(Hd), "post_norm": norm(Hd), "q_norm": norm(GEMMA_HEAD_DIM),
                        "k_norm": norm(GEMMA_HEAD_DIM), "w_qkv": lin(1536, Hd), "w_o": lin(Hd, 1024)},
                       {"pre_norm": norm(Hd), "post_norm": norm(Hd), "w_gate_up": glu_interleave(lin(2 * I, Hd)),
                        "w_down": lin(Hd, I), "gate_up_interleaved": True}))
    cs = ropeTable(L, GEMMA_HEAD_DIM, 1e4, DEV)
    x_in = (8.0 * rng.standard_normal((B, L, Hd))).astype(np.float32)
    x1 = t(x_in)
    for attn, mlp in layers:
        gemma_attention_sublayer(x1, **attn, cs=cs, window=128)
        gemma_mlp_sublayer(x1, **mlp)
    x2 = t(x_in)
    bufs = (gemma_sublayer_buffers(B, L, Hd, DEV), gemma_mlp_buffers(B, L, Hd, I, DEV, True))
    for li, (attn, mlp) in enumerate(layers):
        gemma_layer(x2, attn=attn, mlp=mlp, cs=cs, window=128, buffers=bufs, h_ready=li > 0,
                    next_norm=layers[li + 1][0]["in_norm"] if li + 1 < len(layers) else None)
    check_device()
    np.testing.assert_array_equal(x2.cpu().numpy(), x1.cpu().numpy())
