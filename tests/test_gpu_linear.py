"""nsa_linear (ops.linear with the epilogue of the reference's tiled GEMM) against the CPU oracle:
the reference's lin (tools/reference.py:208-210, pinned by tests/golden/linear.npz) and the GEMM
epilogue (app/gpu/gemm.js:155-165).  Operands are bf16 and the oracle runs in float64 on the same
bf16 values, so the only difference is the fp32 accumulation order."""

import numpy as np
import pytest
import torch

from oracle import attention_oracle as O
from tests._helpers import bf16_round, lora_oracle as _lora_oracle

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


def operands(seed, M, N, K):
    rng = np.random.default_rng(seed)
    a = bf16_round(rng.standard_normal((M, K), dtype=np.float32))
    w = bf16_round(rng.standard_normal((N, K), dtype=np.float32) / np.sqrt(K))
    b = (0.1 * rng.standard_normal(N)).astype(np.float32)
    return rng, a, w, b


def test_dit_output_projection_gated_residual():
    """x += gate[2C + n] * (a @ W_proj^T + b) over 3952 rows, C = 1536 (app/models/nanosaur2.js:210)."""
    from nanosaur2_web_b200.ops import linear
    M, C = 3952, 1536
    rng, a, w, b = operands(3, M, C, C)
    x = rng.standard_normal((M, C), dtype=np.float32)
    mod = rng.standard_normal(6 * C).astype(np.float32)
    out = t(x)
    linear(t(a, torch.bfloat16), t(w, torch.bfloat16), bias=t(b), out=out, resid=True, gate=t(mod), gOff=2 * C)
    check_device()
    want = O.linear_epilogue(O.linear(a, w, b, acc=np.float64), x, mod[2 * C:3 * C], resid=True, acc=np.float64)
    np.testing.assert_allclose(out.cpu().numpy(), want, rtol=1e-3, atol=2e-3)


def test_linear_ragged_silu_column_window():
    """M, N, K off the tiles (300 x 200, K = 200: partial row / column tiles and a partial K slice),
    alpha 0.5, silu, written into columns [8, 208) of a wider output that keeps its other columns."""
    from nanosaur2_web_b200.ops import linear
    M, N, K = 300, 200, 200
    _, a, w, b = operands(4, M, N, K)
    out = torch.full((M, 216), 7.0, device=DEV)
    linear(t(a, torch.bfloat16), t(w, torch.bfloat16), bias=t(b), out=out, act="silu", cOff=8, alpha=0.5)
    check_device()
    y = 0.5 * O.linear(a, w, acc=np.float64) + b
    want = O.linear_epilogue(y, act="silu", acc=np.float64)
    got = out.cpu().numpy()
    np.testing.assert_allclose(got[:, 8:208], want, rtol=1e-3, atol=2e-3)
    assert (got[:, :8] == 7.0).all() and (got[:, 208:] == 7.0).all()


def test_linear_plain_residual_without_bias():
    from nanosaur2_web_b200.ops import linear
    M, N, K = 129, 512, 64
    rng, a, w, _ = operands(5, M, N, K)
    x = rng.standard_normal((M, N), dtype=np.float32)
    out = t(x)
    linear(t(a, torch.bfloat16), t(w, torch.bfloat16), out=out, resid=True)
    check_device()
    want = O.linear_epilogue(O.linear(a, w, acc=np.float64), x, resid=True, acc=np.float64)
    np.testing.assert_allclose(out.cpu().numpy(), want, rtol=1e-3, atol=2e-3)


# ----------------------------------------------------------------------------- ConvRot int8 and LoRA
# The int8 weights are exact integers in the bf16 operand the tensor core reads, so the int8 product is
# compared with the oracle on the same (rotated, bf16-rounded) input at the fp32-accumulation bound.
# The LoRA side path is evaluated as bf16 T = x A_cat^T and bf16 B_cat = scale B / (alpha w_scale); the
# oracle emulates those two roundings, and the bound adds one bf16 step of the delta.

def test_rotate_matches_oracle():
    """ops.rotate (app/gpu/ops.js:38-45) over 300 rows x 1536 columns (6 groups of 256), fp32 and bf16
    in and out, with row pitches wider than the rows."""
    from nanosaur2_web_b200.ops import rotate
    rng = np.random.default_rng(21)
    x = rng.standard_normal((300, 1544), dtype=np.float32)
    want = O.rotate(x[:, :1536], acc=np.float64)
    xt = t(x)[:, :1536]
    y32 = rotate(xt)
    out = torch.full((300, 1560), 5.0, device=DEV, dtype=torch.bfloat16)
    rotate(xt, out=out[:, :1536])
    check_device()
    np.testing.assert_allclose(y32.cpu().numpy(), want, rtol=1e-5, atol=1e-5)
    got = out.float().cpu().numpy()
    np.testing.assert_allclose(got[:, :1536], want, rtol=2 ** -8, atol=1e-6)
    assert (got[:, 1536:] == 5.0).all()
    xb = bf16_round(x[:, :1536])
    y16 = rotate(t(xb, torch.bfloat16), out_dtype=torch.bfloat16)
    check_device()
    np.testing.assert_allclose(y16.float().cpu().numpy(), O.rotate(xb, acc=np.float64), rtol=2 ** -8, atol=1e-6)


def test_int8_convrot_linear_golden(golden):
    """The reference's own int8 layer (tools/quant.py quantiser, tools/reference.py loader and lin,
    tests/golden/convrot.npz): x rotated on the GPU, int8 GEMM with row scales and bias."""
    from nanosaur2_web_b200.ops import linear, rotate
    g = golden("convrot")
    xr = rotate(t(g["x"]), out_dtype=torch.bfloat16)
    y = linear(xr, t(g["q"], torch.int8), bias=t(g["b"]), w_scale=t(g["scale"]))
    check_device()
    xr_np = xr.float().cpu().numpy()
    np.testing.assert_allclose(xr_np, O.rotate(g["x"], acc=np.float64), rtol=2 ** -8, atol=1e-6)
    want = O.linear_int8(xr_np, g["q"], g["scale"], g["b"], acc=np.float64)
    np.testing.assert_allclose(y.cpu().numpy(), want, rtol=1e-4, atol=1e-4)
    # end to end against the reference's fp32 result: the bf16 rounding of the rotated input
    np.testing.assert_allclose(y.cpu().numpy(), g["y_base"], rtol=1e-2, atol=2e-2)


def assert_close_with_bound(got, want, bound, rtol=1e-3, atol=2e-3):
    err = np.abs(np.asarray(got, np.float64) - want)
    lim = rtol * np.abs(want) + atol + bound
    bad = err > lim
    assert not bad.any(), f"{bad.sum()} elements off; worst excess {(err - lim).max():.3g}"


def test_int8_convrot_linear_loras_golden(golden):
    """Two LoRAs (PEFT with alpha, kohya without) on the int8 layer; A rows rotated on the GPU as the
    reference's loader does (app/lora.js:126); against the reference's merged weight."""
    from nanosaur2_web_b200.ops import linear, lora_pack, rotate
    g = golden("convrot")
    N, K = g["q"].shape
    r1 = g["a1"].shape[0]
    ents = [dict(A=t(g["a1"]), B=t(g["b1"]), scale=float(g["s1"]) * float(g["alpha1"]) / r1),
            dict(A=t(g["a2"]), B=t(g["b2"]), scale=float(g["s2"]))]
    scale = t(g["scale"])
    pack = lora_pack(ents, N, K, w_scale=scale, rotate_a=True)
    assert pack.R == 64
    xr = rotate(t(g["x"]), out_dtype=torch.bfloat16)
    y = linear(xr, t(g["q"], torch.int8), bias=t(g["b"]), w_scale=scale, lora=pack)
    check_device()
    xr_np = xr.float().cpu().numpy()
    rot = [dict(e, A=O.rotate(g[a], acc=np.float64).astype(np.float32), B=g[b])
           for e, a, b in ((ents[0], "a1", "b1"), (ents[1], "a2", "b2"))]
    want, bound = _lora_oracle(xr_np, g["q"], g["scale"], g["b"], rot, N)
    assert_close_with_bound(y.cpu().numpy(), want, bound, rtol=1e-3, atol=1e-3)
    np.testing.assert_allclose(y.cpu().numpy(), g["y_lora"], rtol=1e-2, atol=3e-2)


def test_int8_linear_dit_shape_gated_residual_with_lora_slices():
    """The DiT output projection's shape (M 1000, N = K = 1536) with int8 weights, the gated residual,
    and two LoRA entries on column slices (the stacked-weight form, app/lora.js:149 off / n)."""
    from nanosaur2_web_b200.ops import linear, lora_pack
    rng = np.random.default_rng(33)
    M, N, K = 1000, 1536, 1536
    xr = bf16_round(rng.standard_normal((M, K), dtype=np.float32))
    q = rng.integers(-128, 128, size=(N, K), dtype=np.int8)
    scale = (rng.uniform(0.5, 2.0, N) / (127 * np.sqrt(K))).astype(np.float32)
    b = (0.1 * rng.standard_normal(N)).astype(np.float32)
    x0 = rng.standard_normal((M, N), dtype=np.float32)
    mod = rng.standard_normal(3 * N).astype(np.float32)
    ents = [dict(A=rng.standard_normal((16, K), dtype=np.float32) / 40, B=rng.standard_normal((512, 16), dtype=np.float32) / 4,
                 scale=0.7, off=0, n=512),
            dict(A=rng.standard_normal((24, K), dtype=np.float32) / 40, B=rng.standard_normal((1024, 24), dtype=np.float32) / 4,
                 scale=-0.3, off=512, n=1024)]
    pack = lora_pack([dict(e, A=t(e["A"]), B=t(e["B"])) for e in ents], N, K, w_scale=t(scale))
    out = t(x0)
    linear(t(xr, torch.bfloat16), t(q, torch.int8), bias=t(b), w_scale=t(scale), lora=pack, out=out, resid=True,
           gate=t(mod), gOff=N)
    check_device()
    y, bound = _lora_oracle(xr, q, scale, b, ents, N)
    want = O.linear_epilogue(y, x0, mod[N:2 * N], resid=True, acc=np.float64)
    assert_close_with_bound(out.cpu().numpy(), want, bound * np.abs(mod[N:2 * N]))


def test_bf16_linear_lora_alpha_silu_and_bf16_output():
    """bf16 weights with a LoRA, alpha 0.5 (folded out of B_cat and back in the epilogue), silu, and the
    bf16 store form; ragged M / N / K."""
    from nanosaur2_web_b200.ops import linear, lora_pack
    rng, a, w, b = operands(34, 300, 200, 200)
    ents = [dict(A=rng.standard_normal((8, 200), dtype=np.float32) / 8, B=rng.standard_normal((200, 8), dtype=np.float32) / 4,
                 scale=1.5)]
    pack = lora_pack([dict(e, A=t(e["A"]), B=t(e["B"])) for e in ents], 200, 200, alpha=0.5)
    y32 = linear(t(a, torch.bfloat16), t(w, torch.bfloat16), bias=t(b), act="silu", alpha=0.5, lora=pack)
    y16 = linear(t(a, torch.bfloat16), t(w, torch.bfloat16), bias=t(b), act="silu", alpha=0.5, lora=pack,
                 out_dtype=torch.bfloat16)
    check_device()
    y, bound = _lora_oracle(a, w, None, b, ents, 200, alpha=0.5)
    want = O.linear_epilogue(y, act="silu", acc=np.float64)
    assert_close_with_bound(y32.cpu().numpy(), want, bound * 1.1)   # silu' <= 1.1
    # the bf16 store form is the fp32 result rounded once (same tiles, same summation order)
    np.testing.assert_array_equal(y16.float().cpu().numpy(), bf16_round(y32.cpu().numpy()))
    with pytest.raises(Exception, match="another alpha"):
        linear(t(a, torch.bfloat16), t(w, torch.bfloat16), lora=pack)


@pytest.mark.parametrize("N", [640, 352, 96])
def test_linear_half_width_last_tile(N):
    """Column counts whose last 256-wide tile holds at most 128 columns (te.o and the MLP down
    projection at N = 640): that tile multiplies only its first 128 weight rows; a plain store and a
    gated residual both match the oracle."""
    from nanosaur2_web_b200.ops import linear
    M, K = 300, 1024
    rng, a, w, b = operands(40 + N, M, N, K)
    y = linear(t(a, torch.bfloat16), t(w, torch.bfloat16), bias=t(b))
    x0 = rng.standard_normal((M, N), dtype=np.float32)
    g = rng.standard_normal(N).astype(np.float32)
    out = t(x0)
    linear(t(a, torch.bfloat16), t(w, torch.bfloat16), bias=t(b), out=out, resid=True, gate=t(g))
    check_device()
    want = O.linear(a, w, b, acc=np.float64)
    np.testing.assert_allclose(y.cpu().numpy(), want, rtol=1e-3, atol=2e-3)
    np.testing.assert_allclose(out.cpu().numpy(), O.linear_epilogue(want, x0, g, resid=True, acc=np.float64),
                               rtol=1e-3, atol=2e-3)


def _interleave_rows(x, I):
    """The fused GLU's row order (nsa_glu_interleave): row 256 j + i = gate row 128 j + i (i < 128),
    else up row I + 128 j + i - 128."""
    idx = np.concatenate([np.concatenate([np.arange(128 * j, 128 * j + 128), I + np.arange(128 * j, 128 * j + 128)])
                          for j in range(I // 128)])
    return x[idx]


@pytest.mark.parametrize("act,out_dtype", [("gelu_tanh", torch.bfloat16), ("silu", torch.float32),
                                           ("gelu_tanh", torch.float32)])
def test_fused_glu_linear_matches_linear_then_glu(act, out_dtype):
    """The gate_up linear with ops.glu in its epilogue (app/models/gemma3.js:80-81): ragged M = 300,
    K = 200 (a partial K slice), I = 384 (three tiles); interleaved weight and bias.  Same MMAs and the
    same activation code as nsa_linear + nsa_glu, so the two paths agree to the last bit; both match
    the float64 oracle."""
    from nanosaur2_web_b200.ops import glu, glu_interleave, linear
    M, I, K = 300, 384, 200
    rng, a, w, b = operands(50, M, 2 * I, K)
    wi, bi = glu_interleave(t(w, torch.bfloat16)), glu_interleave(t(b))
    np.testing.assert_array_equal(wi.float().cpu().numpy(), _interleave_rows(w, I))
    np.testing.assert_array_equal(bi.cpu().numpy(), _interleave_rows(b, I))
    fused = linear(t(a, torch.bfloat16), wi, bias=bi, glu=act, out_dtype=out_dtype)
    gu = linear(t(a, torch.bfloat16), t(w, torch.bfloat16), bias=t(b))
    plain = glu(gu, act, out_dtype=out_dtype)
    check_device()
    assert fused.shape == (M, I) and fused.dtype == out_dtype
    np.testing.assert_array_equal(fused.float().cpu().numpy(), plain.float().cpu().numpy())
    want = O.glu(O.linear(a, w, b, acc=np.float64), act, acc=np.float64)
    tol = 2 ** -8 if out_dtype == torch.bfloat16 else 1e-3
    np.testing.assert_allclose(fused.float().cpu().numpy(), want, rtol=tol, atol=2e-3)


def test_fused_glu_int8_column_window():
    """int8 ConvRot gate_up weights with interleaved row scales, alpha 0.5, written into columns
    [64, 64 + I) of a wider bf16 output that keeps its other columns; against linear + glu."""
    from nanosaur2_web_b200.ops import glu, glu_interleave, linear
    M, I, K = 260, 256, 512
    rng = np.random.default_rng(51)
    xr = bf16_round(rng.standard_normal((M, K), dtype=np.float32))
    q = rng.integers(-127, 128, size=(2 * I, K), dtype=np.int8)
    scale = (0.02 * (1 + rng.random(2 * I))).astype(np.float32)
    b = (0.1 * rng.standard_normal(2 * I)).astype(np.float32)
    out = torch.full((M, I + 128), 7.0, dtype=torch.bfloat16, device=DEV)
    linear(t(xr, torch.bfloat16), glu_interleave(t(q, torch.int8)), bias=glu_interleave(t(b)),
           w_scale=glu_interleave(t(scale)), alpha=0.5, glu="silu", out=out, cOff=64)
    gu = linear(t(xr, torch.bfloat16), t(q, torch.int8), bias=t(b), w_scale=t(scale), alpha=0.5)
    plain = glu(gu, "silu", out_dtype=torch.bfloat16)
    check_device()
    got = out.float().cpu().numpy()
    np.testing.assert_array_equal(got[:, 64:64 + I], plain.float().cpu().numpy())
    assert (got[:, :64] == 7.0).all() and (got[:, 64 + I:] == 7.0).all()


def test_fused_glu_rejects_unsupported_forms():
    """N off the 256-row tiles, resid, act and LoRA do not combine with the fused GLU."""
    from nanosaur2_web_b200.ops import NsaError, linear
    _, a, w, b = operands(52, 64, 384, 64)
    with pytest.raises(NsaError, match="fused GLU"):
        linear(t(a, torch.bfloat16), t(w, torch.bfloat16), glu="silu")
    _, a, w, b = operands(53, 64, 512, 64)
    out = torch.zeros((64, 256), device=DEV)
    with pytest.raises(NsaError, match="fused GLU"):
        linear(t(a, torch.bfloat16), t(w, torch.bfloat16), glu="silu", out=out, resid=True)
    with pytest.raises(NsaError, match="fused GLU"):
        linear(t(a, torch.bfloat16), t(w, torch.bfloat16), glu="silu", act="silu")


def test_expanded_int8_weight_matches_int8_path():
    """An int8 ConvRot weight expanded once to bf16 (nsa_expand_i8) with the same row scales gives the
    int8 path's bits at the bf16 MMA rate: plain store (N = 640, a half-width last tile), and a gated
    residual with a LoRA packed for the scaled weight."""
    from nanosaur2_web_b200.ops import expand_i8, linear, lora_pack
    M, N, K = 300, 640, 512
    rng = np.random.default_rng(54)
    xr = t(bf16_round(rng.standard_normal((M, K), dtype=np.float32)), torch.bfloat16)
    q = t(rng.integers(-127, 128, size=(N, K), dtype=np.int8), torch.int8)
    scale = t((0.02 * (1 + rng.random(N))).astype(np.float32))
    b = t((0.1 * rng.standard_normal(N)).astype(np.float32))
    wx = expand_i8(q)
    np.testing.assert_array_equal(wx.float().cpu().numpy(), q.float().cpu().numpy())
    np.testing.assert_array_equal(linear(xr, wx, bias=b, w_scale=scale).cpu().numpy(),
                                  linear(xr, q, bias=b, w_scale=scale).cpu().numpy())
    ents = [dict(A=t(rng.standard_normal((16, K), dtype=np.float32) / 16),
                 B=t(rng.standard_normal((N, 16), dtype=np.float32) / 4), scale=0.7)]
    pack = lora_pack(ents, N, K, w_scale=scale)
    x0 = rng.standard_normal((M, N), dtype=np.float32)
    g = t(rng.standard_normal(N).astype(np.float32))
    o8, ox = t(x0), t(x0)
    linear(xr, q, bias=b, w_scale=scale, lora=pack, out=o8, resid=True, gate=g)
    linear(xr, wx, bias=b, w_scale=scale, lora=pack, out=ox, resid=True, gate=g)
    check_device()
    np.testing.assert_array_equal(ox.cpu().numpy(), o8.cpu().numpy())
    with pytest.raises(Exception, match="another alpha or weight format"):
        linear(xr, wx, lora=pack)


@pytest.mark.parametrize("case", ["gated_ragged", "gated_k2056", "lora_silu_bf16", "glu", "half_tile_f32",
                                  "expanded_i8_lora"])
def test_cta_pair_schedule_matches_single(case):
    """The CTA-pair schedule (two CTAs per 256 x 256 tile, 128-wide K steps) and the single-CTA one
    (128 x 256 tiles, 64-wide K steps) add the same products in the same order: equal bits, for ragged
    M / K, LoRA slices, the fused GLU, a half-width last column tile and row-scaled (expanded int8)
    weights; also against the oracle."""
    from nanosaur2_web_b200.ops import expand_i8, glu_interleave, linear, lora_pack
    rng = np.random.default_rng(60)
    if case == "gated_ragged":
        M, N, K = 600, 512, 1544
    elif case == "gated_k2056":
        M, N, K = 600, 512, 2056
    elif case == "lora_silu_bf16":
        M, N, K = 300, 768, 1536
    elif case == "glu":
        M, N, K = 392, 768, 640
    elif case == "half_tile_f32":
        M, N, K = 1000, 640, 2048
    else:
        M, N, K = 260, 384, 1024
    a = bf16_round(rng.standard_normal((M, K), dtype=np.float32))
    w = bf16_round(rng.standard_normal((N, K), dtype=np.float32) / np.sqrt(K))
    b = (0.1 * rng.standard_normal(N)).astype(np.float32)
    A, W, Bv = t(a, torch.bfloat16), t(w, torch.bfloat16), t(b)

    def run(schedule):
        if case in ("gated_ragged", "gated_k2056"):
            x0, g = rng.standard_normal((M, N), dtype=np.float32), rng.standard_normal(N).astype(np.float32)
            out = t(x0)
            linear(A, W, bias=Bv, out=out, resid=True, gate=t(g), schedule=schedule)
            return out, O.linear_epilogue(O.linear(a, w, b, acc=np.float64), x0, g, resid=True, acc=np.float64)
        if case == "lora_silu_bf16":
            ents = [dict(A=t(np.full((8, K), 0.01, np.float32)), B=t(np.full((N, 8), 0.02, np.float32)), scale=0.5)]
            pack = lora_pack(ents, N, K)
            return linear(A, W, bias=Bv, act="silu", lora=pack, out_dtype=torch.bfloat16, schedule=schedule), None
        if case == "glu":
            return linear(A, glu_interleave(W), bias=glu_interleave(Bv), glu="gelu_tanh", schedule=schedule), \
                O.glu(O.linear(a, w, b, acc=np.float64), "gelu_tanh", acc=np.float64)
        if case == "half_tile_f32":
            return linear(A, W, bias=Bv, schedule=schedule), O.linear(a, w, b, acc=np.float64)
        q = t(rng.integers(-127, 128, size=(N, K), dtype=np.int8), torch.int8)
        sc = t((0.02 * (1 + rng.random(N))).astype(np.float32))
        ents = [dict(A=t(rng.standard_normal((16, K), dtype=np.float32) / 16),
                     B=t(rng.standard_normal((N, 16), dtype=np.float32) / 4), scale=0.7)]
        return linear(A, expand_i8(q), bias=Bv, w_scale=sc, lora=lora_pack(ents, N, K, w_scale=sc),
                      schedule=schedule), None

    state = rng.bit_generator.state
    y1, want = run("single")
    rng.bit_generator.state = state
    y2, _ = run("pair")
    check_device()
    np.testing.assert_array_equal(y2.float().cpu().numpy(), y1.float().cpu().numpy())
    if want is not None:
        np.testing.assert_allclose(y2.float().cpu().numpy(), want, rtol=1e-3, atol=2e-3)


def test_cta_pair_schedule_rejects_int8_and_one_row_tile():
    from nanosaur2_web_b200.ops import NsaError, linear
    _, a, w, b = operands(61, 64, 256, 64)
    with pytest.raises(NsaError, match="CTA pairs"):
        linear(t(a, torch.bfloat16), t(w, torch.bfloat16), schedule="pair")
    with pytest.raises(NsaError, match="CTA pairs"):
        linear(t(a, torch.bfloat16), t(np.zeros((256, 64), np.int8), torch.int8), w_scale=t(np.ones(256, np.float32)),
               schedule="pair")
