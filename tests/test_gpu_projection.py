"""The QKV projection with the prologue in its GEMM epilogue (nsa_seq_shard_projection, through
``blocks.dit_block_attention_projected``) against the CPU oracle: the reference's linear
(tools/reference.py:208-210, pinned by tests/golden/linear.npz) followed by the DiT block's head
norms, 2D RoPE and joint attention (:272-286).  Inputs are bf16; the oracle runs in float64 on the
same bf16 values.  Tolerance of the bf16 path: max-abs <= 2e-2 and per-head cosine >= 0.9999."""

import numpy as np
import pytest
import torch

from oracle import attention_oracle as O
from tests._helpers import assert_close_bf16, bf16_round

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
C, H, D = 1536, 16, 96


@pytest.fixture(scope="module", autouse=True)
def _lib_loaded():
    torch.cuda.set_device(DEV)
    from nanosaur2_web_b200 import _lib
    _lib.lib()
    yield
    torch.cuda.synchronize()


def t(x, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(x)).to(device=DEV, dtype=dtype)


def proj_inputs(seed, B, L, Lt, K, lv_range):
    """Block input rows, q|k|v and k|v weights (Linear layout, ~unit-variance outputs), biases,
    norm weights, valid text lengths and log prompt-weight biases."""
    rng = np.random.default_rng(seed)
    x = bf16_round(rng.standard_normal((B, L, K), dtype=np.float32))
    w = bf16_round(rng.standard_normal((3 * C, K), dtype=np.float32) / np.sqrt(K))
    b = (0.1 * rng.standard_normal(3 * C)).astype(np.float32)
    xt = bf16_round(rng.standard_normal((B, Lt, K), dtype=np.float32)) if Lt else None
    wkv = bf16_round(rng.standard_normal((2 * C, K), dtype=np.float32) / np.sqrt(K)) if Lt else None
    bkv = (0.1 * rng.standard_normal(2 * C)).astype(np.float32) if Lt else None
    q_w = (1.0 + 0.2 * rng.standard_normal(D)).astype(np.float32)
    k_w = (1.0 + 0.2 * rng.standard_normal(D)).astype(np.float32)
    lv = rng.integers(lv_range[0], lv_range[1] + 1, size=B).astype(np.int32) if Lt else np.zeros(B, np.int32)
    bias = np.log(rng.choice(np.array([0.7, 1.0, 1.3], np.float32), size=(B, Lt))).astype(np.float32) if Lt else None
    return x, w, b, xt, wkv, bkv, q_w, k_w, lv, bias


def oracle_qkv(x, w, b, xt, wkv, bkv):
    """The packed qkv the reference builds: image rows q|k|v = lin(x), text rows k|v = lin(x_text)."""
    B, L, _ = x.shape
    Lt = 0 if xt is None else xt.shape[1]
    qkv = np.zeros((B, L + Lt, 3 * C), np.float64)
    for bb in range(B):
        qkv[bb, :L] = O.linear(x[bb], w, b, acc=np.float64)
        if Lt:
            qkv[bb, L:, C:] = O.linear(xt[bb], wkv, bkv, acc=np.float64)
    return qkv


def run_projected(x, w, b, xt, wkv, bkv, q_w, k_w, lv, bias, h, wd, buffers=None, out_dtype=torch.float32):
    from nanosaur2_web_b200.blocks import dit_block_attention_projected
    from nanosaur2_web_b200.ops import rope2dTable
    L = h * wd
    Lt = 0 if xt is None else xt.shape[1]
    return dit_block_attention_projected(
        t(x, torch.bfloat16), w_qkv=t(w, torch.bfloat16), b_qkv=t(b), q_norm=t(q_w), k_norm=t(k_w),
        cs=rope2dTable(h, wd, D, DEV), x_text=None if xt is None else t(xt, torch.bfloat16),
        w_kv=None if wkv is None else t(wkv, torch.bfloat16), b_kv=None if bkv is None else t(bkv),
        kv_len=t(L + lv, torch.int32) if Lt else None, bias=None if bias is None else t(bias),
        buffers=buffers, out_dtype=out_dtype)


def check_device():
    from nanosaur2_web_b200.ops import check_device as chk
    chk(DEV)


@pytest.mark.parametrize("K", [1536, 200])
def test_projected_block_matches_oracle(K):
    """20 x 24 image tokens + 64 text slots (10-64 valid), batch 2; K = 200 leaves a partial last
    K slice that the TMA fills with zeros on both operands."""
    h, wd, Lt = 20, 24, 64
    L = h * wd
    x, w, b, xt, wkv, bkv, q_w, k_w, lv, bias = proj_inputs(5 + K, 2, L, Lt, K, (10, 64))
    out = run_projected(x, w, b, xt, wkv, bkv, q_w, k_w, lv, bias, h, wd)
    check_device()
    cos, sin = O.rope_2d(h, wd)
    want = O.joint_attention_batched(oracle_qkv(x, w, b, xt, wkv, bkv), L, Lt, L + lv, q_w, k_w, cos, sin, bias=bias,
                                     acc=np.float64)
    assert_close_bf16(out.cpu().numpy(), want, D, what=f"projected block K={K}")


def test_projection_buffers_and_padding():
    """q' tiles and packed k'|v' rows against the oracle's normalised, rotated q / k and v, and every
    padding row zero: q' rows past L, k'|v' rows past kv_len up to kv_rows."""
    from nanosaur2_web_b200.blocks import projection_buffers
    h, wd, Lt = 9, 15, 40
    L = h * wd
    x, w, b, xt, wkv, bkv, q_w, k_w, lv, bias = proj_inputs(77, 1, L, Lt, 1536, (17, 17))
    q_prime, kv_packed = projection_buffers(1, L, Lt, DEV)
    q_prime.fill_(0xFF)                       # NaN patterns: every byte the attention reads is written
    kv_packed.fill_(float("nan"))
    run_projected(x, w, b, xt, wkv, bkv, q_w, k_w, lv, bias, h, wd, buffers=(q_prime, kv_packed))
    check_device()
    qkv = oracle_qkv(x, w, b, xt, wkv, bkv)[0]
    cos, sin = O.rope_2d(h, wd)
    n = L + int(lv[0])
    qn = O.head_norm(qkv[:L, :C], q_w, H, D, cos, sin, acc=np.float64)
    kn = np.concatenate([O.head_norm(qkv[:L, C:2 * C], k_w, H, D, cos, sin, acc=np.float64),
                         O.head_norm(qkv[L:n, C:2 * C], k_w, H, D, acc=np.float64)])
    v = qkv[:n, 2 * C:]
    q_pad = (L + 255) // 256 * 256
    tiles = q_prime[:H * q_pad * D * 2].view(torch.bfloat16).view(H, q_pad, D).float().cpu().numpy()
    got_q = tiles[:, :L].transpose(1, 0, 2).reshape(L, C)
    assert_close_bf16(got_q, qn, D, what="q' tiles")
    assert not tiles[:, L:].any(), "q' padding rows must be zero"
    kv = kv_packed[0].float().cpu().numpy()
    assert_close_bf16(kv[:n, :C], kn, D, what="k' rows")
    assert_close_bf16(kv[:n, C:], v, D, what="v rows")
    assert not kv[n:].any(), "k'|v' rows past kv_len must be zero"


def test_projected_image_only_block():
    """An odd block (no text rows): Lk = L, the key padding up to kv_rows zero-filled."""
    h, wd = 7, 19
    L = h * wd
    x, w, b, _, _, _, q_w, k_w, _, _ = proj_inputs(91, 1, L, 0, 1536, (0, 0))
    out = run_projected(x, w, b, None, None, None, q_w, k_w, np.zeros(1, np.int32), None, h, wd)
    check_device()
    cos, sin = O.rope_2d(h, wd)
    want = O.joint_attention_batched(oracle_qkv(x, w, b, None, None, None), L, 0, np.array([L]), q_w, k_w, cos, sin,
                                     acc=np.float64)
    assert_close_bf16(out.cpu().numpy(), want, D, what="image-only block")


def test_projected_matches_fused_at_config2():
    """BASELINE config 2 shapes (52 x 76 image tokens, 256 text slots, batch 2): the projected path
    against the unfused one (qkv = x W^T + b by torch in fp32, rounded to bf16, then the fused
    prologue + attention).  Both are bf16 paths; they must agree within the bf16 bound."""
    from nanosaur2_web_b200.blocks import dit_block_attention
    from nanosaur2_web_b200.ops import rope2dTable
    h, wd, Lt = 76, 52, 256
    L = h * wd
    x, w, b, xt, wkv, bkv, q_w, k_w, lv, bias = proj_inputs(123, 2, L, Lt, 1536, (32, 256))
    got = run_projected(x, w, b, xt, wkv, bkv, q_w, k_w, lv, bias, h, wd, out_dtype=torch.bfloat16)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        img = t(x) @ t(w).T + t(b)
        txt = t(xt) @ t(wkv).T + t(bkv)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    qkv = torch.zeros((2, L + Lt, 3 * C), device=DEV)
    qkv[:, :L] = img
    qkv[:, L:, C:] = txt
    ref = dit_block_attention(qkv.to(torch.bfloat16), L=L, q_norm=t(q_w), k_norm=t(k_w), cs=rope2dTable(h, wd, D, DEV),
                              text_rows=Lt, kv_len=t(L + lv, torch.int32), bias=t(bias), out_dtype=torch.bfloat16)
    check_device()
    assert_close_bf16(got.float().cpu().numpy(), ref.float().cpu().numpy(), D, what="projected vs fused")


@pytest.mark.parametrize("world,local", [(2, True), (3, False)])
def test_sequence_sharded_projection(world, local):
    """Each emulated rank projects its own image rows (x holding only them, or all L rows) and every
    text row into one shared kv_packed, then runs its queries: the stitched output matches the
    one-GPU projected step to the bf16 rounding of P (a short last wave splits units differently)
    and the oracle within the bf16 bound.  A key row no rank writes would poison every query."""
    from nanosaur2_web_b200.ops import rope2dTable
    from nanosaur2_web_b200.seqshard import SeqShardedJointAttention
    h, wd, Lt = 12, 20, 64
    L = h * wd
    B = 2
    x, w, b, xt, wkv, bkv, q_w, k_w, lv, bias = proj_inputs(321 + world, B, L, Lt, 1536, (10, 64))
    full = run_projected(x, w, b, xt, wkv, bkv, q_w, k_w, lv, bias, h, wd).cpu().numpy()
    cs = rope2dTable(h, wd, D, DEV)
    xd, xtd = t(x, torch.bfloat16), t(xt, torch.bfloat16)
    wqd, wkvd, bd, bkvd = t(w, torch.bfloat16), t(wkv, torch.bfloat16), t(b), t(bkv)
    kv_len, bias_d = t(L + lv, torch.int32), t(bias)
    ranks, shared = [], None
    for r in range(world):
        m = SeqShardedJointAttention(B=B, L=L, text_rows=Lt, world=world, rank=r, device=DEV, local_qkv=local,
                                     kv_packed=shared, out_dtype=torch.float32, mode="nccl")
        shared = m.kv_packed
        ranks.append(m)
    shared.fill_(float("nan"))
    for m in ranks:
        src = xd[:, m.q_begin:m.q_begin + m.q_count].contiguous() if local else xd
        for bb in range(B):
            m.projection(bb, src, w_qkv=wqd, b_qkv=bd, q_norm=t(q_w), k_norm=t(k_w), cs=cs, kv_len=kv_len,
                         x_text=xtd, w_kv=wkvd, b_kv=bkvd)
    out = torch.full((B, L, C), float("nan"), device=DEV)
    for m in ranks:
        view = out[:, m.q_begin:m.q_begin + m.q_count]
        for bb in range(B):
            m.attention(bb, kv_len=kv_len, bias=bias_d, out=view)
    check_device()
    got = out.cpu().numpy()
    np.testing.assert_allclose(got, full, atol=2e-3, rtol=0)
    cos, sin = O.rope_2d(h, wd)
    want = O.joint_attention_batched(oracle_qkv(x, w, b, xt, wkv, bkv), L, Lt, L + lv, q_w, k_w, cos, sin, bias=bias,
                                     acc=np.float64)
    assert_close_bf16(got, want, D, what=f"sequence-sharded projection x{world}")


@pytest.mark.parametrize("theta,window,L", [(1e6, 0, 300), (1e4, 100, 300), (1e4, 512, 1024)])
def test_gemma_projected_layer(theta, window, L):
    """A Gemma3 layer's attention from its normalised input rows (K = 640): the te.qkv linear with the
    q/k RMSNorm and the 1D RoPE in the GEMM epilogue (one head of 256 per tile), then causal GQA 4/1
    attention with an optional sliding window over the prepared tiles, against the oracle's
    linear + gemma_attention (tools/reference.py:186-194)."""
    from nanosaur2_web_b200.blocks import gemma_layer_attention_projected
    from nanosaur2_web_b200.ops import ropeTable
    B, K, GD = 2, 640, 256
    rng = np.random.default_rng(L + window)
    x = bf16_round(rng.standard_normal((B, L, K), dtype=np.float32))
    w = bf16_round(rng.standard_normal((6 * GD, K), dtype=np.float32) / np.sqrt(K))
    q_w = (1.0 + 0.2 * rng.standard_normal(GD)).astype(np.float32)
    k_w = (1.0 + 0.2 * rng.standard_normal(GD)).astype(np.float32)
    out = gemma_layer_attention_projected(t(x, torch.bfloat16), w_qkv=t(w, torch.bfloat16), q_norm=t(q_w),
                                          k_norm=t(k_w), cs=ropeTable(L, GD, theta, DEV), window=window,
                                          out_dtype=torch.float32)
    check_device()
    got = out.cpu().numpy()
    for bb in range(B):
        qkv = O.linear(x[bb], w, acc=np.float64)
        want = O.gemma_attention(qkv[:, :4 * GD], qkv[:, 4 * GD:5 * GD], qkv[:, 5 * GD:], q_w, k_w, theta, window,
                                 acc=np.float64)
        assert_close_bf16(got[bb], want, GD, what=f"gemma projected theta={theta} window={window} b={bb}")


def test_gemma_projected_unaligned_sin_block():
    """Head dim 256 with a RoPE table whose sin block does not start on a row boundary (sinOff =
    L*128 + 4): the epilogue cannot map the table as rows and reads each row's cos / sin directly.
    Same results as the oracle (and as the staged path of the test above)."""
    from nanosaur2_web_b200.blocks import gemma_layer_attention_projected
    from nanosaur2_web_b200.ops import RopeTable
    B, L, K, GD, theta = 1, 200, 640, 256, 1e4
    rng = np.random.default_rng(77)
    x = bf16_round(rng.standard_normal((B, L, K), dtype=np.float32))
    w = bf16_round(rng.standard_normal((6 * GD, K), dtype=np.float32) / np.sqrt(K))
    q_w = (1.0 + 0.2 * rng.standard_normal(GD)).astype(np.float32)
    k_w = (1.0 + 0.2 * rng.standard_normal(GD)).astype(np.float32)
    cos, sin = O.rope_1d(L, theta, GD)
    buf = np.zeros(L * GD + 4, np.float32)
    buf[:L * GD // 2] = cos.reshape(-1)
    buf[L * GD // 2 + 4:] = sin.reshape(-1)
    cs = RopeTable(t(buf), L * GD // 2 + 4, L, GD)
    out = gemma_layer_attention_projected(t(x, torch.bfloat16), w_qkv=t(w, torch.bfloat16), q_norm=t(q_w),
                                          k_norm=t(k_w), cs=cs, out_dtype=torch.float32)
    check_device()
    qkv = O.linear(x[0], w, acc=np.float64)
    want = O.gemma_attention(qkv[:, :4 * GD], qkv[:, 4 * GD:5 * GD], qkv[:, 5 * GD:], q_w, k_w, theta, acc=np.float64)
    assert_close_bf16(out[0].cpu().numpy(), want, GD, what="gemma projected, sin block off the row grid")


def test_projected_block_int8_convrot_with_loras():
    """The projection with int8 ConvRot weights (given as their exact bf16 values, ops.expand_i8, with
    the row scales in the epilogue: app/gpu/gemm.js:159) and LoRA side paths on both weights: on
    w_qkv a full-width entry and one on the q slice only, on w_kv one full-width entry (app/lora.js:149
    off / n).  The inputs stand for rotated rows (the rotation itself is tested with nsa_rotate).  The
    oracle builds q|k|v with the int8 GEMM plus the side paths (the packed bf16 roundings emulated)
    and runs the DiT block's head norms, RoPE and joint attention on them."""
    from nanosaur2_web_b200.blocks import dit_block_attention_projected
    from nanosaur2_web_b200.ops import expand_i8, lora_pack, rope2dTable
    from tests._helpers import lora_oracle
    rng = np.random.default_rng(123)
    h, wd, Lt, B, K = 12, 20, 32, 2, 512
    L = h * wd
    x = bf16_round(rng.standard_normal((B, L, K), dtype=np.float32))
    xt = bf16_round(rng.standard_normal((B, Lt, K), dtype=np.float32))
    q8 = rng.integers(-128, 128, size=(3 * C, K), dtype=np.int8)
    kv8 = rng.integers(-128, 128, size=(2 * C, K), dtype=np.int8)
    sq = (rng.uniform(0.5, 2.0, 3 * C) / (127 * np.sqrt(K / 3))).astype(np.float32)
    skv = (rng.uniform(0.5, 2.0, 2 * C) / (127 * np.sqrt(K / 3))).astype(np.float32)
    b = (0.1 * rng.standard_normal(3 * C)).astype(np.float32)
    bkv = (0.1 * rng.standard_normal(2 * C)).astype(np.float32)
    q_w = (1.0 + 0.2 * rng.standard_normal(D)).astype(np.float32)
    k_w = (1.0 + 0.2 * rng.standard_normal(D)).astype(np.float32)
    lv = np.array([20, 32], np.int32)
    bias = np.log(rng.choice(np.array([0.7, 1.0, 1.3], np.float32), size=(B, Lt))).astype(np.float32)
    ent_q = [dict(A=rng.standard_normal((16, K), dtype=np.float32) / 30, B=rng.standard_normal((3 * C, 16), dtype=np.float32) / 4,
                  scale=0.6, off=0, n=3 * C),
             dict(A=rng.standard_normal((8, K), dtype=np.float32) / 30, B=rng.standard_normal((C, 8), dtype=np.float32) / 4,
                  scale=-0.4, off=0, n=C)]
    ent_kv = [dict(A=rng.standard_normal((32, K), dtype=np.float32) / 30, B=rng.standard_normal((2 * C, 32), dtype=np.float32) / 4,
                   scale=0.5, off=0, n=2 * C)]
    sq_t, skv_t = t(sq), t(skv)
    pk_q = lora_pack([dict(e, A=t(e["A"]), B=t(e["B"])) for e in ent_q], 3 * C, K, w_scale=sq_t)
    pk_kv = lora_pack([dict(e, A=t(e["A"]), B=t(e["B"])) for e in ent_kv], 2 * C, K, w_scale=skv_t)
    out = dit_block_attention_projected(
        t(x, torch.bfloat16), w_qkv=expand_i8(t(q8, torch.int8)), b_qkv=t(b), q_norm=t(q_w), k_norm=t(k_w),
        cs=rope2dTable(h, wd, D, DEV), x_text=t(xt, torch.bfloat16), w_kv=expand_i8(t(kv8, torch.int8)), b_kv=t(bkv),
        kv_len=t(L + lv, torch.int32), bias=t(bias), out_dtype=torch.float32, w_qkv_scale=sq_t, w_kv_scale=skv_t,
        lora_qkv=pk_q, lora_kv=pk_kv)
    check_device()
    qkv = np.zeros((B, L + Lt, 3 * C), np.float64)
    for bb in range(B):
        qkv[bb, :L] = lora_oracle(x[bb], q8, sq, b, ent_q, 3 * C)[0]
        qkv[bb, L:, C:] = lora_oracle(xt[bb], kv8, skv, bkv, ent_kv, 2 * C)[0]
    cos, sin = O.rope_2d(h, wd)
    want = O.joint_attention_batched(qkv, L, Lt, L + lv, q_w, k_w, cos, sin, bias=bias, acc=np.float64)
    assert_close_bf16(out.cpu().numpy(), want, D, what="int8 ConvRot projection with LoRAs")
    # the side paths matter at this size: without them the result is far outside the bound
    qkv0 = np.zeros_like(qkv)
    for bb in range(B):
        qkv0[bb, :L] = O.linear_int8(x[bb], q8, sq, b, acc=np.float64)
        qkv0[bb, L:, C:] = O.linear_int8(xt[bb], kv8, skv, bkv, acc=np.float64)
    base = O.joint_attention_batched(qkv0, L, Lt, L + lv, q_w, k_w, cos, sin, bias=bias, acc=np.float64)
    assert np.abs(base - want).max() > 10 * np.abs(out.cpu().numpy() - want).max()


def test_projection_rejects_scales_at_head_dim_256():
    from nanosaur2_web_b200 import _lib
    from nanosaur2_web_b200.blocks import gemma_projection_buffers  # noqa: F401  (module import only)
    d = _lib.FusedDesc()
    d.B, d.Lq, d.Lk, d.Hq, d.Hkv, d.D = 1, 128, 128, 4, 1, 256
    d.in_dtype = d.out_dtype = _lib.NSA_BF16
    d.causal = 1
    d.b_begin, d.b_count = 0, 1
    s = _lib.SeqShard(0, 128, 0, 0)
    p = _lib.ProjDesc()
    x = torch.zeros((128, 640), dtype=torch.bfloat16, device=DEV)
    w = torch.zeros((6 * 256, 640), dtype=torch.bfloat16, device=DEV)
    sc = torch.ones(6 * 256, device=DEV)
    p.K, p.x, p.ldx, p.x_bstride, p.x_rows, p.w_qkv = 640, x.data_ptr(), 640, 0, 128, w.data_ptr()
    p.w_qkv_scale = sc.data_ptr()
    qn = torch.ones(256, device=DEV)
    buf = torch.zeros(1 << 22, dtype=torch.uint8, device=DEV)
    st = _lib.lib().nsa_seq_shard_projection(ctypes_ref(d), ctypes_ref(s), ctypes_ref(p), qn.data_ptr(), qn.data_ptr(),
                                             None, None, buf.data_ptr(), buf.data_ptr(), None)
    assert st == _lib.NSA_ERR_UNSUPPORTED


def ctypes_ref(x):
    import ctypes
    return ctypes.byref(x)
