"""The VAE decoder's single-head attention at head dim C = 512 (app/models/vae.js:77-88;
tools/reference.py:352-357) through the C ABI, against the CPU oracle (oracle/attention_oracle.py,
whose vae_attention is pinned by the reference's own VAE.attn output in tests/golden/vae_attention.npz).

  * the golden VAE block itself: group norm and the 1x1 convolutions on the host, the attention on the
    GPU, the projection and residual on the host, compared with the reference's output;
  * head dim 512 at the 832x1216 latent resolution (104 x 152 = 15808 pixels), fp32 inputs as the
    reference's qkv linear writes them, three 128-row query blocks against all keys;
  * ragged pixel counts (fewer than one query tile, not a multiple of 128), bf16 and fp32 inputs and
    outputs, every row.
Tolerance of the bf16 path: max-abs <= 2e-2 and per-head cosine >= 0.9999.
"""

import numpy as np
import pytest
import torch

from oracle import attention_oracle as O
from tests._helpers import assert_close_bf16

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


def test_golden_vae_block_attention_on_gpu(golden):
    """VAE.attn of the reference (C = 64 fixture): only the attention runs on the GPU."""
    from nanosaur2_web_b200.blocks import vae_attention
    from nanosaur2_web_b200.ops import check_device
    g = golden("vae_attention")
    x = g["x"]
    C = x.shape[0]
    n = O.group_norm(x, 32, g["gn_w"], g["gn_b"]).reshape(C, -1).T                # [hw, C]
    qkv = np.concatenate([O.linear(n, g["w_q"], g["b_q"]), O.linear(n, g["w_k"], g["b_k"]),
                          O.linear(n, g["w_v"], g["b_v"])], axis=1).astype(np.float32)
    a = vae_attention(t(qkv), C=C, out_dtype=torch.float32)
    check_device(DEV)
    y = x + O.linear(a.cpu().numpy(), g["w_o"], g["b_o"]).T.reshape(x.shape)
    np.testing.assert_allclose(y, g["y"], atol=2e-2, rtol=0)
    want = O.attention(qkv[:, :C], qkv[:, C:2 * C], qkv[:, 2 * C:], 1, C, acc=np.float64)
    assert_close_bf16(a.cpu().numpy(), want, C, what="VAE block attention")


def _qkv(seed, hw, C=512):
    rng = np.random.default_rng(seed)
    return rng.standard_normal((hw, 3 * C), dtype=np.float32)


def test_vae_d512_latent_resolution():
    """104 x 152 latent pixels (the 832x1216 image), C = 512, fp32 qkv rows."""
    from nanosaur2_web_b200.blocks import vae_attention
    from nanosaur2_web_b200.ops import check_device
    hw, C = 104 * 152, 512
    qkv = _qkv(512, hw)
    got = vae_attention(t(qkv), C=C, out_dtype=torch.float32)
    check_device(DEV)
    rows = np.concatenate([np.arange(0, 128), np.arange(7936, 8064), np.arange(hw - 128, hw)])
    want = O.attention(qkv[rows, :C], qkv[:, C:2 * C], qkv[:, 2 * C:], 1, C, acc=np.float64)
    assert_close_bf16(got.cpu().numpy()[rows], want, C, what="VAE D=512 at 104x152")


@pytest.mark.parametrize("hw,in_dtype,out_dtype", [(7 * 9, torch.float32, torch.float32),
                                                   (20 * 30, torch.bfloat16, torch.bfloat16),
                                                   (300, torch.float32, torch.bfloat16)])
def test_vae_d512_ragged(hw, in_dtype, out_dtype):
    from nanosaur2_web_b200.blocks import vae_attention
    from nanosaur2_web_b200.ops import check_device
    C = 512
    qkv = _qkv(hw, hw)
    if in_dtype == torch.bfloat16:
        qkv = torch.from_numpy(qkv).to(torch.bfloat16).float().numpy()
    got = vae_attention(t(qkv, in_dtype), C=C, out_dtype=out_dtype)
    check_device(DEV)
    want = O.attention(qkv[:, :C], qkv[:, C:2 * C], qkv[:, 2 * C:], 1, C, acc=np.float64)
    assert_close_bf16(got.float().cpu().numpy(), want, C, what=f"VAE D=512 hw={hw}")


def test_d512_multi_head_causal_and_padding():
    """The generic op at head dim 512 beyond the VAE's use: two heads sharing one kv head, a causal
    mask, and per-batch valid key counts."""
    from nanosaur2_web_b200.ops import attention, check_device
    rng = np.random.default_rng(77)
    B, L, D = 2, 333, 512
    q = rng.standard_normal((B, L, 2 * D), dtype=np.float32)
    kv = rng.standard_normal((B, L, 2 * D), dtype=np.float32)
    out = attention(q=t(q), k=t(kv), v=t(kv), Lq=L, Lk=L, H=2, D=D, ldq=2 * D, ldk=2 * D, ldv=2 * D, kOff=0,
                    vOff=D, group=2, causal=True)
    check_device(DEV)
    got = out.cpu().numpy()
    for b in range(B):
        want = O.attention(q[b], kv[b, :, :D], kv[b, :, D:], 2, D, group=2, causal=True, acc=np.float64)
        assert_close_bf16(got[b], want, D, what=f"D=512 causal b={b}")
    lens = np.array([200, 333], np.int32)
    out = attention(q=t(q), k=t(kv), v=t(kv), Lq=L, Lk=L, H=2, D=D, ldq=2 * D, ldk=2 * D, ldv=2 * D, kOff=0,
                    vOff=D, group=2, kv_len=t(lens, torch.int32))
    check_device(DEV)
    got = out.cpu().numpy()
    for b in range(B):
        n = int(lens[b])
        want = O.attention(q[b], kv[b, :n, :D], kv[b, :n, D:], 2, D, group=2, acc=np.float64)
        assert_close_bf16(got[b], want, D, what=f"D=512 kv_len b={b}")
