"""Sequence-sharded joint attention (the 16384-token config's path) on one GPU.

The ranks' prologues (nsa_seq_shard_prologue) all write into one shared kv_packed buffer, which is
the state the per-element all-gather leaves on every rank; each rank's attention
(nsa_seq_shard_attention) then runs over it.  The stitched output must match the CPU oracle within
the bf16 tolerance (max-abs <= 2e-2, per-head cosine >= 0.9999), and the unsharded fused call to
the size of the bf16 rounding of P (max-abs <= 2e-3): a launch whose last wave is short splits
those units' key range over two CTAs, each half rounds its probabilities against its own running
max, and the sharded and unsharded launches differ in that choice.  Where neither splits (config
5's shapes) the two are identical.  The NCCL gather itself is covered by the two-GPU test and, on
CPU, by the gloo test.
"""

import numpy as np
import pytest
import torch

from oracle import attention_oracle as O
from tests._helpers import assert_close_bf16, joint_inputs

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


def _inputs(seed, B, h, w, Lt, lv):
    qkv, q_w, k_w, lvs, bias = joint_inputs(seed, B, h, w, Lt, lv)
    L = h * w
    return dict(qkv=t(qkv, torch.bfloat16), q_w=t(q_w), k_w=t(k_w), kv_len=t(L + lvs, torch.int32), bias=t(bias),
                np=(qkv, q_w, k_w, lvs, bias))


def _seq_sharded(x, h, w, Lt, world, local_qkv, out_dtype=torch.float32):
    from nanosaur2_web_b200.ops import rope2dTable
    from nanosaur2_web_b200.seqshard import SeqShardedJointAttention, local_rows
    L = h * w
    B = x["qkv"].shape[0]
    cs = rope2dTable(h, w, 96, DEV)
    ranks, shared = [], None
    for r in range(world):
        # mode "nccl" maps no peer buffers: the emulated ranks share one kv_packed instead
        m = SeqShardedJointAttention(B=B, L=L, text_rows=Lt, world=world, rank=r, device=DEV, local_qkv=local_qkv,
                                     kv_packed=shared, out_dtype=out_dtype, mode="nccl")
        shared = m.kv_packed
        ranks.append(m)
    shared.fill_(float("nan"))   # a key row no prologue writes would poison every query
    for m in ranks:
        src = local_rows(x["qkv"], L, m.q_begin, m.q_count) if local_qkv else x["qkv"]
        for b in range(B):
            m.prologue(b, src, q_norm=x["q_w"], k_norm=x["k_w"], cs=cs, kv_len=x["kv_len"])
    out = torch.full((B, L, 1536), float("nan"), dtype=out_dtype, device=DEV)
    for m in ranks:
        view = out[:, m.q_begin:m.q_begin + m.q_count]
        for b in range(B):
            m.attention(b, kv_len=x["kv_len"], bias=x["bias"], out=view)
    return out


def _fused(x, h, w, Lt, out_dtype=torch.float32):
    from nanosaur2_web_b200.blocks import dit_block_attention
    from nanosaur2_web_b200.ops import rope2dTable
    L = h * w
    return dit_block_attention(x["qkv"], L=L, text_rows=Lt, q_norm=x["q_w"], k_norm=x["k_w"],
                               cs=rope2dTable(h, w, 96, DEV), kv_len=x["kv_len"], bias=x["bias"], out_dtype=out_dtype)


@pytest.mark.parametrize("hw,Lt,lv,world,local_qkv", [
    ((16, 32), 64, (10, 64), 4, True),     # 128 query rows per rank: half a query tile
    ((16, 32), 64, (0, 0), 2, False),      # no valid text, full-length qkv
    ((10, 13), 40, (1, 40), 2, True),      # 65 rows per rank: odd row offsets and ragged tiles
    ((24, 24), 300, (1, 300), 3, True),    # text longer than one key tile, three ranks
])
def test_seq_shard_matches_fused_and_oracle(hw, Lt, lv, world, local_qkv):
    from nanosaur2_web_b200.ops import check_device
    h, w = hw
    L = h * w
    x = _inputs(500 + L + world, 2, h, w, Lt, lv)
    got = _seq_sharded(x, h, w, Lt, world, local_qkv)
    full = _fused(x, h, w, Lt)
    check_device()
    got_np, full_np = got.cpu().numpy(), full.cpu().numpy()
    np.testing.assert_allclose(got_np, full_np, rtol=0, atol=2e-3)
    qkv, q_w, k_w, lvs, bias = x["np"]
    cos, sin = O.rope_2d(h, w)
    heads = [0, 7, 15]
    want = O.joint_attention_batched(qkv, L, Lt, L + lvs, q_w, k_w, cos, sin, bias=bias, acc=np.float64, heads=heads)
    cols = np.concatenate([np.arange(hh * 96, (hh + 1) * 96) for hh in heads])
    assert_close_bf16(got_np[..., cols], want[..., cols], 96, what=f"seq shard {hw} x{world}")


def test_seq_shard_config5_size_matches_fused_and_oracle():
    """Config 5's shapes (128x128 = 16384 image rows + 256 text slots, batch 2) split over 8 emulated
    ranks: identical to the single fused call, and both within the bf16 tolerance of the fp64 oracle
    for all 16 heads on three 128-row query blocks (the first, one in the middle, the last), each
    against all 16384 + Lv keys (up to 149 key tiles of 112 per query block)."""
    from nanosaur2_web_b200.ops import check_device
    h = w = 128
    L, Lt = h * w, 256
    x = _inputs(555, 2, h, w, Lt, (32, 256))
    got = _seq_sharded(x, h, w, Lt, 8, True, out_dtype=torch.bfloat16)
    full = _fused(x, h, w, Lt, out_dtype=torch.bfloat16)
    check_device()
    assert torch.isfinite(got).all()
    assert torch.equal(got, full)
    qkv, q_w, k_w, lvs, bias = x["np"]
    rows = np.concatenate([np.arange(0, 128), np.arange(8192, 8320), np.arange(L - 128, L)])
    cos, sin = O.rope_2d(h, w)
    want = O.joint_attention_batched(qkv, L, Lt, L + lvs, q_w, k_w, cos, sin, bias=bias, acc=np.float64, rows=rows)
    got_np = got.float().cpu().numpy()
    for b in range(2):
        assert_close_bf16(got_np[b, rows], want[b], 96, what=f"config 5, b={b}, 16 heads")
