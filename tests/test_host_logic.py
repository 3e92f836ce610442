"""Host-side logic that needs no GPU: work partitioning, the text-bias preparation, the Gemma layer
schedule and the bench's algorithmic FLOP count."""

import math

import numpy as np
import pytest

from nanosaur2_web_b200 import blocks, sharding
from oracle import attention_oracle as O


@pytest.mark.parametrize("B,H", [(2, 16), (8, 16), (16, 4), (1, 16), (4, 16)])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shards_cover_units_once(B, H, world):
    seen = []
    for rank in range(world):
        for b0, bc, h0, hc in sharding.shard_batch_heads(B, H, world, rank):
            assert bc >= 1 and hc >= 1 and h0 + hc <= H and b0 + bc <= B
            assert bc == 1 or (h0 == 0 and hc == H)
            seen += [(b, h) for b in range(b0, b0 + bc) for h in range(h0, h0 + hc)]
    assert sorted(seen) == [(b, h) for b in range(B) for h in range(H)]


def test_split_range_balanced():
    sizes = [sharding.split_range(10, 4, r) for r in range(4)]
    assert sizes == [(0, 3), (3, 6), (6, 8), (8, 10)]
    with pytest.raises(ValueError):
        sharding.split_range(10, 0, 0)


def test_prepare_text_bias_matches_reference_bias():
    w = [1.0, 1.3, 0.0, 0.7, -1.0, 1.0]
    keep, bias = blocks.prepare_text_bias(w)
    assert keep == [0, 1, 3, 5]
    ref = O.text_key_bias(w)
    np.testing.assert_allclose(bias, ref[keep], rtol=1e-6)
    assert blocks.prepare_text_bias([1.0, 1.0, 0.0]) == ([0, 1], None)


def test_gemma_schedule():
    assert [blocks.gemma_rope_theta(i) for i in range(18)] == [O.gemma_rope_theta(i) for i in range(18)]
    assert sum(blocks.gemma_rope_theta(i) == 1e6 for i in range(18)) == 3


def test_bench_flop_counts():
    import bench
    assert math.isclose(bench.joint_flops(2, 3952, [256, 256]), 204.35e9, rel_tol=1e-3)
    assert math.isclose(bench.joint_flops(1, 2304, [128]), 34.43e9, rel_tol=1e-3)
    g, l = bench.gemma_pairs(1024, 0), bench.gemma_pairs(1024, 512)
    assert g == 524800 and l == 393472


def test_gemma_encoder_flops_brute_force():
    """Configs 8 and 9: the FLOP count against an explicit count of the masked (query, key) pairs and of
    every linear's multiply-adds, on a short sequence."""
    import bench
    L, window, layers = 40, 16, 7
    pairs = []
    for i in range(layers):
        glob = (i + 1) % 6 == 0
        pairs.append(sum(1 for q in range(L) for k in range(L) if k <= q and (glob or q - window < k)))
    attn = sum(4 * 4 * p * 256 for p in pairs)
    lin_attn = layers * 2 * L * 640 * (1536 + 1024)
    lin_mlp = layers * 2 * L * (640 * 2 * 2048 + 2048 * 640)
    assert bench.gemma_encoder_flops(L, layers, window) == attn + lin_attn
    assert bench.gemma_encoder_flops(L, layers, window, whole=True) == attn + lin_attn + lin_mlp


@pytest.mark.parametrize("L,world", [(16384, 2), (16384, 4), (16384, 8), (3952, 4), (512, 1)])
def test_seq_shard_rows_tile_the_image_rows(L, world):
    from nanosaur2_web_b200.seqshard import seq_shard_rows
    rows = [seq_shard_rows(L, world, r) for r in range(world)]
    assert rows[0][0] == 0 and all(c == L // world for _, c in rows)
    assert all(rows[i][0] + rows[i][1] == rows[i + 1][0] for i in range(world - 1))
    assert rows[-1][0] + rows[-1][1] == L


def test_seq_shard_rows_rejects_uneven_split():
    from nanosaur2_web_b200.seqshard import seq_shard_rows
    with pytest.raises(ValueError):
        seq_shard_rows(3952, 3, 0)
    with pytest.raises(ValueError):
        seq_shard_rows(64, 2, 2)


def test_gather_views_are_in_place_chunks():
    import torch

    from nanosaur2_web_b200.seqshard import gather_views, seq_shard_rows
    L, world, kv_rows, ld = 64, 4, 96, 12
    kv = torch.zeros(2, kv_rows, ld)
    for rank in range(world):
        q0, qn = seq_shard_rows(L, world, rank)
        out, inp = gather_views(kv, 1, L, q0, qn)
        assert out.is_contiguous() and inp.is_contiguous()
        assert out.numel() == world * inp.numel()
        # ncclAllGather's in-place form: sendbuff = recvbuff + rank * sendcount
        assert inp.data_ptr() == out.data_ptr() + rank * inp.numel() * inp.element_size()
        assert out.data_ptr() == kv.data_ptr() + kv_rows * ld * kv.element_size()


def test_rmsnorm_and_sublayer_host_checks():
    """Argument errors of ops.rmsnorm and blocks.gemma_attention_sublayer raise NsaError before any
    device work, as the reference's operators throw synchronously."""
    import torch

    from nanosaur2_web_b200.ops import NsaError, rmsnorm
    x = torch.zeros(2, 8, 64)
    with pytest.raises(NsaError):
        rmsnorm(x, torch.ones(64))                                    # host tensors
    kw = dict(in_norm=None, w_qkv=None, q_norm=None, k_norm=None, post_norm=None, cs=None)
    with pytest.raises(NsaError):
        blocks.gemma_attention_sublayer(x.double(), w_o=torch.zeros(64, 1024), **kw)   # fp32 stream only
    with pytest.raises(NsaError):
        blocks.gemma_attention_sublayer(x[:, :, :32], w_o=torch.zeros(32, 1024), **kw)  # not contiguous
    with pytest.raises(NsaError):
        blocks.gemma_attention_sublayer(x, w_o=torch.zeros(64, 512), **kw)            # w_o [hidden, 1024]
