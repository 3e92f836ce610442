"""Parity at the benchmark configs' own shapes, every head, against the fp64 CPU oracle.

The oracle (oracle/attention_oracle.py, pinned by tests/test_oracle_golden.py) computes every head
over a subset of query rows: blocks at the start, the middle and the ragged end of the sequence,
each against all keys, so the CPU cost stays at a few seconds while every key tile, the text
bias/padding tiles and the last partial query tile of the GPU launch are covered.  Tolerance of the
bf16 path: max-abs <= 2e-2 and per-head cosine >= 0.9999 (tests/_helpers.py).

  * config 2: 52x76 = 3952 image rows + 256 text slots (valid ~U[32, 256]), batch 2, bf16;
  * config 3: the image-only blocks of the 18-block pass, 3952 rows, no text, batch 8.

Config 5 (16384 + 256) is checked the same way in tests/test_gpu_seqshard.py, sequence-sharded.
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


def row_blocks(L, block=128):
    """Query rows of three blocks: the first, one in the middle and the last (ragged) one."""
    mid = (L // 2) // block * block
    last = (L - 1) // block * block
    return np.unique(np.concatenate([np.arange(0, block), np.arange(mid, mid + block), np.arange(last, L)]))


def _run(qkv, L, Lt, q_w, k_w, lv, bias, h, w, out_dtype):
    from nanosaur2_web_b200.blocks import dit_block_attention
    from nanosaur2_web_b200.ops import check_device, rope2dTable
    cs = rope2dTable(h, w, 96, DEV)
    out = dit_block_attention(t(qkv, torch.bfloat16), L=L, text_rows=Lt, q_norm=t(q_w), k_norm=t(k_w), cs=cs,
                              kv_len=t((L + lv).astype(np.int32), torch.int32) if Lt else None,
                              bias=t(bias) if Lt else None, out_dtype=out_dtype)
    check_device(DEV)
    return out.float().cpu().numpy()


@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32])
def test_config2_every_head(out_dtype):
    """Config 2 (B=2, 3952 + 256, 16 x 96): all 16 heads on three row blocks per batch element."""
    h, w, Lt = 76, 52, 256
    L = h * w
    qkv, q_w, k_w, lv, bias = joint_inputs(2202, 2, h, w, Lt, (32, 256))
    got = _run(qkv, L, Lt, q_w, k_w, lv, bias, h, w, out_dtype)
    rows = row_blocks(L)
    cos, sin = O.rope_2d(h, w)
    want = O.joint_attention_batched(qkv, L, Lt, L + lv, q_w, k_w, cos, sin, bias=bias, acc=np.float64, rows=rows)
    for b in range(2):
        assert_close_bf16(got[b, rows], want[b], 96, what=f"config 2, b={b}, 16 heads")


def test_config3_image_only_every_head():
    """Config 3's image-only blocks: 3952 image rows, no text keys, batch 8 (eight seeds)."""
    h, w = 76, 52
    L = h * w
    qkv, q_w, k_w, lv, bias = joint_inputs(3303, 8, h, w, 0, (0, 0))
    got = _run(qkv, L, 0, q_w, k_w, lv, bias, h, w, torch.bfloat16)
    rows = row_blocks(L)
    cos, sin = O.rope_2d(h, w)
    want = O.joint_attention_batched(qkv, L, 0, np.full(8, L), q_w, k_w, cos, sin, acc=np.float64, rows=rows)
    for b in range(8):
        assert_close_bf16(got[b, rows], want[b], 96, what=f"config 3 image-only, b={b}")
