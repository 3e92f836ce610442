"""torchrun worker of the multi-GPU sequence-shard test (tests/test_gpu_multi.py).

Every rank builds the same seeded joint-attention inputs, keeps its own image rows plus the text rows
(the local layout), and runs SeqShardedJointAttention, which gathers the k'|v' rows over NCCL.  Rank 0
stitches the ranks' output rows together and compares them with the single-GPU fused call (to the
size of P's bf16 rounding) and with the CPU oracle on a few heads; it writes the outcome as JSON to
argv[1].
"""

import datetime
import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def main():
    out_path = sys.argv[1]
    mode = sys.argv[2] if len(sys.argv) > 2 else "nccl"
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ["LOCAL_RANK"]))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        from nanosaur2_web_b200.blocks import dit_block_attention
        from nanosaur2_web_b200.ops import check_device, rope2dTable
        from nanosaur2_web_b200.seqshard import SeqShardedJointAttention, local_rows
        from oracle import attention_oracle as O
        from tests._helpers import joint_inputs, per_head_cosine

        h, w, Lt, B = 32, 32, 128, 2
        L = h * w
        qkv, q_w, k_w, lv, bias = joint_inputs(77, B, h, w, Lt, (10, 128))
        x = torch.from_numpy(qkv).to(dev, torch.bfloat16)
        qn, kn = torch.from_numpy(q_w).to(dev), torch.from_numpy(k_w).to(dev)
        kv_len = torch.from_numpy((L + lv).astype(np.int32)).to(dev)
        kb = torch.from_numpy(bias).to(dev)
        cs = rope2dTable(h, w, 96, dev)
        m = SeqShardedJointAttention(B=B, L=L, text_rows=Lt, world=world, rank=rank, device=dev, mode=mode)
        src = local_rows(x, L, m.q_begin, m.q_count)
        for _ in range(3):   # reuses the gather buffers across calls
            out = m(src, q_norm=qn, k_norm=kn, cs=cs, kv_len=kv_len, bias=kb)
        torch.cuda.synchronize()
        check_device(dev)
        timing = m.timing()
        parts = [torch.empty_like(out) for _ in range(world)]
        dist.all_gather(parts, out.contiguous())
        if rank == 0:
            full = torch.cat(parts, dim=1)
            ref = dit_block_attention(x, L=L, text_rows=Lt, q_norm=qn, k_norm=kn, cs=cs, kv_len=kv_len, bias=kb)
            torch.cuda.synchronize()
            heads = [1, 14]
            cos, sin = O.rope_2d(h, w)
            want = O.joint_attention_batched(qkv, L, Lt, L + lv, q_w, k_w, cos, sin, bias=bias, acc=np.float64,
                                             heads=heads)
            cols = np.concatenate([np.arange(hh * 96, (hh + 1) * 96) for hh in heads])
            got = full.float().cpu().numpy()[..., cols]
            # equal to the size of P's bf16 rounding: a split tail rounds each half against its own max
            diff = float((full.float() - ref.float()).abs().max())
            res = {"world": world, "mode": m.mode, "equal_to_fused": diff <= 2e-3, "max_abs_vs_fused": diff,
                   "max_abs_vs_oracle": float(np.abs(got - want[..., cols]).max()),
                   "min_cos_vs_oracle": float(per_head_cosine(got, want[..., cols], 96).min()),
                   "call_ms": timing.call_ms, "gather_ms": timing.gather_ms}
            with open(out_path, "w") as f:
                json.dump(res, f)
        dist.barrier()
        m.close()
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
