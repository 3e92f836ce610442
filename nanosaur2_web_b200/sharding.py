"""Work partitioning across the GPUs of one box (one process per GPU).

The attention hot path shards without any data exchange: (batch x head) units are independent, so
each rank takes a contiguous range of units and writes its own slice of the output (no collective on
the data path).  The only collective is the timing reduction (max over ranks) of the benchmark.
"""

from __future__ import annotations

from typing import List, Tuple


def split_range(n: int, parts: int, index: int) -> Tuple[int, int]:
    """Contiguous, balanced [begin, end) slice ``index`` of ``n`` items split into ``parts``."""
    if parts < 1 or not 0 <= index < parts:
        raise ValueError("bad partition")
    base, extra = divmod(n, parts)
    begin = index * base + min(index, extra)
    return begin, begin + base + (1 if index < extra else 0)


def shard_batch_heads(B: int, H: int, world: int, rank: int) -> List[Tuple[int, int, int, int]]:
    """(b_begin, b_count, h_begin, h_count) shards of rank ``rank`` covering its share of the B*H
    (batch, head) units.  Units are ordered batch-major; a rank's range is cut into at most one
    partial head run per batch element, so each tuple is one kernel launch."""
    begin, end = split_range(B * H, world, rank)
    shards = []
    u = begin
    while u < end:
        b, h = divmod(u, H)
        take = min(H - h, end - u)
        shards.append((b, 1, h, take))
        u += take
    # merge whole-batch runs into one launch
    merged: List[Tuple[int, int, int, int]] = []
    for s in shards:
        if merged and s[2] == 0 and s[3] == H and merged[-1][2] == 0 and merged[-1][3] == H \
                and merged[-1][0] + merged[-1][1] == s[0]:
            last = merged.pop()
            merged.append((last[0], last[1] + 1, 0, H))
        else:
            merged.append(s)
    return merged


def _reduce(value: float, op_name: str, group=None) -> float:
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()):
        return value
    backend = dist.get_backend(group)
    dev = torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else torch.device("cpu")
    t = torch.tensor([value], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=getattr(dist.ReduceOp, op_name), group=group)
    return float(t.item())


def max_over_ranks(value: float, group=None) -> float:
    """Max of a per-rank float over the process group (identity without torch.distributed)."""
    return _reduce(value, "MAX", group)


def sum_over_ranks(value: float, group=None) -> float:
    """Sum of a per-rank float over the process group (identity without torch.distributed)."""
    return _reduce(value, "SUM", group)
