"""Host side of the multi-GPU partitioning: page-aligned sequence shards of
a long history, the exchange of their partial (O, LSE) and the merge.

KV-head groups and requests are independent and need no exchange (one rank
per tensor-parallel group, vLLM's layout).  A history split across ranks is
the one path with a real exchange step: every rank attends its page-aligned
shard, the partials are all-gathered (NCCL over NVLink on GPUs, gloo in the
CPU tests) and folded with the reference's LSE merge (`merge_slab`,
slab_attention.py:341-373, which `oscar_b200.kernels.merge_slab` runs on the
device).
"""
from __future__ import annotations

import torch


def page_shards(prefix: int, block_size: int, world: int) -> list[tuple[int, int]]:
    """Split history positions [0, prefix) into `world` page-aligned ranges of
    (nearly) equal page counts; trailing ranks may be empty."""
    if world < 1 or block_size < 1 or prefix < 0:
        raise ValueError("page_shards: world >= 1, block_size >= 1, prefix >= 0")
    pages = -(-prefix // block_size)
    per = -(-pages // world) if pages else 0
    out = []
    for r in range(world):
        lo = min(prefix, r * per * block_size)
        hi = min(prefix, (r + 1) * per * block_size)
        out.append((lo, hi))
    return out


def exchange_partials(out: torch.Tensor, lse: torch.Tensor, group=None) -> tuple[list, list]:
    """All-gather every rank's partial (out [n, Hq, D], lse [n, Hq]); returns
    the lists in rank order."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    outs = [torch.empty_like(out) for _ in range(world)]
    lses = [torch.empty_like(lse) for _ in range(world)]
    dist.all_gather(outs, out.contiguous(), group=group)
    dist.all_gather(lses, lse.contiguous(), group=group)
    return outs, lses


def merge_partials(outs: list, lses: list, merge) -> tuple:
    """Fold partials in rank order with ``merge(out, lse, part, part_lse)``,
    which updates (out, lse) in place; returns the merged pair."""
    out, lse = outs[0].clone(), lses[0].clone()
    for o, l in zip(outs[1:], lses[1:]):
        merge(out, lse, o, l)
    return out, lse


def max_over_ranks(value: float, device=None, group=None) -> float:
    """The largest `value` over the ranks of `group` (timings of a step are
    reported as the slowest rank's)."""
    import torch.distributed as dist

    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
