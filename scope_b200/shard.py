"""Head sharding of one SCOPE attention layer over ranks (one process per GPU).

Every stage of the hot path is per head: the pointer builder selects and
packs blocks for each (head, q block) row on its own, the spectral bias is a
per-head coefficient set, and the attention of a head reads only that head's
q / k / v.  Rank r of N therefore owns heads [r*H/N, (r+1)*H/N) and runs the
path on them with no collective inside the step.  The layer's results are
combined afterwards, which is the path's one exchange:

  * the attention output [T, H, D] is an all-gather of the ranks' head slices
    (NCCL over NVLink on a B200 node), and
  * the builder's pointer statistics (histograms of list lengths, radii and
    centre offsets over all heads, the reference's debug stats of
    model/attn_bias.py:839-849) are a sum over ranks.

The reference itself trains with data parallelism only (a gradient
all-reduce, scoped_medium.py:2415); head sharding is this implementation's way of
spreading one layer over the GPUs of a node.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.distributed as dist


def head_slice(H: int, rank: int, world: int) -> slice:
    """The heads rank `rank` of `world` owns; H must divide evenly."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world}")
    if H % world:
        raise ValueError(f"H={H} heads do not split over {world} ranks")
    hp = H // world
    return slice(rank * hp, (rank + 1) * hp)


def gather_buffer(T: int, H: int, D: int, world: int, dtype: torch.dtype, device) -> torch.Tensor:
    """Receive buffer of gather_heads: [world, T, H/world, D]."""
    return torch.empty(world, T, H // world, D, dtype=dtype, device=device)


def gather_heads(out_local: torch.Tensor, buf: torch.Tensor, group=None, async_op: bool = False):
    """All-gather of the ranks' output head slices.

    out_local: this rank's output, [T, H/N, D] (any strides; the attention
    writes [H/N, T, D] views of [T, H/N, D] storage, which this takes as
    `out.transpose(0, 1)` without a copy when contiguous that way).
    buf: gather_buffer(...).  Returns (full, work): `full` is the [T, H, D]
    view of `buf` (head h of rank r at r*H/N + h), valid once `work` (None
    unless async_op) has been waited on.
    """
    world, T, hp, D = buf.shape
    src = out_local if out_local.is_contiguous() else out_local.contiguous()
    if tuple(src.shape) != (T, hp, D):
        raise ValueError(f"local output {tuple(src.shape)} does not match the buffer's slice {(T, hp, D)}")
    # the receive tensor as the ranks' inputs stacked along dim 0 (the form every backend takes)
    work = dist.all_gather_into_tensor(buf.view(world * T, hp, D), src, group=group, async_op=async_op)
    full = buf.permute(1, 0, 2, 3)            # [T, N, H/N, D]: head index r*H/N + h
    return full, work


def full_heads(full: torch.Tensor) -> torch.Tensor:
    """[T, N, H/N, D] -> [T, H, D] (a copy)."""
    T, world, hp, D = full.shape
    return full.reshape(T, world * hp, D)


def reduce_stats(stats_local: torch.Tensor, group=None, async_op: bool = False) -> Tuple[torch.Tensor, Optional[object]]:
    """Sum of the ranks' pointer-statistics histograms, in place."""
    work = dist.all_reduce(stats_local, op=dist.ReduceOp.SUM, group=group, async_op=async_op)
    return stats_local, work
