"""Head sharding of one SCOPE attention layer over ranks (one process per GPU).

Every stage of the hot path is per head: the pointer builder selects and
packs blocks for each (head, q block) row on its own, the spectral bias is a
per-head coefficient set, and the attention of a head reads only that head's
q / k / v.  Rank r of N therefore owns heads [r*H/N, (r+1)*H/N) and runs the
path on them with no collective inside the step.  The layer's results are
combined afterwards, which is the path's one exchange:

  * the attention output is an all-gather of the ranks' head slices (NCCL
    over NVLink on a B200 node): each rank writes its [H/N, T, D] slice
    head-major (``flex_attention(..., head_major_out=True)``), so the
    gathered buffer is the [H, T, D] output with no permute, and
  * the builder's pointer statistics (histograms of list lengths, radii and
    centre offsets over this rank's heads, the reference's debug stats of
    model/attn_bias.py:839-849) are all-gathered as [N, n] rows; their sum
    over ranks is the statistics of the whole layer.

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
    """Receive buffer of gather_heads: the [H, T, D] output of the layer."""
    return torch.empty(H, T, D, dtype=dtype, device=device)


def gather_heads(out_local: torch.Tensor, buf: torch.Tensor, group=None, async_op: bool = False):
    """All-gather of the ranks' output head slices.

    out_local: this rank's [H/N, T, D] output, head-major contiguous (what
    ``flex_attention(..., head_major_out=True)`` writes; other layouts are
    copied first).  buf: gather_buffer(...), [H, T, D]; rank r's heads land
    at [r*H/N, (r+1)*H/N).  Returns (buf, work): buf holds the layer's
    [H, T, D] output once `work` (None unless async_op) has been waited on.
    """
    H, T, D = buf.shape
    src = out_local if out_local.is_contiguous() else out_local.contiguous()
    world = dist.get_world_size(group)
    if tuple(src.shape) != (H // world, T, D):
        raise ValueError(f"local output {tuple(src.shape)} does not match the buffer's slice {(H // world, T, D)}")
    work = dist.all_gather_into_tensor(buf, src, group=group, async_op=async_op)
    return buf, work


def stats_buffer(stats_local: torch.Tensor, world: int) -> torch.Tensor:
    """Receive buffer of gather_stats: [world, n]."""
    return torch.empty(world, stats_local.numel(), dtype=stats_local.dtype, device=stats_local.device)


def gather_stats(stats_local: torch.Tensor, buf: torch.Tensor, group=None,
                 async_op: bool = False) -> Tuple[torch.Tensor, Optional[object]]:
    """All-gather of the ranks' pointer-statistics histograms into buf [N, n]
    (row r = rank r's heads); ``buf.sum(0)`` is the whole layer's."""
    # the receive tensor as the ranks' inputs concatenated (the form every backend takes)
    work = dist.all_gather_into_tensor(buf.view(-1), stats_local.contiguous().view(-1), group=group,
                                       async_op=async_op)
    return buf, work
