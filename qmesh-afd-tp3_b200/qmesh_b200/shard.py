"""Column-split tensor parallelism of the routed experts across the GPUs of one box.

The reference splits every expert's 2304 intermediate columns across machines
(NODE-A [0:576), NODE-B [576:1440), NODE-C [1440:2304); pack/build_packs.py:50)
and sums the BF16 partials on NODE-A in FP32 in a fixed order
(native/qmesh_afd_seam.cu:310-361, README.md:88-90). Inside one B200 box the
ranks are GPUs: rank r holds columns [r*2304/N, (r+1)*2304/N) of every expert,
computes its partial from replicated x/ids/tw, and the partials meet on the
output rank, summed in rank order with one BF16 rounding.
"""

from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist

INTER = 2304


def shard_range(rank: int, world: int, inter: int = INTER, align: int = 32) -> tuple[int, int]:
    """Contiguous equal column shard of `rank`; widths must stay `align`-aligned."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    if inter % world or (inter // world) % align:
        raise ValueError(f"{inter} columns do not split into {world} {align}-aligned shards")
    w = inter // world
    return rank * w, (rank + 1) * w


def gather_partials(part: torch.Tensor, group=None, out_list: list[torch.Tensor] | None = None) -> list[torch.Tensor]:
    """All ranks' partials, in rank order (index i = rank i's partial)."""
    world = dist.get_world_size(group)
    if out_list is None:
        out_list = [torch.empty_like(part) for _ in range(world)]
    dist.all_gather(out_list, part, group=group)
    return out_list


def combine_across_ranks(part: torch.Tensor, group=None, dst: int = 0, shared: torch.Tensor | None = None,
                         out: torch.Tensor | None = None,
                         combine: Callable[..., torch.Tensor] | None = None,
                         gathered: list[torch.Tensor] | None = None) -> torch.Tensor | None:
    """Rank-ordered FP32 combine of every rank's BF16 partial on rank `dst`.

    All ranks take the same collective steps; only `dst` returns the combined
    BF16 output (bf16(p0 + p1 + ... [+ shared])), the others return None.
    `combine` defaults to the device kernel (qmesh_b200.combine.combine_ordered).
    """
    if combine is None:
        from .combine import combine_ordered as combine
    parts = gather_partials(part, group, gathered)
    if dist.get_rank(group) != dst:
        return None
    if shared is not None:
        parts = list(parts) + [shared]
    return combine(parts, out=out)
