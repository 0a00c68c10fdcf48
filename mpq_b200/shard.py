"""Row-sharded layer solve across the GPUs of one node (one process per GPU, torch.distributed).

Output rows of W are independent given H: the reference's row-block chain only passes the scalar
obs-precision warm start from one block to the next (mpq/adapters/gptqmodel.py:1065-1066,
mpq/adapters/quip_sharp.py:585-586).  A layer is therefore split into contiguous row shards, one per
rank; each shard starts its chain from the layer-wide warm start ("restart per shard"), so a shard
solves exactly what the single-GPU solve does for a row block of the same rows when that block is the
first of its chain.  There is no collective on the data path: W and H are broadcast once from the
source rank (NCCL over NVLink on GPUs, gloo on CPU), and the per-shard results are gathered where the
caller wants the whole layer.
"""
from __future__ import annotations

from typing import Callable, List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist


def row_shards(m: int, world: int, align: int = 1) -> List[Tuple[int, int]]:
    """Contiguous [r0, r1) row ranges, one per rank, sizes multiples of `align` except the last.

    Rows are split as evenly as the alignment allows; ranks beyond the available rows get empty shards."""
    if m < 0 or world < 1 or align < 1:
        raise ValueError(f"bad shard request m={m} world={world} align={align}")
    units = (m + align - 1) // align
    base, extra = divmod(units, world)
    out, r = [], 0
    for k in range(world):
        u = base + (1 if k < extra else 0)
        r1 = min(m, r + u * align)
        out.append((r, r1))
        r = r1
    return out


def _world(group) -> Tuple[int, int]:
    if not (dist.is_available() and dist.is_initialized()):
        return 0, 1
    return dist.get_rank(group), dist.get_world_size(group)


def broadcast_(tensors: Sequence[torch.Tensor], src: int = 0, group=None) -> None:
    """In-place broadcast of each tensor from `src` (no-op without a process group)."""
    _, world = _world(group)
    if world == 1:
        return
    for t in tensors:
        dist.broadcast(t, src, group=group)


def gather_rows(local: torch.Tensor, shards: Sequence[Tuple[int, int]], group=None) -> torch.Tensor:
    """All-gather row shards (shard k holds rows shards[k]) into the full matrix on every rank."""
    rank, world = _world(group)
    if world == 1:
        return local
    if len(shards) != world:
        raise ValueError("one shard per rank expected")
    r0, r1 = shards[rank]
    if local.shape[0] != r1 - r0:
        raise ValueError(f"rank {rank} holds {local.shape[0]} rows, shard is {r1 - r0}")
    rows = max(b - a for a, b in shards)
    pad = torch.zeros((rows,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    pad[: local.shape[0]] = local
    parts = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(parts, pad, group=group)
    return torch.cat([p[: b - a] for p, (a, b) in zip(parts, shards)], dim=0)


def solve_layer_sharded(W: torch.Tensor, H: torch.Tensor, solve_rows: Callable[[torch.Tensor, torch.Tensor], Sequence[torch.Tensor]],
                        *, align: int = 1, src: int = 0, group=None, gather: bool = True) -> List[torch.Tensor]:
    """Broadcast (W, H) from `src`, solve this rank's rows with `solve_rows(W_rows, H)` and (optionally)
    gather every row-indexed output into the full layer on every rank.

    `solve_rows` returns tensors whose first dimension is the shard's rows."""
    rank, world = _world(group)
    broadcast_([W, H], src=src, group=group)
    shards = row_shards(W.shape[0], world, align)
    r0, r1 = shards[rank]
    outs = list(solve_rows(W[r0:r1].contiguous(), H))
    if not gather or world == 1:
        return outs
    return [gather_rows(o, shards, group=group) for o in outs]
