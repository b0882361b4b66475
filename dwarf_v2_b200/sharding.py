"""Batch-row sharding of the prefill over ranks (one process per GPU).

DWARF-v2 rows never attend to each other, so a global batch splits into
contiguous row ranges, one per rank, with no collective on the data path; the
only exchange is one gather of each row's next-token logits at the end.
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def rows_for_rank(global_batch: int, rank: int, world: int) -> slice:
    """Contiguous rows of rank `rank`; the global batch must divide evenly."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world {world}")
    if global_batch % world:
        raise ValueError(f"global batch {global_batch} must divide by {world} ranks")
    per = global_batch // world
    return slice(rank * per, (rank + 1) * per)


def gather_rows(local: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """Concatenate every rank's rows (rank order) on every rank.

    NCCL uses one all_gather_into_tensor; other backends (gloo, for host
    tests) use the list form. World size 1 is a copy.
    """
    world = dist.get_world_size() if dist.is_available() and dist.is_initialized() else 1
    if out is None:
        out = torch.empty((local.shape[0] * world, *local.shape[1:]), dtype=local.dtype, device=local.device)
    if world == 1:
        out.copy_(local)
    elif dist.get_backend() == "nccl":
        dist.all_gather_into_tensor(out, local.contiguous())
    else:
        parts = list(out.chunk(world, dim=0))
        dist.all_gather(parts, local.contiguous())
    return out
