"""Head-sharded execution across GPUs (one process per GPU).

Every MInference pattern is independent per head, index estimation
included, so a layer's heads split contiguously over the ranks with no
exchange during attention.  The only exchange is re-assembling the head
outputs for ``o_proj``: an all-gather of each rank's ``[B, S, H/G, D]``
slice (NCCL over NVLink/NVSwitch on B200; gloo works for CPU tests).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

__all__ = ["head_range", "gather_heads"]


def head_range(num_heads: int, rank: int, world: int) -> range:
    """Contiguous heads of `rank`; the first num_heads % world ranks take one extra."""
    if world <= 0 or not (0 <= rank < world):
        raise ValueError(f"bad rank/world {rank}/{world}")
    base, extra = divmod(num_heads, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


def gather_heads(local_bshd: torch.Tensor, num_heads: int, group=None) -> torch.Tensor:
    """All-gather per-rank head slices ``[B, S, h_r, D]`` into ``[B, S, H, D]``.

    Equal shards use one ``all_gather_into_tensor`` (NCCL) into a rank-major
    buffer followed by a head-dim permute; uneven shards (or backends without
    the fused collective) fall back to ``all_gather`` of padded slices."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    B, S, h_local, D = local_bshd.shape
    sizes = [len(head_range(num_heads, r, world)) for r in range(world)]
    if sizes[rank] != h_local:
        raise ValueError(f"rank {rank} holds {h_local} heads, expected {sizes[rank]}")
    hmax = max(sizes)
    x = local_bshd.contiguous()
    if h_local < hmax:
        x = torch.cat([x, x.new_zeros(B, S, hmax - h_local, D)], dim=2)
    use_fused = dist.get_backend(group) == "nccl"
    if use_fused:
        buf = torch.empty((world,) + tuple(x.shape), dtype=x.dtype, device=x.device)
        dist.all_gather_into_tensor(buf, x, group=group)
        parts = list(buf.unbind(0))
    else:
        parts = [torch.empty_like(x) for _ in range(world)]
        dist.all_gather(parts, x, group=group)
    parts = [p[:, :, : sizes[r]] for r, p in enumerate(parts)]
    return torch.cat(parts, dim=2)
