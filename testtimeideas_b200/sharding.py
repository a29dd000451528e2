"""Sharding of the grad-grad attention step over the GPUs of one box.

Every (batch, head) pair is an independent problem in the forward, the
first-order backward and the double backward, so the flattened b*h axis is cut
into contiguous chunks, one per rank, and each rank runs the whole step on its
chunk with no collective on the data path. Collectives appear only around it:
``max_over_ranks`` for the timing (the job takes as long as its slowest rank)
and ``gather_heads`` to bring every rank's results to rank 0 for verification.

Inputs are generated per global head from (seed, head index), so a head's
inputs, and therefore its results, are the same whatever the number of ranks.
"""

from __future__ import annotations

from typing import Optional, Sequence

import torch

INPUT_NAMES = ("q", "k", "v", "do", "uq", "uk", "uv")


def head_range(total_heads: int, world: int, rank: int) -> range:
    """Contiguous chunk of the flattened b*h axis owned by ``rank``.

    Chunks differ in size by at most one head; the first ``total_heads % world``
    ranks take the extra ones. A rank may own no head when world > total_heads.
    """
    if total_heads < 0 or world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad sharding: total_heads={total_heads} world={world} rank={rank}")
    base, extra = divmod(total_heads, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


def head_inputs(heads: range, t: int, d: int, dtype: torch.dtype, device, *, seed: int = 1234,
                scale_in: float = 1.0, names: Sequence[str] = INPUT_NAMES) -> dict:
    """iid N(0,1)*scale_in inputs ``[1, len(heads), t, d]`` for the given global heads.

    Head ``g`` draws its values from a generator seeded with (seed, g) alone, so
    the inputs of a head do not depend on how the heads are split over ranks.
    """
    out = {n: torch.empty((1, len(heads), t, d), dtype=dtype, device=device) for n in names}
    gen = torch.Generator(device=device)
    for j, g in enumerate(heads):
        gen.manual_seed(seed * 1_000_003 + g)
        block = torch.randn((len(names), t, d), generator=gen, device=device, dtype=torch.float32)
        block.mul_(scale_in)
        for i, n in enumerate(names):
            out[n][0, j].copy_(block[i])
    return out


def max_over_ranks(x: float, group=None, device=None) -> float:
    """Largest value of ``x`` over all ranks (x itself without a process group)."""
    import torch.distributed as dist
    if not dist.is_available() or not dist.is_initialized():
        return float(x)
    t = torch.tensor([float(x)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


def gather_heads(x: torch.Tensor, total_heads: int, group=None) -> Optional[torch.Tensor]:
    """Concatenate every rank's ``[1, heads_r, t, d]`` chunk along the head axis.

    Returns the full ``[1, total_heads, t, d]`` tensor on rank 0 and ``None`` on
    the other ranks. Chunks are padded to the largest chunk size so that one
    all_gather of equal-sized tensors serves both NCCL and gloo.
    """
    import torch.distributed as dist
    if not dist.is_available() or not dist.is_initialized():
        return x
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    mine = head_range(total_heads, world, rank)
    if x.size(1) != len(mine):
        raise ValueError(f"rank {rank} holds {x.size(1)} heads, owns {len(mine)}")
    width = -(-total_heads // world)
    padded = x.new_zeros((x.size(0), width, *x.shape[2:]))
    padded[:, : len(mine)].copy_(x)
    parts = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(parts, padded.contiguous(), group=group)
    if rank != 0:
        return None
    return torch.cat([p[:, : len(head_range(total_heads, world, r))] for r, p in enumerate(parts)], dim=1)
