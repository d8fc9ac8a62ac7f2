"""Batch x head partitioning of the delta-rule core across the GPUs of one node.

Heads never interact in the delta rule (each (batch, head) pair owns its own
state, src/delta/recurrent.rs:41-99), so the work splits into independent
units with no exchange on the data path.  One process per GPU owns a
contiguous block of the (batch, head) grid, runs the kernels on it, and — only
when every rank needs the whole output — the outputs are all-gathered once at
the end (NCCL over NVLink; gloo on CPU for tests).

Blocks are batch-major: when the batch divides evenly every rank owns whole
sequences, so the gathered buffer is already [batch, seq, heads, dv] with no
permute.  Otherwise each sequence's heads are split into `world / batch`
groups, and the gather permutes once.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional

import torch


@dataclass(frozen=True)
class Shard:
    """Rank `rank`'s block: batches [b0, b1) x heads [h0, h1)."""
    rank: int
    world: int
    b0: int
    b1: int
    h0: int
    h1: int

    @property
    def batch(self) -> int:
        return self.b1 - self.b0

    @property
    def heads(self) -> int:
        return self.h1 - self.h0


def plan(batch: int, heads: int, world: int) -> List[Shard]:
    """Contiguous batch-major blocks of the (batch, head) grid, one per rank.

    Whole sequences per rank when ``batch % world == 0``; otherwise requires
    ``world % batch == 0`` and splits each sequence's heads evenly.
    """
    if world < 1:
        raise ValueError("world must be >= 1")
    if batch % world == 0:
        per = batch // world
        return [Shard(r, world, r * per, (r + 1) * per, 0, heads) for r in range(world)]
    if world % batch == 0 and heads % (world // batch) == 0:
        groups = world // batch
        hp = heads // groups
        return [Shard(r, world, r // groups, r // groups + 1, (r % groups) * hp, (r % groups + 1) * hp)
                for r in range(world)]
    raise ValueError(f"cannot split batch={batch} x heads={heads} evenly over {world} ranks")


def take(t: Optional[torch.Tensor], shard: Shard, head_axis: int = 2) -> Optional[torch.Tensor]:
    """The shard's slice of a global tensor (batch on axis 0, heads on
    `head_axis`), contiguous.  [b, s, h, .] tensors use head_axis=2, the state
    [b, h, dk, dv] head_axis=1."""
    if t is None:
        return None
    idx = [slice(None)] * t.dim()
    idx[0] = slice(shard.b0, shard.b1)
    idx[head_axis] = slice(shard.h0, shard.h1)
    return t[tuple(idx)].contiguous()


def gather_into(out: torch.Tensor, local: torch.Tensor, shards: List[Shard], group=None) -> torch.Tensor:
    """All-gather batch-major whole-sequence blocks into a caller-owned global
    buffer ``out`` ([world * local_batch, ...]), with no allocation: the form a
    caller that gathers every step's output into the same buffer uses."""
    import torch.distributed as dist

    if not all(s.h0 == 0 for s in shards):
        raise ValueError("gather_into takes whole-sequence shards (batch % world == 0)")
    if tuple(out.shape) != (len(shards) * local.shape[0],) + tuple(local.shape[1:]):
        raise ValueError(f"out has shape {tuple(out.shape)}")
    dist.all_gather_into_tensor(out, local, group=group)
    return out


def gather(local: torch.Tensor, shards: List[Shard], head_axis: int = 2, group=None) -> torch.Tensor:
    """All-gather every rank's output block into the global tensor.

    One collective (``all_gather_into_tensor``); batch-major shards concatenate
    along batch directly, head-split shards are permuted back once."""
    import torch.distributed as dist

    world = len(shards)
    # concatenated along the batch axis: [world * local_batch, ...]
    out = torch.empty((world * local.shape[0],) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(out, local.contiguous(), group=group)
    if all(s.h0 == 0 for s in shards):
        return out  # whole sequences: already [batch, ...]
    groups = sum(1 for s in shards if s.b0 == 0)
    # ranks are (batch, head group) row-major and each holds one sequence:
    # [world, 1, ...] -> [B, G, ...] with the per-rank batch axis dropped
    out = out.reshape((world // groups, groups) + tuple(local.shape[1:]))
    # move the group axis in front of the per-group head axis, then merge them
    out = out.movedim(1, head_axis)
    sizes = list(out.shape)
    merged = sizes[:head_axis] + [sizes[head_axis] * sizes[head_axis + 1]] + sizes[head_axis + 2:]
    return out.reshape(merged)
