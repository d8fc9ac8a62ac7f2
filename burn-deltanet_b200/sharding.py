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


class PeerGather:
    """The all-gather of :func:`gather_into` on the NVLink copy engines instead of the SMs.

    Every rank holds a global buffer ``out`` ([world * local_batch, ...], batch-major whole-sequence
    shards), writes its own block (rows [b0, b1)) there directly, and :meth:`push` copies that block into
    the same rows of every peer's buffer: one peer-to-peer copy per peer, in ring order on one stream, through
    CUDA IPC mappings of the peers' buffers exchanged once through the process group (driver API, in the
    device's primary context, which torch makes current).  An NCCL gather runs as kernels whose CTAs take
    SMs from a one-wave prefill; these copies take none, so the gather of one step runs beside the
    kernels of the next.

    Collective: every rank constructs it with buffers of the same shape, in the same order, and every
    rank calls :meth:`close` before any rank frees its buffer.
    """

    _opened = {}  # (peer rank, IPC handle) -> [mapped base, references]: one mapping per allocation

    def __init__(self, out: torch.Tensor, shards: List[Shard], group=None, streams: int = 1, parts: int = 1):
        import torch.distributed as dist
        from cuda.bindings import driver as drv

        self._drv = drv
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        if len(shards) != world or not all(s.h0 == 0 for s in shards):
            raise ValueError("PeerGather takes whole-sequence shards, one per rank")
        if not out.is_cuda or not out.is_contiguous() or out.shape[0] != shards[-1].b1:
            raise ValueError(f"out must be a contiguous CUDA buffer of {shards[-1].b1} rows")
        row = out[0].numel() * out.element_size()
        self.offset = shards[rank].b0 * row
        self.nbytes = shards[rank].batch * row
        # Every rank takes the same collective steps whatever fails locally: the export and the mappings
        # each end in an exchange of (result, error), and all ranks raise together if any rank failed.
        mine, error = None, ""
        try:
            torch.cuda.set_device(out.device)
            err, dev = drv.cuCtxGetDevice()
            _check(err, "cuCtxGetDevice")
            if int(dev) != out.device.index:
                raise RuntimeError(f"the current CUDA context is device {int(dev)}, not {out.device}")
            err, base, _ = drv.cuMemGetAddressRange(out.data_ptr())
            _check(err, "cuMemGetAddressRange")
            err, handle = drv.cuIpcGetMemHandle(base)
            _check(err, "cuIpcGetMemHandle")
            mine = (bytes(handle.reserved), out.data_ptr() - int(base))
        except Exception as e:  # noqa: BLE001 (raised on every rank below)
            error = f"rank {rank}: {type(e).__name__}: {e}"
        every = [None] * world
        dist.all_gather_object(every, (mine, error), group=group)
        errors = [e for _, e in every if e]
        if errors:
            raise RuntimeError("PeerGather: " + "; ".join(errors))
        self.peers = []  # (peer rank, IPC handle key, address of the peer's `out`)
        error = ""
        for p in range(world):
            if p == rank:
                continue
            key = (p, every[p][0][0])
            try:
                if key not in PeerGather._opened:
                    h = drv.CUipcMemHandle()
                    h.reserved = every[p][0][0]
                    err, ptr = drv.cuIpcOpenMemHandle(h, drv.CUipcMem_flags.CU_IPC_MEM_LAZY_ENABLE_PEER_ACCESS)
                    _check(err, "cuIpcOpenMemHandle")
                    PeerGather._opened[key] = [int(ptr), 0]
                PeerGather._opened[key][1] += 1
                self.peers.append((p, key, PeerGather._opened[key][0] + every[p][0][1]))
            except Exception as e:  # noqa: BLE001
                error = f"rank {rank}: {type(e).__name__}: {e}"
                break
        results = [None] * world
        dist.all_gather_object(results, error, group=group)
        if any(results):
            self.streams, self._pool = [], []
            self._release()
            raise RuntimeError("PeerGather: " + "; ".join(r for r in results if r))
        # Peers in ring order from this rank (rank + 1, rank + 2, ...), so that ranks copying in step
        # send to different peers at any moment; `streams` copy streams (0: one per peer) take the peers
        # round robin, each stream's copies in that order.  One stream measured fastest: config 2 at
        # N = 8, 1.71 ms per gathered step against 2.09 (2 streams), 2.22 (4) and 2.23 (7), and 1.95
        # with NCCL's gather.
        self.peers.sort(key=lambda e: (e[0] - rank) % world)
        self.out = out
        self.src = out.data_ptr() + self.offset
        # `parts` > 1 cuts every copy into that many pieces, piece s of each peer's copy on its own stream.
        n = len(self.peers) if streams <= 0 else min(streams, len(self.peers))
        self.parts = max(1, int(parts))
        self._pool = [torch.cuda.Stream(device=out.device) for _ in range(n * self.parts)] if n else []
        self.streams = [i % n for i in range(len(self.peers))] if n else []

    def push(self, after: torch.cuda.Event) -> List[torch.cuda.Event]:
        """Copy this rank's block into every peer's buffer once ``after`` has fired; returns one event per
        copy stream (this rank's block may be rewritten once they have all fired)."""
        drv = self._drv
        for stream in self._pool:
            stream.wait_event(after)
        piece = (self.nbytes // self.parts + 15) // 16 * 16
        for (_, _, dst), si in zip(self.peers, self.streams):
            for s in range(self.parts):
                lo = s * piece
                n = min(piece, self.nbytes - lo)
                if n <= 0:
                    continue
                stream = self._pool[si * self.parts + s]
                (err,) = drv.cuMemcpyAsync(dst + self.offset + lo, self.src + lo, n, stream.cuda_stream)
                _check(err, "cuMemcpyAsync")
        done = []
        for stream in self._pool:
            ev = torch.cuda.Event()
            ev.record(stream)
            done.append(ev)
        return done

    def close(self) -> None:
        """Drain the copies and release the peer mappings (every rank, before any buffer is freed)."""
        for stream in getattr(self, "_pool", []):
            stream.synchronize()
        self._release()
        self.streams, self._pool = [], []

    def _release(self) -> None:
        for _, key, _ in self.peers:
            ent = PeerGather._opened[key]
            ent[1] -= 1
            if ent[1] == 0:
                _check(self._drv.cuIpcCloseMemHandle(ent[0])[0], "cuIpcCloseMemHandle")
                del PeerGather._opened[key]
        self.peers = []


def _check(err, what: str) -> None:
    if int(err) != 0:
        raise RuntimeError(f"{what} failed: {err}")


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
