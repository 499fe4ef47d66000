"""Sequence sharding across ranks (one process per GPU).

Every (sequence, layer) unit of the replay step is independent: the
reference's kernels launch one program per (sequence, value head)
(prototype/gdn_replayssm_fp8_kernel.py:369-405) and nothing in the step reads
another sequence's state.  The multi-GPU form of the path therefore partitions
the batch: rank r owns a contiguous range of sequences with its own
checkpoint, scales and rings and calls the same entry points on its own
device.  Nothing crosses GPUs on the data path.  The collectives below are
host-side plumbing over an existing ``torch.distributed`` process group: a
max over ranks for timing, and a gather of per-rank results for validation.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


def shard_range(global_batch: int, world: int, rank: int) -> range:
    """Contiguous sequences of ``rank``: sizes differ by at most one, lower
    ranks take the remainder."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if global_batch < 0:
        raise ValueError(f"global batch {global_batch} < 0")
    base, extra = divmod(global_batch, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


@dataclass(frozen=True)
class ShardPlan:
    """The batch split of one job: ``ranges[r]`` are rank r's sequences."""

    global_batch: int
    world: int

    @property
    def ranges(self) -> list[range]:
        return [shard_range(self.global_batch, self.world, r) for r in range(self.world)]

    def local(self, rank: int) -> range:
        return shard_range(self.global_batch, self.world, rank)

    def owner(self, seq: int) -> int:
        """Rank holding global sequence ``seq``."""
        if not 0 <= seq < self.global_batch:
            raise ValueError(f"sequence {seq} outside a batch of {self.global_batch}")
        for r, rg in enumerate(self.ranges):
            if seq in rg:
                return r
        raise AssertionError("ranges do not cover the batch")

    def take(self, x: torch.Tensor, rank: int, dim: int = 0) -> torch.Tensor:
        """Rank ``rank``'s slice of a global tensor along the batch dimension."""
        if x.shape[dim] != self.global_batch:
            raise ValueError(f"dimension {dim} has {x.shape[dim]} sequences, the plan {self.global_batch}")
        rg = self.local(rank)
        return x.narrow(dim, rg.start, len(rg))


def _collective_device(group=None) -> torch.device:
    import torch.distributed as dist

    if dist.get_backend(group) == "nccl":
        return torch.device("cuda", torch.cuda.current_device())
    return torch.device("cpu")


def max_over_ranks(x: float, group=None) -> float:
    """The largest ``x`` over the ranks of ``group`` (every rank calls it)."""
    import torch.distributed as dist

    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return float(x)
    t = torch.tensor([float(x)], dtype=torch.float64, device=_collective_device(group))
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


def gather_shards(local: torch.Tensor, plan: ShardPlan, group=None) -> torch.Tensor:
    """All ranks' batch slices (dimension 0) concatenated in sequence order, on
    every rank.  Shards of unequal size are padded for the exchange."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    if world != plan.world:
        raise ValueError(f"plan for {plan.world} ranks, process group of {world}")
    rank = dist.get_rank(group)
    if local.shape[0] != len(plan.local(rank)):
        raise ValueError(f"rank {rank} holds {local.shape[0]} sequences, the plan gives it {len(plan.local(rank))}")
    dev = _collective_device(group)
    width = max(len(rg) for rg in plan.ranges)
    buf = torch.zeros((width,) + tuple(local.shape[1:]), dtype=local.dtype, device=dev)
    buf[: local.shape[0]] = local.to(dev)
    parts = [torch.empty_like(buf) for _ in range(world)]
    dist.all_gather(parts, buf, group=group)
    return torch.cat([parts[r][: len(plan.ranges[r])] for r in range(world)], dim=0)
