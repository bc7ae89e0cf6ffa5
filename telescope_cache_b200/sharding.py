"""Batch x head sharding of the hot path across GPUs (one process per GPU).

Every (batch, KV head) unit of the builder, the Phase-2 forward / backward
and the decode step is independent (reference.py:897-898, :1494-1495), so a
job shards by giving each rank a contiguous block of KV heads (with their
GQA query heads) or of batch rows; no collective is needed on the data path.
``gather_heads`` / ``gather_batch`` assemble full outputs with one
``all_gather`` when the caller wants them whole (NCCL on GPUs; any
torch.distributed backend works, the tests use gloo on CPU).
"""

from typing import Optional, Tuple

import torch
import torch.distributed as dist


def shard_range(units: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous [start, end) block of `units` for `rank` of `world`: the
    first units % world ranks take one extra unit."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of size {world}")
    if units < 0:
        raise ValueError(f"units must be non-negative, got {units}")
    base, extra = divmod(units, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def head_shard(Hq: int, Hkv: int, world: int, rank: int) -> Tuple[int, int, int, int]:
    """(hkv0, hkv1, hq0, hq1): this rank's KV heads and the query heads of
    their GQA groups (query head hq = hkv * E + e)."""
    if Hkv <= 0 or Hq % Hkv:
        raise ValueError(f"Hq={Hq} must be a positive multiple of Hkv={Hkv}")
    E = Hq // Hkv
    k0, k1 = shard_range(Hkv, world, rank)
    return k0, k1, k0 * E, k1 * E


def _world(group) -> Tuple[int, int]:
    if group is None and not dist.is_initialized():
        return 1, 0
    return dist.get_world_size(group), dist.get_rank(group)


def local_heads(x: torch.Tensor, H: int, group=None, *, E: int = 1, dim: int = 2) -> torch.Tensor:
    """This rank's head block of a tensor with H heads along `dim`, as a
    contiguous tensor.  Heads are split in units of E (the GQA group size for
    query-head tensors, 1 for KV-head tensors), so a rank's query heads are
    exactly those of its KV heads."""
    world, rank = _world(group)
    if E <= 0 or H % E:
        raise ValueError(f"H={H} must be a positive multiple of E={E}")
    u0, u1 = shard_range(H // E, world, rank)
    return x.narrow(dim, u0 * E, (u1 - u0) * E).contiguous()


def _gather(local: torch.Tensor, dim: int, sizes, group) -> torch.Tensor:
    world, _ = _world(group)
    if world == 1:
        return local
    # all_gather needs equal shapes: pad each block to the largest along dim
    mx = max(sizes)
    pad_shape = list(local.shape)
    pad_shape[dim] = mx
    buf = local.new_zeros(pad_shape)
    buf.narrow(dim, 0, local.shape[dim]).copy_(local)
    parts = [torch.empty_like(buf) for _ in range(world)]
    dist.all_gather(parts, buf, group=group)
    return torch.cat([p.narrow(dim, 0, n) for p, n in zip(parts, sizes)], dim=dim)


def gather_heads(local: torch.Tensor, H: int, group=None, *, E: int = 1, dim: int = 2) -> torch.Tensor:
    """Inverse of ``local_heads``: the full tensor with H heads along `dim` on
    every rank, blocks in rank order."""
    world, _ = _world(group)
    sizes = [E * (b - a) for a, b in (shard_range(H // E, world, r) for r in range(world))]
    return _gather(local, dim, sizes, group)


def gather_batch(local: torch.Tensor, B: int, group=None) -> torch.Tensor:
    """Inverse of a batch shard (dim 0)."""
    world, _ = _world(group)
    sizes = [b - a for a, b in (shard_range(B, world, r) for r in range(world))]
    return _gather(local, 0, sizes, group)


__all__ = ["shard_range", "head_shard", "local_heads", "gather_heads", "gather_batch"]
