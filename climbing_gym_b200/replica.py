"""One engine replica per GPU: request sharding and the NCCL policy-weight broadcast.

The 1.2B model fits one B200 many times over, so multi-GPU rollout is replicas, not model
parallelism: requests are independent units (each carries its own RNG stream), they are dealt
round-robin to the ranks, and no collective touches the data path. The single exchange is the
policy update: the trainer rank broadcasts the packed bf16 weights over NVLink straight into every
replica's EXISTING buffers (captured graphs hold those addresses), after which each replica
re-quantises its FP8 copies locally. The reference is single-GPU and syncs with a same-device
``copy_`` (src/climbing_gym/inference/lfm25_engine.py:225-367, 555-578); this module is its
multi-GPU counterpart.

``torch.distributed`` is the plumbing (backend "nccl" on GPUs, "gloo" in the CPU tests).
"""
from __future__ import annotations

from typing import Sequence, TypeVar

import torch
import torch.distributed as dist

T = TypeVar("T")


def shard_round_robin(items: Sequence[T], rank: int, world_size: int) -> list[T]:
    """Items rank, rank + world, rank + 2 world, ... (a group of samples of one prompt is ONE item,
    so its prefix pages are shared inside one replica)."""
    if not 0 <= rank < world_size:
        raise ValueError("rank must be in [0, world_size)")
    return [item for index, item in enumerate(items) if index % world_size == rank]


def shard_indices(count: int, rank: int, world_size: int) -> list[int]:
    return shard_round_robin(range(count), rank, world_size)


def gather_results(local: list, count: int, rank: int, world_size: int, group=None) -> list | None:
    """Inverse of shard_round_robin on rank 0 (host objects: token lists, log-prob lists)."""
    if world_size == 1:
        return list(local)
    gathered = [None] * world_size if rank == 0 else None
    dist.gather_object(local, gathered, dst=0, group=group)
    if rank != 0:
        return None
    merged = [None] * count
    for r, part in enumerate(gathered):
        for item, index in zip(part, shard_indices(count, r, world_size)):
            merged[index] = item
    return merged


def broadcast_tensors(tensors: Sequence[torch.Tensor], src: int = 0, group=None, *, bucket_bytes: int = 256 << 20) -> int:
    """In-place broadcast of every tensor from ``src``. Small tensors (norm weights, conv taps) are
    packed into buckets so the ~150 per-tensor launches become a handful; NVSwitch gives every
    peer full bandwidth, so buckets are sized for launch latency, not link count. Returns bytes moved."""
    rank = dist.get_rank(group)
    moved = 0
    small: list[torch.Tensor] = []

    def flush():
        if not small:
            return
        flat = torch.cat([t.reshape(-1).view(torch.uint8) for t in small])
        dist.broadcast(flat, src=src, group=group)
        if rank != src:
            offset = 0
            for t in small:
                n = t.numel() * t.element_size()
                t.reshape(-1).view(torch.uint8).copy_(flat[offset:offset + n])
                offset += n
        small.clear()

    pending = 0
    for t in tensors:
        size = t.numel() * t.element_size()
        moved += size
        if size >= (8 << 20) and t.is_contiguous():
            dist.broadcast(t, src=src, group=group)  # large matrices go straight into place
        else:
            if not t.is_contiguous():
                raise ValueError("packed weight buffers must be contiguous for an in-place broadcast")
            small.append(t)
            pending += size
            if pending >= bucket_bytes:
                flush()
                pending = 0
    flush()
    return moved


def broadcast_policy_weights(engine, src: int = 0, group=None) -> int:
    """Trainer rank -> every replica, then local FP8 refresh and a policy-version bump."""
    moved = broadcast_tensors(engine.weights.tensors(), src=src, group=group)
    engine.weights_updated()
    return moved
