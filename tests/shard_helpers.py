"""Test helpers for the hash-sharded store across ranks (one process per GPU).

A plain-Python restatement of the store's key placement (fnv1a32(key) % n_shards, the function
the C ABI applies in kvs_client_shard_of), used by the tests to check the product's vectorised
placement and to group a batch by owning shard; and the max-over-ranks reduction of a time."""

from __future__ import annotations

from typing import Sequence

import numpy as np


def fnv1a32(data: bytes) -> int:
    h = 2166136261
    for b in data:
        h ^= b
        h = (h * 16777619) & 0xFFFFFFFF
    return h


def shard_of(key: int | bytes, n_shards: int) -> int:
    """Owning shard of a key (64-bit keys are their 8 little-endian bytes)."""
    if n_shards == 1:
        return 0
    b = int(key).to_bytes(8, "little") if not isinstance(key, (bytes, bytearray)) else bytes(key)
    return fnv1a32(b) % n_shards


def bucket_by_shard(keys: Sequence[int], n_shards: int) -> tuple[np.ndarray, np.ndarray]:
    """(perm, counts): keys[perm] is grouped by owning shard in ascending order (stable), counts[s]
    is the number of keys shard s owns."""
    owners = np.array([shard_of(int(k), n_shards) for k in keys], dtype=np.int64)
    perm = np.argsort(owners, kind="stable")
    counts = np.bincount(owners, minlength=n_shards)
    return perm, counts


def max_over_ranks(value: float, device=None) -> float:
    """The job's time for a per-rank time: the max over ranks (identity without a process group)."""
    import torch
    import torch.distributed as dist

    if not dist.is_available() or not dist.is_initialized():
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
