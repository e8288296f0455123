"""Chunk gather / scatter ops over paged KV members (torch CUDA tensors).

B200 counterparts of ttnn.kvcache_manager.gather_tp_shards_to_chip / scatter_chunk_from_chip /
pack_local_shards / unpack_local_shards (patch 0003 gather.hpp lines 9335-9453). A "rank" is a
GPU that owns one TP shard of every member; `members[r][m]` is rank r's shard of member m. The
master GPU (the device of `dst` / `src`) moves every byte with one kernel, reading or writing the
other ranks' shards over NVLink peer access. Layout: for member m, chunk block cb and rank r, the
shard_block_bytes bytes at block_ids[cb] * shard_block_bytes of members[r][m] live in the blob at
region_bases[m] + cb * shard_block_bytes * n_ranks + r * shard_block_bytes.
"""

from __future__ import annotations

import ctypes as C
from typing import Any, Sequence

from . import _native
from ._native import check, load


def _torch():
    import torch

    return torch


def _nbytes(t: Any) -> int:
    return t.numel() * t.element_size()


def _enable_peers(master: int, devices: set[int]) -> None:
    torch = _torch()
    lib = load()  # noqa: F841 - the library must be loaded before any op
    for d in devices:
        if d != master and not torch.cuda.can_device_access_peer(master, d):
            raise RuntimeError(f"device {master} cannot access peer device {d}")


def _member_arrays(members: Sequence[Sequence[Any]], shard_block_bytes: int):
    n_ranks, n_members = len(members), len(members[0])
    if any(len(r) != n_members for r in members):
        raise RuntimeError("every rank must provide the same members")
    flat = [members[r][m] for r in range(n_ranks) for m in range(n_members)]
    for i, t in enumerate(flat):
        if t.device.type != "cuda":
            raise RuntimeError("kvcache gather: tensor must be on device")
        if not t.is_contiguous():
            raise RuntimeError("kvcache gather: tensor must be contiguous")
    ptrs = (C.c_uint64 * len(flat))(*[t.data_ptr() for t in flat])
    sbb = (C.c_uint64 * n_members)(*([shard_block_bytes] * n_members))
    extent = (C.c_uint64 * n_members)(*[min(_nbytes(members[r][m]) for r in range(n_ranks)) for m in range(n_members)])
    return n_ranks, n_members, ptrs, sbb, extent, {t.device.index for t in flat}


def gather_tp_shards_to_chip(members: Sequence[Sequence[Any]], dst: Any, block_ids: Sequence[int],
                             shard_block_bytes: int, region_bases: Sequence[int],
                             header_words: Sequence[int] = (), blocking: bool = True) -> None:
    """Gather one chunk of a TP-sharded paged cache into `dst` on its GPU (see module doc)."""
    torch = _torch()
    n_ranks, n_members, ptrs, sbb, extent, devs = _member_arrays(members, shard_block_bytes)
    if len(region_bases) != n_members:
        raise RuntimeError(f"kvcache gather: {n_members} members but {len(region_bases)} region bases")
    master = dst.device.index
    _enable_peers(master, devs)
    ids = (C.c_uint32 * len(block_ids))(*block_ids)
    rb = (C.c_uint64 * n_members)(*region_bases)
    hw = (C.c_uint32 * max(1, len(header_words)))(*[int(w) & 0xFFFFFFFF for w in header_words])
    with torch.cuda.device(master):
        stream = torch.cuda.current_stream(master)
        check(load().kvs_gather_chunk(ptrs, n_ranks, n_members, sbb, extent, ids, len(block_ids), rb, hw,
                                      len(header_words), C.c_void_p(dst.data_ptr()), _nbytes(dst),
                                      C.c_void_p(stream.cuda_stream)))
        if blocking:
            stream.synchronize()


def scatter_chunk_from_chip(src: Any, members: Sequence[Sequence[Any]], block_ids: Sequence[int],
                            shard_block_bytes: int, region_bases: Sequence[int], blocking: bool = True) -> None:
    """Inverse of gather_tp_shards_to_chip: write each rank's slice of `src` into its blocks."""
    torch = _torch()
    n_ranks, n_members, ptrs, sbb, extent, devs = _member_arrays(members, shard_block_bytes)
    if len(region_bases) != n_members:
        raise RuntimeError(f"kvcache scatter: {n_members} members but {len(region_bases)} region bases")
    master = src.device.index
    _enable_peers(master, devs)
    ids = (C.c_uint32 * len(block_ids))(*block_ids)
    rb = (C.c_uint64 * n_members)(*region_bases)
    with torch.cuda.device(master):
        stream = torch.cuda.current_stream(master)
        check(load().kvs_scatter_chunk(C.c_void_p(src.data_ptr()), _nbytes(src), ptrs, n_ranks, n_members, sbb,
                                       extent, ids, len(block_ids), rb, C.c_void_p(stream.cuda_stream)))
        if blocking:
            stream.synchronize()


def pack_local_shards(members: Sequence[Any], dst: Any, block_ids: Sequence[int], shard_block_bytes: int,
                      region_bases: Sequence[int], header_words: Sequence[int] = (), blocking: bool = True) -> None:
    """Per-GPU pack: this GPU's own shard of every member into `dst` (one rank, no peers)."""
    gather_tp_shards_to_chip([list(members)], dst, block_ids, shard_block_bytes, region_bases, header_words, blocking)


def unpack_local_shards(src: Any, members: Sequence[Any], block_ids: Sequence[int], shard_block_bytes: int,
                        region_bases: Sequence[int], blocking: bool = True) -> None:
    scatter_chunk_from_chip(src, [list(members)], block_ids, shard_block_bytes, region_bases, blocking)


__all__ = ["gather_tp_shards_to_chip", "scatter_chunk_from_chip", "pack_local_shards", "unpack_local_shards"]
_ = _native
