"""Chunk gather / scatter ops over paged KV members, and the token-granular paged fill (torch
CUDA tensors).

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


def paged_fill_cache_varlen(k_fill_value: Any, v_fill_value: Any, cu_seqlens: Any, page_table: Any,
                            start_positions: Any, cache_k: Any, cache_v: Any, out_of_range: Any = None):
    """Fill packed K/V of several requests into a paged KV cache, one token at a time.

    The B200 counterpart of ttnn.experimental.moreh_paged_fill_cache_varlen (patch 0002: kernels at
    lines 106-421, validation at 441-545), with its argument order and checks:
    k_fill_value / v_fill_value [1, num_kv_heads, total_tokens, head_dim]; cache_k / cache_v
    [max_num_blocks, num_kv_heads, block_size, head_dim] of the same dtype; cu_seqlens int32
    [batch_size + 1] (-1 after the valid offsets); page_table int32 [batch_size,
    max_num_blocks_per_seq]; start_positions int32 [batch_size]; every tensor a contiguous CUDA
    tensor on one device. Page-table entries <= 0 skip a token (vLLM's null block 0, -1 for unused
    slots). out_of_range: optional int32 CUDA tensor of one element, incremented for tokens skipped
    because their position or block is out of range. Asynchronous on the current stream; returns
    (cache_k, cache_v) as the reference's device operation does."""
    _check_fill(k_fill_value, v_fill_value, cu_seqlens, page_table, start_positions, cache_k, cache_v, out_of_range)
    torch = _torch()
    dev = k_fill_value.device
    heads, total, dim = k_fill_value.shape[1], k_fill_value.shape[2], k_fill_value.shape[3]
    P = C.c_void_p
    check(load().kvs_paged_fill_varlen(
        P(k_fill_value.data_ptr()), P(v_fill_value.data_ptr()), heads, total, dim * k_fill_value.element_size(),
        P(cu_seqlens.data_ptr()), page_table.shape[0], P(page_table.data_ptr()), page_table.shape[1],
        P(start_positions.data_ptr()), P(cache_k.data_ptr()), P(cache_v.data_ptr()), cache_k.shape[0],
        cache_k.shape[2], P(out_of_range.data_ptr() if out_of_range is not None else None),
        P(torch.cuda.current_stream(dev).cuda_stream)))
    return cache_k, cache_v


def _check_fill(k_fill_value, v_fill_value, cu_seqlens, page_table, start_positions, cache_k, cache_v,
                out_of_range) -> None:
    """The reference's validation of one fill (patch 0002 lines 441-545)."""
    torch = _torch()
    ts = {"k_fill_value": k_fill_value, "v_fill_value": v_fill_value, "cu_seqlens": cu_seqlens,
          "page_table": page_table, "start_positions": start_positions, "cache_k": cache_k, "cache_v": cache_v}
    for name, t in ts.items():
        if not isinstance(t, torch.Tensor) or t.device.type != "cuda":
            raise RuntimeError(f"{name} must be on device!")
        if not t.is_contiguous():
            raise RuntimeError(f"{name} must be contiguous")
    dev = k_fill_value.device
    if any(t.device != dev for t in ts.values()):
        raise RuntimeError("All tensors must be on the same device!")
    if k_fill_value.dtype != cache_k.dtype:
        raise RuntimeError(f"k_fill_value dtype ({k_fill_value.dtype}) must match cache_k dtype ({cache_k.dtype})")
    if v_fill_value.dtype != cache_v.dtype:
        raise RuntimeError(f"v_fill_value dtype ({v_fill_value.dtype}) must match cache_v dtype ({cache_v.dtype})")
    if k_fill_value.dim() != 4 or cache_k.dim() != 4:
        raise RuntimeError("k_fill_value and cache_k must be 4-D")
    if k_fill_value.shape[0] != 1:
        raise RuntimeError(f"k_fill_value first dim must be 1, got {k_fill_value.shape[0]}")
    if v_fill_value.shape[0] != 1:
        raise RuntimeError(f"v_fill_value first dim must be 1, got {v_fill_value.shape[0]}")
    if k_fill_value.shape[-1] != cache_k.shape[-1]:
        raise RuntimeError("head_dim of k_fill_value must match cache_k")
    if v_fill_value.shape[-1] != cache_v.shape[-1]:
        raise RuntimeError("head_dim of v_fill_value must match cache_v")
    if k_fill_value.shape != v_fill_value.shape:
        raise RuntimeError("k_fill_value and v_fill_value must have the same shape")
    if cache_k.shape != cache_v.shape:
        raise RuntimeError("cache_k and cache_v must have the same shape")
    if k_fill_value.shape[1] != cache_k.shape[1]:
        raise RuntimeError("num_kv_heads of k_fill_value must match cache_k")
    for name in ("cu_seqlens", "page_table", "start_positions"):
        if ts[name].dtype != torch.int32:
            raise RuntimeError(f"{name} must be INT32")
    if page_table.dim() != 2:
        raise RuntimeError("page_table must be [batch_size, max_num_blocks_per_seq]")
    if page_table.shape[1] > cache_k.shape[0]:
        raise RuntimeError(f"max_num_blocks_per_seq ({page_table.shape[1]}) must be <= max_num_blocks ({cache_k.shape[0]})")
    if start_positions.shape[0] != page_table.shape[0]:
        raise RuntimeError(f"start_positions size ({start_positions.shape[0]}) must match batch_size ({page_table.shape[0]})")
    if cu_seqlens.numel() != page_table.shape[0] + 1:
        raise RuntimeError(f"cu_seqlens must hold batch_size + 1 = {page_table.shape[0] + 1} entries")
    if out_of_range is not None and (out_of_range.dtype != torch.int32 or out_of_range.device != dev):
        raise RuntimeError("out_of_range must be an int32 tensor on the fill's device")


def paged_fill_cache_varlen_layers(k_fill_values: Sequence[Any], v_fill_values: Sequence[Any], cu_seqlens: Any,
                                   page_table: Any, start_positions: Any, cache_ks: Sequence[Any],
                                   cache_vs: Sequence[Any], out_of_range: Any = None):
    """paged_fill_cache_varlen for several layers that share the requests and page tables, in one
    launch per 64 layers (no counterpart in the reference, which fills one layer per call). Layer
    l fills cache_ks[l] / cache_vs[l] from k_fill_values[l] / v_fill_values[l], every layer
    validated as the single-layer op validates it and of the first layer's shapes. Each layer's
    result equals the single-layer fill; out_of_range counts each skipped token once."""
    torch = _torch()
    n = len(k_fill_values)
    if not (len(v_fill_values) == len(cache_ks) == len(cache_vs) == n):
        raise RuntimeError("k_fill_values, v_fill_values, cache_ks and cache_vs must name the same layers")
    if n == 0:
        return cache_ks, cache_vs
    k0, c0 = k_fill_values[0], cache_ks[0]
    for l in range(n):
        _check_fill(k_fill_values[l], v_fill_values[l], cu_seqlens, page_table, start_positions, cache_ks[l],
                    cache_vs[l], out_of_range)
        if k_fill_values[l].shape != k0.shape or cache_ks[l].shape != c0.shape or cache_ks[l].dtype != c0.dtype:
            raise RuntimeError(f"layer {l}: every layer must have the first layer's shapes and dtype")
        if k_fill_values[l].device != k0.device:
            raise RuntimeError("All tensors must be on the same device!")
    heads, total, dim = k0.shape[1], k0.shape[2], k0.shape[3]
    P = C.c_void_p
    arr = lambda ts: (P * n)(*[t.data_ptr() for t in ts])
    check(load().kvs_paged_fill_varlen_layers(
        n, arr(k_fill_values), arr(v_fill_values), heads, total, dim * k0.element_size(),
        P(cu_seqlens.data_ptr()), page_table.shape[0], P(page_table.data_ptr()), page_table.shape[1],
        P(start_positions.data_ptr()), arr(cache_ks), arr(cache_vs), c0.shape[0], c0.shape[2],
        P(out_of_range.data_ptr() if out_of_range is not None else None),
        P(torch.cuda.current_stream(k0.device).cuda_stream)))
    return cache_ks, cache_vs
