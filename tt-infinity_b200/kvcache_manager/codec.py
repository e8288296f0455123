"""Chunk layout, blob format and key derivation of the connector side of the hot path.

Restates, for the B200 store, the pure-host helpers the reference connector uses around
Client.put / Client.get:

* `RawByteCodec`: chunk slot validation and the on-device chunk plans (header words, member
  region bases, block ids, value length) of lmcache_t3knic/t3knic_lmcache/tt_raw_byte.py
  (patch 0005 lines 12148-12365).
* `decode_chunk_layout`: slot_mapping -> per-DP block runs (tt_paged_slice.py, patch 0005
  lines 10842-10955).
* `hash_layer_key`: the fixed-length per-layer wire key (tt_kv_serde.py, patch 0005 lines
  6955-6972).
* `chained_block_hashes`: 64-bit chained prefix-block hashes for the paged-block path.
"""

from __future__ import annotations

import hashlib
from dataclasses import dataclass
from typing import Any, Optional, Sequence, Tuple

import numpy as np

MAGIC = 0x524B564E
HEADER_ALIGN = 32
MAX_KEY_BYTES = 128


def header_words(count: int, sizes: Sequence[int]) -> list[int]:
    """[MAGIC, count, *sizes] zero padded to a multiple of 32 bytes."""
    words = [MAGIC, int(count)] + [int(s) for s in sizes]
    while (4 * len(words)) % HEADER_ALIGN:
        words.append(0)
    return words


class RawByteCodec:
    """Chunk geometry of a (dp, tp)-sharded paged cache, one chunk = whole cache blocks."""

    def __init__(self, *, tp_size: int, dp_size: int, block_size: int, blocks_per_dp: int,
                 shard_block_bytes: int) -> None:
        self.tp_size = int(tp_size)
        self.dp_size = int(dp_size)
        self.block_size = int(block_size)
        self.blocks_per_dp = int(blocks_per_dp)
        self.shard_block_bytes = int(shard_block_bytes)
        self.block_bytes = self.shard_block_bytes * self.tp_size

    def _chunk_slots(self, slot_mapping_slice: Any) -> list[int]:
        slots = [int(s) for s in (slot_mapping_slice.tolist() if hasattr(slot_mapping_slice, "tolist")
                                  else slot_mapping_slice)]
        if not slots:
            raise ValueError("raw-byte codec: empty slot_mapping slice")
        first = slots[0]
        if first % self.block_size != 0:
            raise RuntimeError(
                "raw-byte codec: chunk does not start on a cache-block boundary "
                f"(first slot {first}, block_size {self.block_size})"
            )
        if any(s != first + i for i, s in enumerate(slots)):
            raise RuntimeError("raw-byte codec: chunk slots must be sequential within one DP group")
        return slots

    def _chunk_span(self, slot_mapping_slice: Any) -> tuple[int, int]:
        """_chunk_slots's checks (same errors) with numpy, returning (first slot, slot count): the
        batched restore needs only these: 5 us per 256-token chunk against 28 us for the Python loop
        over every slot (8-core host)."""
        a = slot_mapping_slice
        if hasattr(a, "detach"):  # a torch tensor (a CUDA one is read back once)
            a = a.detach().cpu().numpy()
        a = np.asarray(a).reshape(-1)
        if a.size == 0:
            raise ValueError("raw-byte codec: empty slot_mapping slice")
        first = int(a[0])
        if first % self.block_size != 0:
            raise RuntimeError(
                "raw-byte codec: chunk does not start on a cache-block boundary "
                f"(first slot {first}, block_size {self.block_size})"
            )
        if not np.array_equal(a, np.arange(first, first + a.size)):
            raise RuntimeError("raw-byte codec: chunk slots must be sequential within one DP group")
        return first, int(a.size)

    def _n_blocks(self, num_slots: int) -> int:
        return -(-int(num_slots) // self.block_size)

    def chunk_buffer_bytes(self, num_slots: int) -> int:
        return 2 * self._n_blocks(num_slots) * self.block_bytes

    def _local_blocks(self, slots: list[int]) -> Tuple[int, list[int]]:
        return self._local_blocks_of(slots[0], len(slots))

    def _local_blocks_of(self, first_slot: int, num_slots: int) -> Tuple[int, list[int]]:
        n_blocks = self._n_blocks(num_slots)
        first_block = first_slot // self.block_size
        dp, local_first = divmod(first_block, self.blocks_per_dp)
        if local_first + n_blocks > self.blocks_per_dp:
            raise RuntimeError(
                f"raw-byte codec: chunk blocks {local_first}..{local_first + n_blocks} cross the "
                f"{self.blocks_per_dp}-block DP group"
            )
        return dp, list(range(local_first, local_first + n_blocks))

    def _plan(self, kvcaches: Any, num_layers: int, block_ids: list[int], alloc: int) -> dict:
        n_layers = int(num_layers)
        words = header_words(n_layers, [2 * alloc] * n_layers)
        hdr = 4 * len(words)
        members, region_bases = [], []
        for layer in range(n_layers):
            k, v = kvcaches[layer]
            base = hdr + layer * 2 * alloc
            members += [k, v]
            region_bases += [base, base + alloc]
        return {
            "members": members,
            "region_bases": region_bases,
            "block_ids": block_ids,
            "header_words": words,
            "value_len": hdr + n_layers * 2 * alloc,
            "shard_block_bytes": self.shard_block_bytes,
            "n_layers": n_layers,
            "member_bytes": alloc,
        }

    def device_chunk_plan(self, kvcaches: Any, num_layers: int, slot_mapping_slice: Any) -> dict:
        dp, block_ids = self._local_blocks_of(*self._chunk_span(slot_mapping_slice))
        plan = self._plan(kvcaches, num_layers, block_ids, len(block_ids) * self.block_bytes)
        plan.update(rank_coords=[(dp, t) for t in range(self.tp_size)], dp=dp)
        return plan

    def device_shard_plan(self, kvcaches: Any, num_layers: int, slot_mapping_slice: Any, tp_rank: int) -> dict:
        if not 0 <= int(tp_rank) < self.tp_size:
            raise ValueError(f"raw-byte codec: tp_rank {tp_rank} outside 0..{self.tp_size - 1}")
        dp, block_ids = self._local_blocks_of(*self._chunk_span(slot_mapping_slice))
        plan = self._plan(kvcaches, num_layers, block_ids, len(block_ids) * self.shard_block_bytes)
        coord = (dp, int(tp_rank))
        plan.update(coord=coord, rank_coords=[coord], dp=dp, tp_rank=int(tp_rank),
                    shard_index=dp * self.tp_size + int(tp_rank))
        return plan


@dataclass(frozen=True)
class PagedChunkLayout:
    block_size: int
    dp_size: int
    per_dp_runs: Tuple[Tuple[Tuple[int, int], ...], ...]
    per_dp_intra_offsets: Tuple[Tuple[int, ...], ...]
    per_dp_chunk_positions: Tuple[Tuple[int, ...], ...]
    per_dp_local_blocks: Tuple[Tuple[int, ...], ...]
    tp_size: int = 1
    dp_axis: int = 0
    tp_axis: int = 1


def decode_chunk_layout(slot_mapping_slice: Sequence[int], block_size: int, *, dp_size: int = 1,
                        blocks_per_dp: Optional[int] = None, tp_size: int = 1, dp_axis: int = 0,
                        tp_axis: int = 1) -> PagedChunkLayout:
    """Group a chunk's slots per DP group into sorted contiguous block runs.

    Slots past the last DP group stay in the last group (offset from its base)."""
    if block_size <= 0:
        raise ValueError(f"block_size must be positive, got {block_size}")
    if dp_size <= 0:
        raise ValueError(f"dp_size must be positive, got {dp_size}")
    if dp_size > 1 and (blocks_per_dp is None or blocks_per_dp <= 0):
        raise ValueError(f"dp_size={dp_size} requires blocks_per_dp > 0, got {blocks_per_dp}")
    groups: list[list[Tuple[int, int, int]]] = [[] for _ in range(dp_size)]
    for pos, slot in enumerate(int(s) for s in slot_mapping_slice):
        if slot < 0:
            raise ValueError(f"negative slot {slot} at position {pos}")
        block, intra = divmod(slot, block_size)
        if dp_size == 1:
            dp, local = 0, block
        else:
            dp, local = divmod(block, blocks_per_dp)
            if dp >= dp_size:
                dp = dp_size - 1
                local = block - dp * blocks_per_dp
        groups[dp].append((local, intra, pos))
    runs, intra_offs, positions, locals_ = [], [], [], []
    for g in groups:
        g = sorted(g)
        uniq = sorted({t[0] for t in g})
        r: list[Tuple[int, int]] = []
        for b in uniq:
            if r and r[-1][1] == b:
                r[-1] = (r[-1][0], b + 1)
            else:
                r.append((b, b + 1))
        runs.append(tuple(r))
        intra_offs.append(tuple(t[1] for t in g))
        positions.append(tuple(t[2] for t in g))
        locals_.append(tuple(t[0] for t in g))
    return PagedChunkLayout(block_size, dp_size, tuple(runs), tuple(intra_offs), tuple(positions),
                            tuple(locals_), tp_size, dp_axis, tp_axis)


def hash_layer_key(chunk_key: str, layer_idx: int, component: str = "kv") -> str:
    """64-hex-character blake2b-256 digest of "{chunk_key}:{layer_idx}:{component}"."""
    digest = hashlib.blake2b(f"{chunk_key}:{layer_idx}:{component}".encode("utf-8"), digest_size=32).hexdigest()
    assert len(digest) <= MAX_KEY_BYTES
    return digest


_M64 = (1 << 64) - 1


def mix64(x: int) -> int:
    """splitmix64 finaliser (Steele, Lea, Flood 2014)."""
    x &= _M64
    x = ((x ^ (x >> 30)) * 0xBF58476D1CE4E5B9) & _M64
    x = ((x ^ (x >> 27)) * 0x94D049BB133111EB) & _M64
    return x ^ (x >> 31)


def chained_block_hashes(seed: int, n_blocks: int, block_tokens: Optional[Sequence[Sequence[int]]] = None,
                         parent: int = 0) -> list[int]:
    """64-bit chained prefix-block hashes h_i = mix64(h_{i-1} ^ mix64(seed + i) ^ content_i).

    A block's key depends on every earlier block of the prefix, so two prompts share keys exactly
    on their common block-aligned prefix. `block_tokens[i]` (if given) contributes its tokens."""
    out = []
    h = parent & _M64
    for i in range(n_blocks):
        content = 0
        if block_tokens is not None:
            for t in block_tokens[i]:
                content = mix64(content ^ (int(t) & _M64))
        h = mix64(h ^ mix64((seed + i) & _M64) ^ content)
        if h == 0:
            h = 1
        out.append(h)
    return out
