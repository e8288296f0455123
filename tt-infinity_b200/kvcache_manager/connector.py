"""LMCache connector layer over the B200 store, for vLLM CUDA paged KV caches.

The B200 counterparts of the reference's LMCache connector triplet (patch 0005):

* `KVCacheClient`     -- the device-path subset of ``TTKVCacheClient`` (P5:7061-10706): the
  pending-op registries that carry a chunk across the LMCache API boundary, ``exists`` / ``delete``
  of a chunk, and ``put_chunk_device`` / ``get_chunk_device`` (P5:9653-9760): one gather of the
  chunk's blocks into a blob and one ``Client.put`` of it, or one ``Client.get`` and one scatter.
  The key is ``hash_layer_key(chunk_key, tp_rank, "raw")`` and the blob is the raw-byte chunk
  layout (header ``[MAGIC, n_layers, layer bytes...]``, then per layer the K region and the V
  region, block-major), so a value written by the reference's device path decodes the same.
* `GPUConnector`      -- ``TTGPUConnector`` (P5:6195-6903): ``from_gpu`` records the chunk's
  slot mapping against the MemoryObj placeholder, ``to_gpu`` restores the chunk the matching
  ``get`` announced.
* `RemoteConnector`   -- ``TTRemoteConnector`` (P5:12425-12728): ``exists``, ``put`` (performs
  the store of the chunk ``from_gpu`` recorded), ``get`` (returns a placeholder and records the
  key for ``to_gpu``), ``batched_*``, ``list``, ``remove_sync``.

LMCache itself is not a dependency: keys are anything with ``to_string()`` (LMCache's
``CacheEngineKey``), MemoryObj placeholders are any objects, and `RemoteConnector` takes the
allocator callable LMCache's ``LocalCPUBackend.allocate`` provides. One connector serves one vLLM
worker (one GPU, one tensor-parallel rank): caches are vLLM's per-layer
``[2, num_blocks, block_size, num_kv_heads, head_dim]`` tensors (`kv_caches_from_vllm`).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Callable, Dict, List, Optional, Sequence

from . import codec, ops
from ._facade import Client


def _stream_of(t: Any) -> int:
    """Raw handle of the current stream on the tensor's device."""
    import torch

    return torch.cuda.current_stream(t.device).cuda_stream


def kv_caches_from_vllm(kv_caches: Sequence[Any]) -> list:
    """vLLM CUDA caches (per layer ``[2, num_blocks, block_size, heads, head_dim]``) as per-layer
    ``(K, V)`` tensors whose first dimension is the block index (views, no copy)."""
    out = []
    for i, t in enumerate(kv_caches):
        if t.dim() != 5 or t.shape[0] != 2:
            raise ValueError(
                f"kv cache of layer {i} has shape {tuple(t.shape)}; expected [2, num_blocks, block_size, "
                "num_kv_heads, head_dim] (the K/V-major layout; a block-major [num_blocks, 2, ...] cache "
                "interleaves K and V inside every block and is not a pair of block arrays)")
        if not t.is_contiguous():
            raise ValueError(f"kv cache of layer {i} must be contiguous")
        out.append((t[0], t[1]))
    return out


def raw_codec_for(kvcaches: Sequence[Any], block_size: int) -> codec.RawByteCodec:
    """The raw-byte chunk codec of one worker's caches (per-layer (K, V), block index first)."""
    k = kvcaches[0][0]
    shard_block_bytes = k[0].numel() * k.element_size()
    if k.shape[1] != block_size:
        raise ValueError(f"cache blocks hold {k.shape[1]} tokens, not block_size {block_size}")
    return codec.RawByteCodec(tp_size=1, dp_size=1, block_size=block_size, blocks_per_dp=int(k.shape[0]),
                              shard_block_bytes=shard_block_bytes)


@dataclass
class ChunkRef:
    """What ``from_gpu`` hands to ``put`` (the reference's KVChunkRef): the caches and the chunk's
    slot mapping."""

    kvcaches: Any
    slot_mapping_slice: Any
    num_layers: int


class KVCacheClient:
    """Chunk store of one vLLM worker over a `Client`; holds the pending-op registries."""

    def __init__(self, client: Client, raw_codec: codec.RawByteCodec, tp_rank: int = 0) -> None:
        self.client = client
        self.raw_codec = raw_codec
        self.tp_rank = int(tp_rank)
        self._pending_send: Dict[int, ChunkRef] = {}
        self._pending_get: Dict[int, Any] = {}
        self._blob = None
        self.stats = {"puts": 0, "gets": 0, "get_misses": 0, "put_bytes": 0, "get_bytes": 0}

    # ---- pending-op registries (the MemoryObj's id links from_gpu/put and get/to_gpu)
    def record_pending_send(self, mo_id: int, ref: ChunkRef) -> None:
        self._pending_send[mo_id] = ref

    def pop_pending_send(self, mo_id: int) -> Optional[ChunkRef]:
        return self._pending_send.pop(mo_id, None)

    def record_pending_get(self, memory_obj: Any, key: Any) -> None:
        self._pending_get[id(memory_obj)] = key

    def pop_pending_get(self, mo_id: int) -> Optional[Any]:
        return self._pending_get.pop(mo_id, None)

    # ---- keys and the wire
    def raw_key(self, key: str) -> bytes:
        """The store key of this rank's shard of a chunk (the reference's _raw_shard_key / _raw_wire_key)."""
        return codec.hash_layer_key(key, self.tp_rank, "raw").encode("utf-8")

    def wire_uses_device_path(self) -> bool:
        return True

    def exists(self, key: str) -> bool:
        return self.client.exists(self.raw_key(key))

    def delete(self, key: str) -> bool:
        return self.client.delete(self.raw_key(key))

    def _blob_tensor(self, nbytes: int, device: Any):
        import torch

        words = (nbytes + 3) // 4
        if self._blob is None or self._blob.numel() < words or self._blob.device != device:
            self._blob = torch.empty(words, dtype=torch.int32, device=device)
        return self._blob

    def _plan(self, kvcaches: Any, num_layers: int, slot_mapping_slice: Any) -> dict:
        return self.raw_codec.device_shard_plan(kvcaches, num_layers, slot_mapping_slice, self.tp_rank)

    def put_chunk_device(self, key: str, kvcaches: Any, num_layers: int, slot_mapping_slice: Any) -> bool:
        """Gather the chunk's blocks from the live caches into one blob and store it."""
        plan = self._plan(kvcaches, num_layers, slot_mapping_slice)
        members = plan["members"]
        blob = self._blob_tensor(int(plan["value_len"]), members[0].device)
        ops.pack_local_shards(members, blob, plan["block_ids"], int(plan["shard_block_bytes"]),
                              plan["region_bases"], plan["header_words"], blocking=False)
        self.client.put(self.raw_key(key), blob, int(plan["value_len"]))
        self.stats["puts"] += 1
        self.stats["put_bytes"] += int(plan["value_len"])
        return True

    def get_chunk_device(self, key: str, kvcaches: Any, num_layers: int, slot_mapping_slice: Any) -> bool:
        """Restore one chunk into the live caches; False on a miss. The reference gets the chunk's
        blob and scatters it (P5:9710-9760); here the chunk's rows go from the store straight into
        the caches (get_chunks_device), one copy instead of two."""
        return self.get_chunks_device([key], kvcaches, num_layers, [slot_mapping_slice])[0]

    def get_chunks_device(self, keys: Sequence[str], kvcaches: Any, num_layers: int,
                          slot_mapping_slices: Sequence[Any]) -> list[bool]:
        """Restore several chunks in one store call: every chunk's rows go from where its value
        lives straight into the caches, all layers in one fill launch (kvs_restore_chunks).
        The reference fetches the chunks and fills one layer per call (TTGPUConnector's batched
        restore, P5:6780-6870 with _paged_fill_layer_coalesced, P5:11563-11770). Returns found per
        chunk; a missing chunk leaves its blocks untouched."""
        import ctypes as C

        import numpy as np

        from . import _native

        n = len(keys)
        if n == 0:
            return []
        if len(slot_mapping_slices) != n:
            raise ValueError("get_chunks_device: one slot mapping slice per key")
        k0 = kvcaches[0][0]
        bs = int(k0.shape[1])
        if bs != self.raw_codec.block_size:
            raise ValueError(f"cache blocks hold {bs} tokens, not block_size {self.raw_codec.block_size}")
        row_bytes = int(k0[0, 0].numel() * k0.element_size())
        spans = [self.raw_codec._chunk_span(sl) for sl in slot_mapping_slices]
        tokens = np.array([cnt for _, cnt in spans], np.uint32)
        max_blocks = int(max(-(-int(t) // bs) for t in tokens))
        # a chunk starts on a block boundary with sequential slots: its blocks follow its first one
        page = np.zeros((n, max_blocks), np.int32)
        for i, (first, cnt) in enumerate(spans):
            nb = -(-cnt // bs)
            page[i, :nb] = np.arange(first // bs, first // bs + nb, dtype=np.int32)
        starts = np.zeros(n, np.int32)
        raw = [self.raw_key(k) for k in keys]
        key_arr = (C.c_void_p * n)(*[C.cast(C.c_char_p(b), C.c_void_p) for b in raw])
        lens = np.array([len(b) for b in raw], np.uint32)
        ks = (C.c_void_p * num_layers)(*[kvcaches[l][0].data_ptr() for l in range(num_layers)])
        vs = (C.c_void_p * num_layers)(*[kvcaches[l][1].data_ptr() for l in range(num_layers)])
        found = np.zeros(n, np.uint8)
        _native.check(_native.load().kvs_restore_chunks(
            self.client._handle(), n, key_arr, lens.ctypes.data_as(_native._u32p),
            tokens.ctypes.data_as(_native._u32p), num_layers, ks, vs, int(k0.shape[0]), bs, row_bytes,
            page.ctypes.data_as(C.POINTER(C.c_int32)), max_blocks, starts.ctypes.data_as(C.POINTER(C.c_int32)),
            found.ctypes.data_as(_native._u8p), C.c_void_p(_stream_of(k0))))
        hits = int(found.sum())
        payload = int(sum(2 * num_layers * int(t) * row_bytes for t, f in zip(tokens, found) if f))
        self.stats["gets"] += hits
        self.stats["get_misses"] += n - hits
        self.stats["get_bytes"] += payload
        return [bool(f) for f in found]

    def wait_put_done(self, key: str) -> None:
        """Puts land before Client.put returns (write-through finishes asynchronously)."""


class GPUConnector:
    """``from_gpu`` / ``to_gpu`` between LMCache placeholders and vLLM's CUDA paged caches."""

    def __init__(self, client: KVCacheClient, num_layers: int, block_size: int) -> None:
        self.client = client
        self.num_layers = int(num_layers)
        self.block_size = int(block_size)
        self.kvcaches = None
        self.load_misses = 0

    def initialize_kvcaches_ptr(self, **kwargs: Any) -> None:
        if self.kvcaches is None and kwargs.get("kvcaches") is not None:
            caches = kwargs["kvcaches"]
            self.kvcaches = kv_caches_from_vllm(caches) if hasattr(caches[0], "dim") else list(caches)

    def _slice(self, start: int, end: int, kwargs: dict, op: str):
        if kwargs.get("kvcaches") is None:
            raise ValueError(f"'kvcaches' must be provided in kwargs for {op}")
        if kwargs.get("slot_mapping") is None:
            raise ValueError(f"'slot_mapping' must be provided in kwargs for {op}")
        self.initialize_kvcaches_ptr(**kwargs)
        return kwargs["slot_mapping"][start:end]

    def from_gpu(self, memory_obj: Any, start: int, end: int, **kwargs: Any) -> None:
        """Record the chunk for the matching ``RemoteConnector.put``; memory_obj is not written."""
        sl = self._slice(start, end, kwargs, "from_gpu")
        self.client.record_pending_send(id(memory_obj), ChunkRef(self.kvcaches, sl, self.num_layers))

    def to_gpu(self, memory_obj: Any, start: int, end: int, **kwargs: Any) -> None:
        """Restore the chunk ``RemoteConnector.get`` announced for this placeholder."""
        sl = self._slice(start, end, kwargs, "to_gpu")
        key = self.client.pop_pending_get(id(memory_obj))
        if key is None:
            raise RuntimeError(
                f"GPUConnector.to_gpu: no pending-get entry for id(memory_obj)={id(memory_obj)}; "
                "RemoteConnector.get must run before to_gpu")
        if not self.client.get_chunk_device(key.to_string(), self.kvcaches, self.num_layers, sl):
            self.load_misses += 1

    def batched_from_gpu(self, memory_objs: List[Any], starts: List[int], ends: List[int], **kwargs: Any) -> None:
        for mo, s, e in zip(memory_objs, starts, ends):
            self.from_gpu(mo, s, e, **kwargs)

    def batched_to_gpu(self, memory_objs: List[Any], starts: List[int], ends: List[int], **kwargs: Any) -> None:
        """Restore every announced chunk in one store call (KVCacheClient.get_chunks_device): one
        fill launch writes all chunks into all layers, reading each chunk where the store holds it."""
        sm = kwargs.get("slot_mapping")
        if sm is not None and getattr(getattr(sm, "device", None), "type", "cpu") != "cpu":
            kwargs = dict(kwargs, slot_mapping=sm.cpu())  # one device-to-host read for the whole batch
        keys, slices = [], []
        for mo, s, e in zip(memory_objs, starts, ends):
            sl = self._slice(s, e, kwargs, "batched_to_gpu")
            key = self.client.pop_pending_get(id(mo))
            if key is None:
                raise RuntimeError(
                    f"GPUConnector.batched_to_gpu: no pending-get entry for id(memory_obj)={id(mo)}; "
                    "RemoteConnector.get must run before batched_to_gpu")
            keys.append(key.to_string())
            slices.append(sl)
        found = self.client.get_chunks_device(keys, self.kvcaches, self.num_layers, slices)
        self.load_misses += sum(1 for f in found if not f)

    def get_shape(self, num_tokens: int):
        """Shape of one chunk as LMCache sizes it: [2, layers, tokens, hidden] of this rank."""
        import torch

        k = self.kvcaches[0][0] if self.kvcaches else None
        hidden = int(k.shape[-1] * k.shape[-2]) if k is not None else 0
        return torch.Size([2, self.num_layers, int(num_tokens), hidden])


class RemoteConnector:
    """LMCache's remote-storage side: exists / put / get / list / remove of chunk keys."""

    def __init__(self, client: KVCacheClient, allocate: Callable[..., Any], meta_shape: Any, meta_dtype: Any,
                 meta_fmt: Any = None) -> None:
        self.client = client
        self.allocate = allocate
        self.meta_shape, self.meta_dtype, self.meta_fmt = meta_shape, meta_dtype, meta_fmt

    async def exists(self, key: Any) -> bool:
        return self.client.exists(key.to_string())

    def exists_sync(self, key: Any) -> bool:
        return self.client.exists(key.to_string())

    async def put(self, key: Any, memory_obj: Any) -> None:
        """Store the chunk ``from_gpu`` recorded for memory_obj (no entry: already in flight)."""
        info = self.client.pop_pending_send(id(memory_obj))
        if info is None:
            return
        if not isinstance(info, ChunkRef):
            raise TypeError(f"RemoteConnector.put expected a ChunkRef in the pending-send registry, got "
                            f"{type(info).__name__}")
        key_str = key.to_string()
        self.client.put_chunk_device(key_str, info.kvcaches, info.num_layers, info.slot_mapping_slice)
        self.client.wait_put_done(key_str)

    async def batched_put(self, keys: List[Any], memory_objs: List[Any]) -> None:
        for key, mo in zip(keys, memory_objs):
            await self.put(key, mo)

    def support_batched_put(self) -> bool:
        return True

    async def get(self, key: Any) -> Optional[Any]:
        """A placeholder MemoryObj whose chunk ``to_gpu`` fetches; None if the allocator is full."""
        memory_obj = self.allocate(self.meta_shape, self.meta_dtype, fmt=self.meta_fmt)
        if memory_obj is None:
            return None
        self.client.record_pending_get(memory_obj, key)
        return memory_obj

    async def batched_get(self, keys: List[Any]) -> List[Optional[Any]]:
        return [await self.get(k) for k in keys]

    def support_batched_get(self) -> bool:
        return True

    async def list(self) -> List[str]:
        """The store protocol has put / get / exists / delete only: nothing to enumerate."""
        return []

    def remove_sync(self, key: Any) -> bool:
        return self.client.delete(key.to_string())

    async def close(self) -> None:
        pass
