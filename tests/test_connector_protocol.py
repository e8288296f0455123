"""The LMCache connector glue of kvcache_manager.connector on CPU, with a fake chunk store: the
pending-send / pending-get registries that link from_gpu -> put and get -> to_gpu (the
reference's TTGPUConnector / TTRemoteConnector contract, patch 0005), the error paths, and the
store key (hash_layer_key(chunk_key, tp_rank, "raw"))."""

import asyncio

import pytest

from kvcache_manager import codec
from kvcache_manager.connector import ChunkRef, GPUConnector, KVCacheClient, RemoteConnector


class Key:
    def __init__(self, s):
        self.s = s

    def to_string(self):
        return self.s


class FakeStoreClient(KVCacheClient):
    """KVCacheClient whose chunk store is a dict: records what put/get were asked to move."""

    def __init__(self):
        super().__init__(client=None, raw_codec=None)
        self.store = {}
        self.restored = []
        self.restore_calls = []

    def exists(self, key):
        return self.raw_key(key) in self.store

    def delete(self, key):
        return self.store.pop(self.raw_key(key), None) is not None

    def put_chunk_device(self, key, kvcaches, num_layers, slot_mapping_slice):
        self.store[self.raw_key(key)] = (list(slot_mapping_slice), num_layers)
        return True

    def get_chunk_device(self, key, kvcaches, num_layers, slot_mapping_slice):
        hit = self.raw_key(key) in self.store
        if hit:
            self.restored.append((key, list(slot_mapping_slice)))
        return hit

    def get_chunks_device(self, keys, kvcaches, num_layers, slot_mapping_slices):
        self.restore_calls.append(list(keys))
        return [self.get_chunk_device(k, kvcaches, num_layers, sl) for k, sl in zip(keys, slot_mapping_slices)]


def make():
    client = FakeStoreClient()
    gpu = GPUConnector(client, num_layers=2, block_size=16)
    remote = RemoteConnector(client, allocate=lambda shape, dtype, fmt=None: object(), meta_shape=(1,), meta_dtype=None)
    return client, gpu, remote


def test_store_then_restore_through_the_registries():
    client, gpu, remote = make()
    caches = [("k0", "v0"), ("k1", "v1")]
    slots = list(range(64, 128))
    mo = object()
    gpu.from_gpu(mo, 16, 48, kvcaches=caches, slot_mapping=slots)
    asyncio.run(remote.put(Key("chunk-a"), mo))
    assert remote.exists_sync(Key("chunk-a")) and asyncio.run(remote.exists(Key("chunk-a")))
    assert client.store[codec.hash_layer_key("chunk-a", 0, "raw").encode()] == (slots[16:48], 2)
    ph = asyncio.run(remote.get(Key("chunk-a")))
    gpu.to_gpu(ph, 0, 32, kvcaches=caches, slot_mapping=slots)
    assert client.restored == [("chunk-a", slots[:32])]
    assert asyncio.run(remote.list()) == []
    assert remote.remove_sync(Key("chunk-a")) and not remote.exists_sync(Key("chunk-a"))


def test_batched_paths_and_a_put_without_a_recorded_chunk():
    client, gpu, remote = make()
    caches = [("k0", "v0"), ("k1", "v1")]
    slots = list(range(256))
    mos = [object() for _ in range(3)]
    gpu.batched_from_gpu(mos, [0, 64, 128], [64, 128, 192], kvcaches=caches, slot_mapping=slots)
    keys = [Key(f"c{i}") for i in range(3)]
    asyncio.run(remote.batched_put(keys, mos))
    asyncio.run(remote.put(Key("dup"), object()))  # no pending send (already in flight): a no-op
    assert sorted(client.store) == sorted(client.raw_key(f"c{i}") for i in range(3))
    phs = asyncio.run(remote.batched_get(keys))
    gpu.batched_to_gpu(phs, [0, 64, 128], [64, 128, 192], kvcaches=caches, slot_mapping=slots)
    assert [k for k, _ in client.restored] == ["c0", "c1", "c2"]
    assert client.restore_calls == [["c0", "c1", "c2"]]  # one store call restores the whole batch
    assert gpu.load_misses == 0
    assert remote.support_batched_put() and remote.support_batched_get()


def test_error_paths():
    client, gpu, remote = make()
    with pytest.raises(ValueError, match="kvcaches"):
        gpu.from_gpu(object(), 0, 16, slot_mapping=[0] * 16)
    with pytest.raises(ValueError, match="slot_mapping"):
        gpu.to_gpu(object(), 0, 16, kvcaches=[("k", "v")])
    with pytest.raises(RuntimeError, match="no pending-get"):
        gpu.to_gpu(object(), 0, 16, kvcaches=[("k", "v")], slot_mapping=[0] * 16)
    client.record_pending_send(id(mo := object()), "not a ref")
    with pytest.raises(TypeError, match="ChunkRef"):
        asyncio.run(remote.put(Key("x"), mo))
    full = RemoteConnector(client, allocate=lambda *a, **k: None, meta_shape=(1,), meta_dtype=None)
    assert asyncio.run(full.get(Key("y"))) is None  # allocator exhausted: no placeholder, nothing recorded
    assert client.pop_pending_get(0) is None


def test_store_key_per_tensor_parallel_rank():
    a = KVCacheClient(client=None, raw_codec=None, tp_rank=0)
    b = KVCacheClient(client=None, raw_codec=None, tp_rank=3)
    assert a.raw_key("k") == codec.hash_layer_key("k", 0, "raw").encode()
    assert b.raw_key("k") == codec.hash_layer_key("k", 3, "raw").encode() != a.raw_key("k")
    assert ChunkRef(None, [1], 2).num_layers == 2
