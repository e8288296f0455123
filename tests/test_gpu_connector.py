"""The LMCache connector layer on a B200 with vLLM-layout CUDA caches: from_gpu -> put stores each
chunk under hash_layer_key(key, 0, "raw") as the raw-byte chunk blob (checked byte for byte against
the oracle's gather of the same blocks with the reference's header), the caches are wiped, and
get -> to_gpu restores every chunk bit-exactly; misses are counted, not fatal."""

import asyncio

import numpy as np
import pytest
import torch

from kvcache_manager import Client, Server, codec
from kvcache_manager.connector import GPUConnector, KVCacheClient, RemoteConnector, kv_caches_from_vllm, raw_codec_for
from oracle import kvs_oracle as O

pytestmark = pytest.mark.gpu


class Key:
    def __init__(self, s):
        self.s = s

    def to_string(self):
        return self.s


def test_connector_store_wipe_restore_round_trip():
    layers, nb, bs, heads, dim = 3, 64, 16, 4, 64
    g = torch.Generator(device="cuda")
    g.manual_seed(4)
    vllm_caches = [torch.empty((2, nb, bs, heads, dim), dtype=torch.bfloat16, device="cuda").normal_(generator=g)
                   for _ in range(layers)]
    caches = kv_caches_from_vllm(vllm_caches)
    raw = raw_codec_for(caches, bs)
    server = Server(0, max_keys=64, heap_bytes=64 << 20, host_pool_bytes=64 << 20)
    client = Client(0, server)
    kc = KVCacheClient(client, raw)
    gpu = GPUConnector(kc, num_layers=layers, block_size=bs)
    remote = RemoteConnector(kc, allocate=lambda shape, dtype, fmt=None: object(), meta_shape=(1,), meta_dtype=None)
    try:
        # a request of 160 tokens on blocks 8..17 (vLLM slots = block * bs + offset); 64-token chunks
        slots = torch.arange(8 * bs, 18 * bs, device="cuda")
        chunks = [(0, 64), (64, 128), (128, 160)]
        keys = [Key(f"req0@chunk{i}") for i in range(len(chunks))]
        before = [t.clone() for t in vllm_caches]
        mos = [object() for _ in chunks]
        gpu.batched_from_gpu(mos, [s for s, _ in chunks], [e for _, e in chunks], kvcaches=vllm_caches,
                             slot_mapping=slots)
        asyncio.run(remote.batched_put(keys, mos))
        assert all(remote.exists_sync(k) for k in keys) and not remote.exists_sync(Key("never"))
        # the stored value is the reference's raw chunk blob of those blocks
        host = [t.view(torch.uint8).reshape(-1).cpu().numpy() for p in caches for t in p]
        plan = raw.device_shard_plan(caches, layers, slots[0:64].tolist(), 0)
        want = O.gather([host], [plan["shard_block_bytes"]] * len(host), plan["block_ids"], plan["region_bases"],
                        plan["header_words"], plan["value_len"])
        out = torch.zeros(plan["value_len"], dtype=torch.uint8, device="cuda")
        assert client.get(codec.hash_layer_key("req0@chunk0", 0, "raw").encode(), out)
        assert np.array_equal(out.cpu().numpy(), want)
        # wipe the request's blocks, then restore through get -> to_gpu
        for t in vllm_caches:
            t[:, 8:18].zero_()
        phs = asyncio.run(remote.batched_get(keys))
        gpu.batched_to_gpu(phs, [s for s, _ in chunks], [e for _, e in chunks], kvcaches=vllm_caches,
                           slot_mapping=slots)
        torch.cuda.synchronize()
        for a, b in zip(vllm_caches, before):
            assert torch.equal(a.view(torch.int16), b.view(torch.int16))
        # a chunk nobody stored: counted as a load miss, caches untouched
        ph = asyncio.run(remote.get(Key("absent")))
        gpu.to_gpu(ph, 0, 64, kvcaches=vllm_caches, slot_mapping=slots)
        assert gpu.load_misses == 1 and kc.stats["get_misses"] == 1
        assert remote.remove_sync(keys[0]) and not remote.exists_sync(keys[0])
    finally:
        client.close()
        server.close()


def _caches(layers, nb, bs, heads, dim, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return [torch.empty((2, nb, bs, heads, dim), dtype=torch.bfloat16, device="cuda").normal_(generator=g)
            for _ in range(layers)]


def test_batched_restore_partial_chunk_host_tier_and_evictions_match_the_oracle_fill():
    """kvs_restore_chunks through GPUConnector.batched_to_gpu: a chunk that ends inside a block
    writes only its tokens (token-granular, as moreh_paged_fill_cache_varlen), chunks whose values
    sit in the host tier are admitted on the way, and a slab of two values makes the admissions of
    one call evict each other (those chunks are read from their host copies). Every restored cache
    equals the oracle's fill of the stored rows."""
    layers, nb, bs, heads, dim = 4, 48, 16, 2, 64
    vllm_caches = _caches(layers, nb, bs, heads, dim, 9)
    caches = kv_caches_from_vllm(vllm_caches)
    raw = raw_codec_for(caches, bs)
    row = heads * dim * 2
    # chunks of one request on blocks 4.. : 64 tokens (4 blocks), 64, and a 40-token tail (3 blocks)
    chunks = [(0, 64), (64, 128), (128, 168)]
    slots = torch.arange(4 * bs, 4 * bs + 168, device="cuda")
    vlen = raw.device_shard_plan(caches, layers, slots[0:64].tolist(), 0)["value_len"]
    units = -(-vlen // 4288)
    server = Server(0, max_keys=64, heap_bytes=2 * (1 << (units - 1).bit_length()) * 4288, host_pool_bytes=64 << 20)
    client = Client(0, server)
    kc = KVCacheClient(client, raw)
    gpu = GPUConnector(kc, num_layers=layers, block_size=bs)
    remote = RemoteConnector(kc, allocate=lambda shape, dtype, fmt=None: object(), meta_shape=(1,), meta_dtype=None)
    try:
        keys = [Key(f"req1@chunk{i}") for i in range(len(chunks))]
        mos = [object() for _ in chunks]
        gpu.batched_from_gpu(mos, [s for s, _ in chunks], [e for _, e in chunks], kvcaches=vllm_caches,
                             slot_mapping=slots)
        asyncio.run(remote.batched_put(keys, mos))
        client.flush()
        # the stored rows (the oracle's fill input): what the caches held when the chunks were put
        src = [t.clone() for t in vllm_caches]
        # the third put evicted the first chunk's device copy; send the second to the host tier too
        client.move_to_host(kc.raw_key(keys[1].to_string()))
        locs = [server.location(kc.raw_key(k.to_string()))[0] for k in keys]
        assert locs.count(1) >= 2, locs
        # clobber the request's blocks with a pattern the restore must overwrite exactly where it writes
        for t in vllm_caches:
            t[:, 4:15].fill_(7.0)
        clobbered = [t.clone() for t in vllm_caches]
        phs = asyncio.run(remote.batched_get(keys))
        gpu.batched_to_gpu(phs, [s for s, _ in chunks], [e for _, e in chunks], kvcaches=vllm_caches,
                           slot_mapping=slots)
        torch.cuda.synchronize()
        assert gpu.load_misses == 0
        # the oracle: token-granular fill of each chunk's stored rows into the clobbered caches
        cu = np.array([0] + [e for _, e in chunks], np.int32)
        pt = np.array([[4 + s // bs + b for b in range(4)] for s, _ in chunks], np.int32)
        sp = np.zeros(len(chunks), np.int32)
        for l in range(layers):
            for side in range(2):
                exp = clobbered[l][side].view(torch.uint8).reshape(nb, 1, bs, row).cpu().numpy().copy()
                fill_rows = src[l][side].view(torch.uint8).reshape(nb * bs, row)[slots.cpu()].cpu().numpy()
                O.paged_fill_varlen(fill_rows.reshape(1, -1, row), fill_rows.reshape(1, -1, row), cu, pt, sp, exp,
                                    exp.copy())
                got = vllm_caches[l][side].view(torch.uint8).reshape(nb, 1, bs, row).cpu().numpy()
                assert np.array_equal(got, exp), (l, side)
        # rows past the 40-token tail of the last block stay as they were
        for l in range(layers):
            assert torch.equal(vllm_caches[l][:, 14, 8:].view(torch.int16), clobbered[l][:, 14, 8:].view(torch.int16))
        st = server.stats()
        assert st["admissions"] >= 1 and st["host_serves"] >= 2
    finally:
        client.close()
        server.close()


def test_restore_rejects_a_value_of_another_shape_before_changing_anything():
    layers, nb, bs, heads, dim = 2, 16, 16, 2, 64
    vllm_caches = _caches(layers, nb, bs, heads, dim, 10)
    caches = kv_caches_from_vllm(vllm_caches)
    raw = raw_codec_for(caches, bs)
    server = Server(0, max_keys=16, heap_bytes=16 << 20, host_pool_bytes=16 << 20)
    client = Client(0, server)
    kc = KVCacheClient(client, raw)
    try:
        client.put(kc.raw_key("odd"), torch.zeros(1000, dtype=torch.uint8, device="cuda"), 1000, sync_commit=True)
        before = [t.clone() for t in vllm_caches]
        order = server.lru_order()
        with pytest.raises(RuntimeError, match="needs"):
            kc.get_chunks_device(["odd"], caches, layers, [list(range(0, 32))])
        assert server.lru_order() == order
        assert all(torch.equal(a, b) for a, b in zip(vllm_caches, before))
        assert kc.get_chunks_device(["missing"], caches, layers, [list(range(0, 32))]) == [False]
    finally:
        client.close()
        server.close()
