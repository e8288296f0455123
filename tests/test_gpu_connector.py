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
