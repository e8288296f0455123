"""Multi-turn prefix reuse (config-1 KV shape, slab = 25 % of the working set) on the GPU store
against the oracle: the same driver runs exists -> get of the longest hit prefix -> put of the rest
for every turn; restored pool bytes, every key's residency and the store counters must match."""

import numpy as np
import pytest
import torch

import bench
from kvcache_manager import Client, PagedLayout, Server, codec
from oracle import kvs_oracle as O

pytestmark = pytest.mark.gpu
U = 4288


class OracleClient:
    """The oracle store behind the Client methods the workload driver calls."""

    def __init__(self, store, members, member_bytes):
        self.s, self.members, self.mb = store, members, member_bytes

    def exists_batch(self, keys):
        return np.array([self.s.exists(int(k)) for k in keys], bool)

    def get_blocks(self, layout, keys, ids):
        return self.s.get_blocks(self.members, self.mb, keys, ids)

    def put_blocks(self, layout, keys, ids):
        self.s.put_blocks(self.members, self.mb, keys, ids)


def test_multiturn_prefix_reuse_matches_oracle():
    layers, heads, dim, bt, pool = 2, 4, 64, 32, 512
    g = torch.Generator().manual_seed(13)
    kv = [tuple(torch.randn((pool, heads, bt, dim), generator=g).to(torch.bfloat16).cuda() for _ in range(2))
          for _ in range(layers)]
    layout = PagedLayout.from_kv_caches(kv)
    members = [t for p in kv for t in p]
    host = [t.view(torch.uint8).reshape(-1).cpu().numpy().copy() for t in members]
    plan = bench.multiturn_plan(8, 5, seed=5, lo=128, hi=1024, block_tokens=bt)
    working_set = sum(p[-1] for p in plan)
    vlen = layout.value_bytes()
    units = -(-vlen // U)
    block_bytes = (1 << (units - 1).bit_length()) * U
    slab = working_set * block_bytes // 4
    cfg = dict(max_keys=2 * working_set, heap_bytes=slab, host_pool_bytes=(working_set + 16) * units * U)
    server = Server(0, **cfg)
    client = Client(0, server)
    ostore = O.Store(**cfg)
    oclient = OracleClient(ostore, host, layout.member_block_bytes)
    try:
        st = bench.run_multiturn_workload(client, layout, plan, pool, seed=5)
        ost = bench.run_multiturn_workload(oclient, layout, plan, pool, seed=5)
        assert st == ost
        assert st["prefix_hits"] > 0 and st["puts"] > 0
        torch.cuda.synchronize()
        for m, t in enumerate(members):
            assert np.array_equal(t.view(torch.uint8).reshape(-1).cpu().numpy(), host[m]), f"member {m} differs"
        client.flush()
        ostore.flush()
        for s_idx, turns in enumerate(plan):
            for k in codec.chained_block_hashes(1_000_003 * (s_idx + 1), turns[-1]):
                assert server.location(int(k))[0] == ostore.location(int(k))[0]
        ss, so = server.stats(), ostore.stats()
        for f in ("live_keys", "device_resident_keys", "victims_evicted", "host_serves", "admissions",
                  "live_device_bytes", "epoch"):
            assert ss[f] == so[f], (f, ss[f], so[f])
        assert ss["victims_evicted"] > 0 and ss["host_serves"] > 0
    finally:
        client.close()
        server.close()
