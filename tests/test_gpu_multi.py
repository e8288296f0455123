"""Hash-sharded store across two GPUs in one process: puts and gets move blocks over NVLink
(peer stores into the remote slab, peer loads on get), checked bit-exact against one oracle
store per shard. Needs two visible GPUs."""

import json

import numpy as np
import pytest
import torch

from kvcache_manager import Client, PagedLayout, Server, codec
from oracle import kvs_oracle as O

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs"),
]


def kv_pool(device, n_layers, heads, bs, dim, n_blocks, seed):
    g = torch.Generator().manual_seed(seed)
    return [tuple(torch.randn((n_blocks, heads, bs, dim), generator=g).to(torch.bfloat16).to(device) for _ in range(2))
            for _ in range(n_layers)]


def test_two_gpu_sharded_put_get_matches_per_shard_oracles():
    s0, s1 = Server(0, max_keys=256, heap_bytes=64 << 20, host_pool_bytes=64 << 20), Server(1, max_keys=256, heap_bytes=64 << 20, host_pool_bytes=64 << 20)
    c0 = Client(0, [s0, s1])
    c1 = Client(1, [s0, s1])
    try:
        kv0 = kv_pool("cuda:0", 2, 8, 32, 128, 256, seed=1)
        kv1 = kv_pool("cuda:1", 2, 8, 32, 128, 256, seed=2)
        L0, L1 = PagedLayout.from_kv_caches(kv0), PagedLayout.from_kv_caches(kv1)
        keys = np.array(codec.chained_block_hashes(42, 64), np.uint64)
        shards = np.array([c0.shard_of(int(k)) for k in keys])
        assert 0 < shards.sum() < 64, "keys must land on both shards"
        rng = np.random.default_rng(0)
        src = rng.permutation(256)[:64]
        c0.put_blocks(L0, keys, src)
        # every client sees every shard (the reference's "a shard is visible from every chip")
        assert c1.exists_batch(keys).all()
        dst = rng.permutation(256)[:64]
        before = [t.clone() for p in kv1 for t in p]
        assert c1.get_blocks(L1, keys, dst).all()
        m0 = [t for p in kv0 for t in p]
        m1 = [t for p in kv1 for t in p]
        for m in range(4):
            got = m1[m].view(torch.int16)[torch.as_tensor(dst, device="cuda:1")].cpu()
            exp = m0[m].view(torch.int16)[torch.as_tensor(src, device="cuda:0")].cpu()
            assert torch.equal(got, exp)
            untouched = torch.as_tensor(np.setdiff1d(np.arange(256), dst), device="cuda:1")
            assert torch.equal(m1[m].view(torch.int16)[untouched], before[m].view(torch.int16)[untouched])
        # per-shard directory state equals one oracle store per shard fed the same keys
        host = [t.view(torch.uint8).reshape(-1).cpu().numpy() for t in m0]
        for sid, srv in enumerate((s0, s1)):
            o = O.Store(max_keys=256, heap_bytes=64 << 20)
            sel = shards == sid
            o.put_blocks(host, L0.member_block_bytes, keys[sel], src[sel])
            o.flush()
            for k in keys[sel]:
                assert srv.location(int(k)) == o.location(int(k))
        assert s0.stats()["live_keys"] + s1.stats()["live_keys"] == 64
    finally:
        c0.close()
        c1.close()
        s0.close()
        s1.close()


def test_gather_tp_shards_across_two_gpus_golden(golden_dir):
    from kvcache_manager import ops

    fx = json.loads((golden_dir / "gather_roundtrip.json").read_text())
    expected = (golden_dir / "gather_roundtrip_expected.bin").read_bytes()
    sbb, nm = fx["SHARD_BLOCK_BYTES"], fx["N_MEMBERS"]
    wpm = fx["BLOCKS"] * sbb // 4
    host = []
    for m in range(nm):
        g = torch.Generator().manual_seed(fx["member_seed0"] + m)
        host.append(torch.randint(0, 2**31 - 1, (fx["chips"], wpm), dtype=torch.int32, generator=g))
    ranks = fx["rank_indices"]
    # rank 0 and 2 on GPU 1 (peer), rank 1 on GPU 0 (the master)
    dev = {r: ("cuda:1" if r != 1 else "cuda:0") for r in ranks}
    members = [[host[m][r].clone().to(dev[r]) for m in range(nm)] for r in ranks]
    blob = torch.zeros(fx["value_len"], dtype=torch.uint8, device="cuda:0")
    ops.gather_tp_shards_to_chip(members, blob, fx["CHUNK_BLOCKS"], sbb, fx["region_bases"], fx["header_words"])
    assert blob.cpu().numpy().tobytes() == expected
    for r in members:
        for t in r:
            t.zero_()
    ops.scatter_chunk_from_chip(blob, members, fx["CHUNK_BLOCKS"], sbb, fx["region_bases"])
    for i, r in enumerate(ranks):
        for m in range(nm):
            for blk in fx["CHUNK_BLOCKS"]:
                lo, hi = blk * sbb // 4, (blk + 1) * sbb // 4
                assert torch.equal(members[i][m].cpu()[lo:hi], host[m][r][lo:hi])
