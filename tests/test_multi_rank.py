"""Host logic of the N > 1 path on CPU: two gloo ranks agree on key ownership with the C ABI's
shard function, exchange per-shard counts, and reduce their times to the max over ranks."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from kvcache_manager import codec

import shard_helpers as kdist


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        keys = codec.chained_block_hashes(100 + rank, 256)
        perm, counts = kdist.bucket_by_shard(keys, world)
        # everyone learns how many keys every rank sends to every shard
        mine = torch.tensor(counts, dtype=torch.int64)
        allc = [torch.zeros_like(mine) for _ in range(world)]
        dist.all_gather(allc, mine)
        incoming = sum(int(c[rank]) for c in allc)
        t = kdist.max_over_ranks(float(rank + 1) * 1.5)
        q.put((rank, counts.tolist(), incoming, t, [int(keys[i]) for i in perm[:4]]))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_agree_on_ownership_and_timing():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = sorted(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    total_sent = sum(sum(o[1]) for o in out)
    assert total_sent == 2 * 256 and sum(o[2] for o in out) == total_sent
    assert all(o[3] == 3.0 for o in out)  # max over ranks of 1.5, 3.0
    for rank, counts, _, _, first in out:
        assert all(kdist.shard_of(k, world) == 0 for k in first[: counts[0]][:4])


def test_shard_function_matches_the_c_abi_and_oracle():
    from oracle import kvs_oracle as O

    for k in codec.chained_block_hashes(7, 64):
        b = int(k).to_bytes(8, "little")
        assert kdist.fnv1a32(b) == O.fnv1a32(b)
        for n in (2, 4, 8):
            assert kdist.shard_of(k, n) == O.fnv1a32(b) % n
    perm, counts = kdist.bucket_by_shard(codec.chained_block_hashes(3, 100), 4)
    assert counts.sum() == 100 and sorted(perm.tolist()) == list(range(100))
