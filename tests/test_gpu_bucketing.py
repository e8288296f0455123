"""GPU bucketing of a sharded step's requests (kvs_bucket_requests) against the host path
(sharded.pack_requests): the same records, word for word, and the same per-owner batch positions,
with and without a placement table; overflow of one owner's capacity is reported."""

import ctypes as C

import numpy as np
import pytest
import torch

from kvcache_manager import _native
from kvcache_manager.sharded import pack_requests, placement_table, request_words

pytestmark = pytest.mark.gpu


def _bucket(world, cap, op, gk, gi, pk, pi, table):
    lib = _native.load()
    dev = torch.device("cuda", 0)
    keys = torch.from_numpy(np.concatenate([gk, pk]).view(np.int64).copy()).to(dev)
    ids = torch.from_numpy(np.concatenate([gi, pi]).astype(np.int64)).to(dev)
    rec = torch.full((world * request_words(cap),), -7, dtype=torch.int64, device=dev)  # stale words
    back = torch.full((world * 2 * cap,), -1, dtype=torch.int32, device=dev)
    counts = torch.full((2 * world,), -1, dtype=torch.int32, device=dev)
    overflow = torch.full((1,), 5, dtype=torch.int32, device=dev)
    tab = torch.from_numpy(table.astype(np.int32)).to(dev) if table is not None else None
    p = lambda t: C.c_void_p(t.data_ptr()) if t is not None else None
    n = gk.size + pk.size
    _native.check(lib.kvs_bucket_requests(0, p(keys) if n else None, p(ids) if n else None, n, gk.size, p(tab),
                                          world, cap, op, p(rec), p(back), p(counts), p(overflow), None))
    torch.cuda.synchronize()
    return (rec.cpu().numpy().reshape(world, -1), back.cpu().numpy().reshape(world, 2, cap),
            counts.cpu().numpy().reshape(2, world), int(overflow.item()))


@pytest.mark.parametrize("world,cap,weighted", [(1, 8, False), (2, 16, False), (3, 32, True), (8, 256, False),
                                                (8, 256, True), (5, 64, True)])
def test_records_and_positions_equal_the_host_path(world, cap, weighted):
    rng = np.random.default_rng(world * 1000 + cap)
    table = placement_table(rng.uniform(0.5, 1.5, world)) if weighted else None
    for op in (0, 1):
        # sizes that keep every owner within cap: at most cap // 2 keys of each kind per owner on average
        ng = int(rng.integers(0, world * cap // 2 + 1))
        npt = int(rng.integers(0, world * cap // 2 + 1))
        gk = rng.integers(0, 1 << 63, ng, dtype=np.int64).view(np.uint64) * np.uint64(2) + np.uint64(1)
        pk = rng.integers(0, 1 << 63, npt, dtype=np.int64).view(np.uint64)
        if ng > 3:
            gk[1] = gk[0]  # a repeated key keeps both positions
        gi = rng.integers(0, 1 << 40, ng, dtype=np.int64)
        pi = rng.integers(0, 1 << 40, npt, dtype=np.int64)
        try:
            want, g_pos, p_pos = pack_requests(world, cap, op, gk, gi, pk, pi, table)
        except ValueError:  # an owner over cap: the overflow test covers it
            continue
        rec, back, counts, overflow = _bucket(world, cap, op, gk, gi, pk, pi, table)
        assert overflow == 0
        assert np.array_equal(rec, want)
        for o in range(world):
            assert np.array_equal(back[o, 0, :counts[0, o]], g_pos[o])
            assert np.array_equal(back[o, 1, :counts[1, o]], p_pos[o])


def test_empty_batch_gives_empty_records():
    world, cap = 4, 8
    e = np.zeros(0, np.uint64)
    rec, _, counts, overflow = _bucket(world, cap, 0, e, np.zeros(0, np.int64), e, np.zeros(0, np.int64), None)
    want, _, _ = pack_requests(world, cap, 0, e, np.zeros(0, np.int64), e, np.zeros(0, np.int64))
    assert overflow == 0 and not counts.any()
    assert np.array_equal(rec, want)


def test_overflow_of_one_owner_is_reported_and_capped():
    world, cap = 2, 4
    keys = np.arange(1, 4000, dtype=np.uint64)
    from kvcache_manager.sharded import shard_of_u64

    own = shard_of_u64(keys, world)
    gk = keys[own == 1][:10]  # ten gets for owner 1
    gi = np.arange(10, dtype=np.int64)
    e = np.zeros(0, np.uint64)
    with pytest.raises(ValueError):
        pack_requests(world, cap, 0, gk, gi, e, np.zeros(0, np.int64))
    rec, back, counts, overflow = _bucket(world, cap, 0, gk, gi, e, np.zeros(0, np.int64), None)
    assert overflow == 1
    assert counts[0, 1] == cap and counts[0, 0] == 0
    assert np.array_equal(back[1, 0, :cap], np.arange(cap))
    assert np.array_equal(rec[1, 4:4 + cap].view(np.uint64), gk[:cap])
