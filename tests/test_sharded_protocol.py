"""The collective protocol of the process-per-GPU sharded store on CPU gloo ranks: routing of
requests and replies, the row transport, multi-round put grants and the per-step order (gets of
every rank, then puts of every rank) must reproduce one oracle store per shard exactly."""

import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from kvcache_manager import sharded
from sharded_common import HostEngine, make_plan, make_pools, replay

MB = 512  # bytes of one member block
N_MEMBERS = 4
N_POOL = 96
CFG = dict(max_keys=48, heap_bytes=40 * 4288, host_pool_bytes=256 * 4288)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, steps, batch, grant_limit, q, weights=None):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        plan = make_plan(world, steps, N_POOL, batch, seed=11)
        pools = make_pools(world, N_MEMBERS, MB, N_POOL, seed=3)
        eng = HostEngine(pools[rank], MB, CFG, grant_limit=grant_limit)
        store = sharded.ShardedStore(eng, max_batch=batch, transport="nccl", weights=weights)
        found = []
        for row in plan:
            gk, gi, pk, pi = row[rank]
            found.append(store.step(gk, gi, pk, pi))
        ex = store.exists_batch(plan[-1][rank][2])
        store.flush()
        q.put((rank, [m.copy() for m in eng.members], found, eng.stats(), ex, eng.rounds))
        store.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,grant_limit", [(2, None), (3, 2)])
def test_sharded_protocol_matches_per_shard_oracle(world, grant_limit):
    steps, batch = 6, 12
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, steps, batch, grant_limit, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = sorted((q.get(timeout=240) for _ in range(world)), key=lambda o: o[0])
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    plan = make_plan(world, steps, N_POOL, batch, seed=11)
    pools = make_pools(world, N_MEMBERS, MB, N_POOL, seed=3)
    exp_pools, exp_found, exp_stats = replay(plan, pools, MB, CFG)
    for rank, members, found, stats, ex, rounds in out:
        for m in range(N_MEMBERS):
            assert np.array_equal(members[m], exp_pools[rank][m]), f"rank {rank} member {m}"
        for s in range(steps):
            assert np.array_equal(found[s], exp_found[s][rank]), f"rank {rank} step {s}"
        for f in ("live_keys", "device_resident_keys", "victims_evicted", "host_serves", "admissions",
                  "writes_through", "epoch"):
            assert stats[f] == exp_stats[rank][f], (rank, f)
        assert ex.all()  # every key this rank put in the last step exists somewhere
        if grant_limit:
            assert rounds > steps  # some steps took more than one grant round
    assert any(f.any() for fs in exp_found for f in fs) and not all(f.all() for fs in exp_found for f in fs)


def test_weighted_placement_matches_per_shard_oracle():
    """Keys placed in proportion to per-shard weights (as by each GPU's device->host rate): the
    shards own their share of the keys and every rank's results equal the oracle replay with the
    same placement."""
    world, steps, batch, weights = 3, 5, 12, [1.0, 2.5, 1.5]
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, steps, batch, None, q, weights)) for r in range(world)]
    for p in procs:
        p.start()
    out = sorted((q.get(timeout=240) for _ in range(world)), key=lambda o: o[0])
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    table = sharded.placement_table(weights)
    plan = make_plan(world, steps, N_POOL, batch, seed=11)
    pools = make_pools(world, N_MEMBERS, MB, N_POOL, seed=3)
    exp_pools, exp_found, exp_stats = replay(plan, pools, MB, CFG, table=table)
    for rank, members, found, stats, ex, rounds in out:
        for m in range(N_MEMBERS):
            assert np.array_equal(members[m], exp_pools[rank][m]), f"rank {rank} member {m}"
        for s in range(steps):
            assert np.array_equal(found[s], exp_found[s][rank]), f"rank {rank} step {s}"
        assert stats["live_keys"] == exp_stats[rank]["live_keys"]
    keys = np.random.default_rng(0).integers(0, 2**63, 30000).astype(np.uint64)
    share = np.bincount(sharded.shard_of_u64(keys, world, table), minlength=world) / keys.size
    assert np.allclose(share, np.array(weights) / sum(weights), atol=0.02)


def test_placement_table_shares():
    for w in ([1, 1], [1, 2, 3], [11.5] * 4 + [18.2] * 4, [3.0]):
        t = sharded.placement_table(w)
        assert t.size == sharded.PLACEMENT_SLOTS and (np.diff(t) >= 0).all()
        counts = np.bincount(t, minlength=len(w))
        assert np.all(np.abs(counts - np.array(w) / sum(w) * sharded.PLACEMENT_SLOTS) < 1)
    for bad in ([], [1, 0], [1, -2], [float("nan")]):
        with pytest.raises(ValueError):
            sharded.placement_table(bad)


def test_pack_unpack_requests_round_trip():
    world, cap = 3, 8
    rng = np.random.default_rng(1)
    gk = rng.integers(0, 2**63, 7).astype(np.uint64)
    pk = rng.integers(0, 2**63, 5).astype(np.uint64)
    gi, pi = np.arange(7), np.arange(10, 15)
    rec, g_pos, p_pos = sharded.pack_requests(world, cap, 0, gk, gi, pk, pi)
    for o in range(world):
        (k, i, k2, i2), = sharded.unpack_requests(rec[o:o + 1], cap)
        assert np.array_equal(k, gk[g_pos[o]]) and np.array_equal(i, gi[g_pos[o]])
        assert np.array_equal(k2, pk[p_pos[o]]) and np.array_equal(i2, pi[p_pos[o]])
        assert (sharded.shard_of_u64(k, world) == o).all()


def test_shard_of_u64_matches_the_c_abi_function():
    import shard_helpers as kdist

    keys = np.random.default_rng(2).integers(0, 2**64 - 1, 300, dtype=np.uint64)
    for n in (1, 2, 3, 8):
        assert sharded.shard_of_u64(keys, n).tolist() == [kdist.shard_of(int(k), n) for k in keys]


def _empty_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        pools = make_pools(world, N_MEMBERS, MB, N_POOL, seed=8)
        eng = HostEngine(pools[rank], MB, CFG)
        store = sharded.ShardedStore(eng, max_batch=8, transport="nccl")
        keys = np.arange(100 + 10 * rank, 104 + 10 * rank, dtype=np.uint64)
        # rank 1 sits out the put step and rank 0 the get step: every rank still takes every collective
        store.step((), (), keys if rank == 0 else (), np.arange(4) if rank == 0 else ())
        got = store.step(np.arange(100, 104, dtype=np.uint64) if rank == 1 else (), np.arange(8, 12) if rank == 1 else ())
        ex = store.exists_batch(np.arange(98, 106, dtype=np.uint64) if rank == 1 else ())
        none = store.step()  # nobody has anything
        q.put((rank, got.tolist(), ex.tolist(), none.tolist(), [m.copy() for m in eng.members]))
        store.close()
    finally:
        dist.destroy_process_group()


def test_sharded_protocol_with_empty_batches():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_empty_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = sorted((q.get(timeout=240) for _ in range(world)), key=lambda o: o[0])
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    pools = make_pools(world, N_MEMBERS, MB, N_POOL, seed=8)
    (r0, got0, ex0, none0, _), (r1, got1, ex1, none1, mem1) = out
    assert got0 == [] and ex0 == [] and none0 == [] and none1 == []
    assert got1 == [True] * 4 and ex1 == [False, False, True, True, True, True, False, False]
    for m in range(N_MEMBERS):  # rank 1's blocks 8..11 now hold rank 0's blocks 0..3
        want = pools[1][m].reshape(N_POOL, MB).copy()
        want[8:12] = pools[0][m].reshape(N_POOL, MB)[0:4]
        assert np.array_equal(mem1[m].reshape(N_POOL, MB), want)
