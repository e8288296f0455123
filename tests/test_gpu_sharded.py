"""The process-per-GPU sharded store on B200s against one oracle store per shard.

* owner API on one GPU: one shard serves the gets of two paged pools in one scatter launch
  (kvs_serve_gets with two member sets) and grants puts that the pools gather into its slab
  (kvs_grant_puts / kvs_copy_blocks / kvs_puts_landed), over a small slab that forces evictions,
  host-tier serves and multi-round grants;
* the collective ShardedStore with one rank (NCCL world of 1), both transports;
* two ranks on two GPUs (skipped with fewer): P2P stores over NVLink through CUDA IPC mappings,
  and the NCCL send/recv comparison transport.
Every restored pool byte, every found flag and the store counters must equal the replay."""

import ctypes as C
import os
import socket

import numpy as np
import pytest
import torch

from kvcache_manager import PagedLayout, _native, sharded
from kvcache_manager._native import check, load
from sharded_common import make_plan, make_pools, replay, replay_steps

pytestmark = pytest.mark.gpu
MB = 512
N_MEMBERS = 4
N_POOL = 96
CFG = dict(max_keys=48, heap_bytes=40 * 4288, host_pool_bytes=256 * 4288)
STAT_FIELDS = ("live_keys", "device_resident_keys", "victims_evicted", "host_serves", "admissions",
               "writes_through", "epoch")


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _gpu_pool(host_members, device):
    members = [torch.from_numpy(m.reshape(N_POOL, MB)).to(device) for m in host_members]
    return members, PagedLayout(members, members_per_layer=2)


def _host(members):
    return [m.reshape(-1).cpu().numpy() for m in members]


@pytest.mark.parametrize("slab_units", [40, 10])
def test_owner_api_serves_two_pools_like_the_oracle(slab_units):
    cfg = dict(CFG, heap_bytes=slab_units * 4288)
    plan = make_plan(2, 8, N_POOL, 12, seed=21)
    pools = make_pools(2, N_MEMBERS, MB, N_POOL, seed=4)
    expected = replay_steps(plan, pools, MB, cfg, n_shards=1)
    gpu = [_gpu_pool(p, "cuda:0") for p in pools]
    eng = sharded.DeviceEngine(gpu[0][1], **cfg)
    eng._peer_layouts = (_native.BlockLayout * 2)(gpu[0][1].c, gpu[1][1].c)
    lib = load()
    rounds = 0
    try:
        for s_idx, row in enumerate(plan):
            keys = np.concatenate([row[0][0], row[1][0]])
            ids = np.concatenate([row[0][1], row[1][1]])
            sets = np.repeat(np.arange(2, dtype=np.uint32), [row[0][0].size, row[1][0].size])
            exp_pools, exp_found, exp_stats = next(expected)
            found = eng.serve_gets(sets, ids, keys)
            assert np.array_equal(found[:row[0][0].size], exp_found[0]), s_idx
            assert np.array_equal(found[row[0][0].size:], exp_found[1]), s_idx
            pk = np.concatenate([row[0][2], row[1][2]])
            src = np.repeat([0, 1], [row[0][2].size, row[1][2].size])
            pid = np.concatenate([row[0][3], row[1][3]])
            cursor = 0
            while cursor < pk.size:
                offs, ng, rc = eng.grant_puts(pk[cursor:])
                assert rc == _native.OK
                rounds += 1
                for p in (0, 1):
                    sel = np.flatnonzero(src[cursor:cursor + ng] == p) + cursor
                    if sel.size:
                        addrs = np.ascontiguousarray(offs[sel - cursor] + np.uint64(eng.slab_base))
                        b = np.ascontiguousarray(pid[sel])
                        check(lib.kvs_copy_blocks(eng.client._handle(), C.byref(gpu[p][1].c), sel.size,
                                                  b.ctypes.data_as(_native._i64p), addrs.ctypes.data_as(_native._u64p),
                                                  1, torch.cuda.current_stream().cuda_stream))
                eng.puts_landed()
                cursor += ng
            if s_idx == len(plan) - 1:
                eng.flush()
            torch.cuda.synchronize()
            st = eng.stats()
            for p in (0, 1):
                for m, (got, exp) in enumerate(zip(_host(gpu[p][0]), exp_pools[p])):
                    bad = np.flatnonzero((got.reshape(N_POOL, MB) != exp.reshape(N_POOL, MB)).any(1))
                    assert bad.size == 0, (
                        f"step {s_idx} pool {p} member {m}: blocks {bad.tolist()} differ; gets of this pool "
                        f"{list(zip(row[p][0].tolist(), row[p][1].tolist()))}, found {found.tolist()}, "
                        f"stats {st}, expected {exp_stats[0]}")
        next(expected, None)
        for f in STAT_FIELDS:
            assert st[f] == exp_stats[0][f], (f, st[f], exp_stats[0][f])
        assert st["victims_evicted"] > 0 and st["host_serves"] > 0
        if slab_units < 24:  # a step's 24 puts do not fit: some wait for the commit of a landed one
            assert rounds > len(plan)
    finally:
        eng.close()


def _run_ranks(rank, world, port, transport, steps, batch, q):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    store = None
    try:
        plan = make_plan(world, steps, N_POOL, batch, seed=31)
        pools = make_pools(world, N_MEMBERS, MB, N_POOL, seed=5)
        members, layout = _gpu_pool(pools[rank], f"cuda:{rank}")
        store = sharded.create(layout, max_batch=batch, transport=transport, **CFG)
        found, snaps = [], []
        for row in plan:
            gk, gi, pk, pi = row[rank]
            found.append(store.step(gk, gi, pk, pi))
            torch.cuda.synchronize()
            snaps.append(_host(members))
        store.flush()
        torch.cuda.synchronize()
        out = (rank, snaps, found, store.stats())
        store.close()
        store = None
        q.put(out)
    finally:
        dist.destroy_process_group()


def _check_against_replay(outs, world, steps, batch):
    plan = make_plan(world, steps, N_POOL, batch, seed=31)
    pools = make_pools(world, N_MEMBERS, MB, N_POOL, seed=5)
    for s, (exp_pools, exp_found, exp_stats) in enumerate(replay_steps(plan, pools, MB, CFG)):
        for rank, snaps, found, _ in outs:
            assert np.array_equal(found[s], exp_found[rank]), f"rank {rank} step {s}"
            for m in range(N_MEMBERS):
                got = snaps[s][m].reshape(N_POOL, MB)
                bad = np.flatnonzero((got != exp_pools[rank][m].reshape(N_POOL, MB)).any(1))
                origin = []
                for b in bad[:2]:
                    # where the delivered bytes came from: a block of some rank's initial pool?
                    for r2 in range(world):
                        src = pools[r2][m].reshape(N_POOL, MB)
                        hit = np.flatnonzero((src == got[b]).all(1))
                        if hit.size:
                            origin.append((int(b), r2, hit.tolist()))
                    nz = int(np.count_nonzero(got[b] != exp_pools[rank][m].reshape(N_POOL, MB)[b]))
                    origin.append((int(b), "bytes differing", nz, "first", got[b][:8].tolist(),
                                   exp_pools[rank][m].reshape(N_POOL, MB)[b][:8].tolist()))
                assert bad.size == 0, (
                    f"origin {origin}; "
                    f"step {s} rank {rank} member {m}: blocks {bad.tolist()} differ; this rank's gets "
                    f"{list(zip(plan[s][rank][0].tolist(), plan[s][rank][1].tolist(), found[s].tolist()))}; "
                    f"puts {list(zip(plan[s][rank][2].tolist(), plan[s][rank][3].tolist()))}")
    for rank, _, _, stats in outs:
        for f in STAT_FIELDS:
            assert stats[f] == exp_stats[rank][f], (rank, f, stats[f], exp_stats[rank][f])


@pytest.mark.parametrize("transport", ["p2p", "nccl"])
def test_sharded_store_single_rank(transport):
    import queue

    q = queue.Queue()
    _run_ranks(0, 1, _free_port(), transport, 6, 12, q)
    _check_against_replay([q.get()], 1, 6, 12)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("transport", ["p2p", "nccl"])
def test_sharded_store_two_gpus(transport):
    import torch.multiprocessing as mp

    world, steps, batch = 2, 8, 12
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_run_ranks, args=(r, world, port, transport, steps, batch, q)) for r in range(world)]
    for p in procs:
        p.start()
    outs = sorted((q.get(timeout=300) for _ in range(world)), key=lambda o: o[0])
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    _check_against_replay(outs, world, steps, batch)


def test_owner_and_copy_entry_points_reject_bad_arguments():
    """Host-side checks of the process-per-GPU entry points (nothing reaches a kernel)."""
    import ctypes as C

    from kvcache_manager import Client, KvsError, Server

    lib = load()
    members = [torch.zeros((8, 512), dtype=torch.uint8, device="cuda") for _ in range(2)]
    layout = PagedLayout(members, members_per_layer=2)
    other = PagedLayout([torch.zeros((8, 256), dtype=torch.uint8, device="cuda") for _ in range(2)], members_per_layer=2)
    s0, s1 = Server(0, max_keys=16, heap_bytes=16 * 4288), Server(0, max_keys=16, heap_bytes=16 * 4288)
    two = Client(0, [s0, s1])
    one = Client(0, s0)
    try:
        keys = np.arange(1, 3, dtype=np.uint64)
        offs = np.zeros(2, np.uint64)
        ng = C.c_uint32()
        # an owner client has exactly one shard
        rc = lib.kvs_grant_puts(two._handle(), 2, keys.ctypes.data_as(_native._u64p), 1056,
                                offs.ctypes.data_as(_native._u64p), C.byref(ng))
        assert rc == _native.E_INVAL and b"exactly one shard" in lib.kvs_last_error()
        # a value longer than max_value_bytes
        rc = lib.kvs_grant_puts(one._handle(), 2, keys.ctypes.data_as(_native._u64p), 1 << 40,
                                offs.ctypes.data_as(_native._u64p), C.byref(ng))
        assert rc == _native.E_INVAL
        # serve_gets: every pool must have the same member sizes; pool index and block range checked
        pools = (_native.BlockLayout * 2)(layout.c, other.c)
        sets = np.zeros(1, np.uint32)
        ids = np.zeros(1, np.int64)
        found = np.zeros(1, np.uint8)
        k1 = keys[:1].copy()
        args = lambda n_sets, ls, st, bi: (one._handle(), n_sets, ls, 1, st.ctypes.data_as(_native._u32p),
                                           bi.ctypes.data_as(_native._i64p), k1.ctypes.data_as(_native._u64p),
                                           found.ctypes.data_as(_native._u8p), None)
        assert lib.kvs_serve_gets(*args(2, pools, sets, ids)) == _native.E_INVAL
        assert b"other member sizes" in lib.kvs_last_error()
        assert lib.kvs_serve_gets(*args(1, pools, np.array([3], np.uint32), ids)) == _native.E_INVAL
        assert lib.kvs_serve_gets(*args(1, pools, sets, np.array([99], np.int64))) == _native.E_INVAL
        # copy_blocks: 16-byte aligned addresses, block ids inside the pool
        addr = np.array([members[0].data_ptr() + 8], np.uint64)
        rc = lib.kvs_copy_blocks(one._handle(), C.byref(layout.c), 1, ids.ctypes.data_as(_native._i64p),
                                 addr.ctypes.data_as(_native._u64p), 1, None)
        assert rc == _native.E_INVAL and b"16-byte aligned" in lib.kvs_last_error()
        addr[0] -= 8
        rc = lib.kvs_copy_blocks(one._handle(), C.byref(layout.c), 1, np.array([8], np.int64).ctypes.data_as(_native._i64p),
                                 addr.ctypes.data_as(_native._u64p), 1, None)
        assert rc == _native.E_INVAL and b"outside" in lib.kvs_last_error()
        # puts_landed with nothing granted is a no-op
        assert lib.kvs_puts_landed(one._handle(), None) == _native.OK
        with pytest.raises(KvsError):
            check(lib.kvs_grant_puts(two._handle(), 0, None, 1056, None, C.byref(ng)))
    finally:
        one.close()
        two.close()
        s0.close()
        s1.close()
