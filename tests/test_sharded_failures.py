"""Failures of the process-per-GPU sharded store, made on the host with gloo ranks on CPU: a
shard that cannot grant space fails only the puts it owns, and every rank still takes the same
collective steps; a rank that stops calling ends the other ranks' next step with an error after
the process group's timeout instead of leaving them waiting."""

import os
import socket
import time
from datetime import timedelta

import numpy as np
import torch.distributed as dist
import torch.multiprocessing as mp

from kvcache_manager import _native, sharded
from kvcache_manager._native import KvsError
from sharded_common import HostEngine, make_pools

MB = 512
N_MEMBERS = 4
N_POOL = 32
CFG = dict(max_keys=48, heap_bytes=40 * 4288, host_pool_bytes=256 * 4288)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


class FullShard(HostEngine):
    """A shard whose device cache never has room: every grant fails."""

    def grant_puts(self, keys):
        return np.zeros(keys.size, np.uint64), 0, _native.E_NOSPACE


def _keys_owned_by(owner, world, n, start):
    out, k = [], start
    while len(out) < n:
        if int(sharded.shard_of_u64(np.array([k], np.uint64), world)[0]) == owner:
            out.append(k)
        k += 1
    return np.array(out, np.uint64)


def _full_shard_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        pools = make_pools(world, N_MEMBERS, MB, N_POOL, seed=5)
        eng = (FullShard if rank == 1 else HostEngine)(pools[rank], MB, CFG)
        store = sharded.ShardedStore(eng, max_batch=8, transport="nccl")
        to0 = _keys_owned_by(0, world, 3, 1000)
        to1 = _keys_owned_by(1, world, 2, 2000)
        # rank 0 puts to both shards, rank 1 only to shard 0
        pk = np.concatenate([to0, to1]) if rank == 0 else _keys_owned_by(0, world, 2, 3000)
        err = None
        try:
            store.step((), (), pk, np.arange(pk.size))
        except KvsError as e:
            err = (e.code, str(e))
        # the next step runs on every rank: rank 0 reads back what it put
        got = store.step(np.concatenate([to0, to1]) if rank == 0 else (),
                         np.arange(10, 15) if rank == 0 else ())
        q.put((rank, err, got.tolist()))
        store.close()
    finally:
        dist.destroy_process_group()


def test_a_full_shard_fails_only_the_puts_it_owns():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_full_shard_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = sorted((q.get(timeout=240) for _ in range(world)), key=lambda o: o[0])
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    (_, err0, got0), (_, err1, got1) = out
    assert err0 is not None and err0[0] == _native.E_NOSPACE and "shards [1]" in err0[1]
    assert err1 is None  # rank 1's puts all went to the healthy shard
    assert got0 == [True, True, True, False, False] and got1 == []


def _silent_rank_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=3))
    pools = make_pools(world, N_MEMBERS, MB, N_POOL, seed=6)
    store = sharded.ShardedStore(HostEngine(pools[rank], MB, CFG), max_batch=8, transport="nccl")
    keys = np.arange(50 + 10 * rank, 54 + 10 * rank, dtype=np.uint64)
    store.step((), (), keys, np.arange(4))  # one step together
    if rank == 1:
        time.sleep(12)  # stops calling (stays alive, never joins the next step)
        q.put((rank, None, 0.0))
        return
    t0 = time.monotonic()
    err = None
    try:
        store.step(keys, np.arange(8, 12))
    except Exception as e:  # the collective gives up after the process group's timeout
        err = type(e).__name__
    q.put((rank, err, time.monotonic() - t0))


def test_a_rank_that_stops_calling_ends_the_next_step_with_an_error():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_silent_rank_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = sorted((q.get(timeout=240) for _ in range(world)), key=lambda o: o[0])
    for p in procs:
        p.join(timeout=60)
        if p.exitcode is None:
            p.kill()
    (_, err0, waited), _ = out
    assert err0 is not None, "rank 0's step returned although rank 1 never joined it"
    assert waited < 11, f"rank 0 waited {waited:.1f} s, past the 3 s process-group timeout"
