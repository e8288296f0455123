"""Shared pieces of the sharded-store tests: a seeded multi-rank workload, its replay on one
oracle store per shard (the expected result), and an oracle-backed engine that lets the
collective protocol run on CPU gloo ranks.

The replay is the protocol's contract: in every step each owner first serves the gets of every
rank (rank order, then batch order), then stores the puts of every rank (same order)."""

from __future__ import annotations

import numpy as np

from kvcache_manager import codec
from kvcache_manager.sharded import shard_of_u64
from oracle import kvs_oracle as O


def make_plan(world: int, steps: int, n_pool: int, batch: int, seed: int, get_frac: float = 0.7):
    """plan[step][rank] = (get_keys, get_ids, put_keys, put_ids). Gets draw from keys put in earlier
    steps by any rank plus a few never-put keys; puts are fresh keys or overwrites (two ranks may
    put one key in the same step); block ids of one rank's step are distinct."""
    rng = np.random.default_rng(seed)
    fresh = [iter(codec.chained_block_hashes(7919 * (r + 1) + seed, steps * batch + 1)) for r in range(world)]
    written: list[int] = []
    plan = []
    for _ in range(steps):
        row, new = [], []
        for r in range(world):
            n_get = int(round(batch * get_frac)) if written else 0
            n_put = batch - n_get
            ids = rng.permutation(n_pool)[:batch]
            gk = []
            for _ in range(n_get):
                if rng.random() < 0.1:
                    gk.append(int(rng.integers(1, 2**63)))  # a miss
                else:
                    gk.append(written[int(rng.integers(len(written)))])
            pk = []
            for _ in range(n_put):
                if written and rng.random() < 0.15:
                    pk.append(written[int(rng.integers(len(written)))])  # overwrite
                else:
                    pk.append(int(next(fresh[r])))
            pk = list(dict.fromkeys(pk))  # a key once per rank's step
            row.append((np.array(gk, np.uint64), ids[:len(gk)].astype(np.int64), np.array(pk, np.uint64),
                        ids[len(gk):len(gk) + len(pk)].astype(np.int64)))
            new += pk
        written = list(dict.fromkeys(written + new))
        plan.append(row)
    return plan


def make_pools(world: int, n_members: int, member_bytes: int, n_pool: int, seed: int):
    rng = np.random.default_rng(seed)
    return [[rng.integers(0, 256, n_pool * member_bytes, dtype=np.uint8) for _ in range(n_members)]
            for _ in range(world)]


def replay(plan, pools, member_bytes, store_cfg, n_shards: int | None = None, table=None):
    """Expected result: (final pools, found flags [step][rank], per-shard stats). n_shards defaults
    to one shard per rank; `table` is the store's key placement table (None: fnv1a32 mod n)."""
    found = []
    for pools_now, f_row, stats in replay_steps(plan, pools, member_bytes, store_cfg, n_shards, table):
        found.append(f_row)
    return pools_now, found, stats


def replay_steps(plan, pools, member_bytes, store_cfg, n_shards: int | None = None, table=None):
    """The replay one step at a time: yields (pools, found flags per rank, per-shard stats) after
    every step; the stats of the last step follow a final flush."""
    world = len(pools)
    n_shards = world if n_shards is None else n_shards
    pools = [[m.copy() for m in p] for p in pools]
    stores = [O.Store(**store_cfg) for _ in range(n_shards)]
    mb = [member_bytes] * len(pools[0])
    for step, row in enumerate(plan):
        f_row = [np.zeros(row[r][0].size, bool) for r in range(world)]
        for o in range(n_shards):
            for s in range(world):
                gk, gi = row[s][0], row[s][1]
                sel = np.flatnonzero(shard_of_u64(gk, n_shards, table) == o)
                if sel.size:
                    f_row[s][sel] = stores[o].get_blocks(pools[s], mb, gk[sel], gi[sel])
        for o in range(n_shards):
            for s in range(world):
                pk, pi = row[s][2], row[s][3]
                sel = np.flatnonzero(shard_of_u64(pk, n_shards, table) == o)
                if sel.size:
                    stores[o].put_blocks(pools[s], mb, pk[sel], pi[sel])
        if step == len(plan) - 1:
            for st in stores:
                st.flush()
        yield pools, f_row, [st.stats() for st in stores]
    for st in stores:
        st.close()


class HostEngine:
    """The engine interface of kvcache_manager.sharded on host memory: an oracle store as the shard
    and numpy arrays as the paged pool; values travel as rows (the "nccl" transport)."""

    def __init__(self, pool, member_bytes: int, store_cfg: dict, grant_limit: int | None = None) -> None:
        self.members = pool
        self.mb = [member_bytes] * len(pool)
        self.header, self.region_bases, self.value_len = O.block_format(self.mb)
        self.store = O.Store(**store_cfg)
        self.device = 0
        self.grant_limit = grant_limit
        self._next_off = 0
        self._granted: dict[int, int] = {}
        self.rounds = 0

    def serve_gets_packed(self, keys, rows):
        found = np.zeros(keys.size, bool)
        for i, k in enumerate(keys):
            found[i] = self.store.get(int(k), rows[i].numpy())
        return found

    def grant_puts(self, keys):
        n = keys.size if self.grant_limit is None else min(keys.size, self.grant_limit)
        offs = np.arange(self._next_off, self._next_off + n, dtype=np.uint64)
        for o, k in zip(offs, keys[:n]):
            self._granted[int(o)] = int(k)
        self._next_off += n
        self.rounds += 1
        return offs, n, 0

    def write_rows(self, rows, offsets):
        for i, o in enumerate(np.asarray(offsets, np.uint64)):
            self.store.put(self._granted.pop(int(o)), rows[i].numpy())

    def puts_landed(self):
        pass

    def gather_rows(self, ids, rows):
        for i, b in enumerate(ids):
            rows[i].numpy()[:] = O.gather([self.members], self.mb, [int(b)], self.region_bases, self.header,
                                          self.value_len)

    def scatter_rows(self, ids, rows, row_index):
        for b, r in zip(ids, row_index):
            O.scatter(rows[int(r)].numpy(), [self.members], self.mb, [int(b)], self.region_bases)

    def exists(self, keys):
        return np.array([self.store.exists(int(k)) for k in keys], bool)

    def flush(self):
        self.store.flush()

    def stats(self):
        return self.store.stats()

    def close(self):
        self.store.close()
