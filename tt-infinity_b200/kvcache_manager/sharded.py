"""Hash-sharded KV block store across processes: one shard and one paged KV pool per GPU.

The reference serves several server worker groups, each an independent directory, behind one
Fabric endpoint (src/native/ttnn/server_runtime/server.cpp:80-86; the client picks the group).
Here every rank of a torch.distributed job owns one shard (a `Server` on its GPU) and one paged
KV pool, and a 64-bit key belongs to shard fnv1a32(key) % world -- the function the C ABI
applies (`kvs_client_shard_of`).

A step is collective (every rank calls it, possibly with empty batches):

  1. requests: each rank sends its get and put keys (with block ids) to the owning shards in one
     all-to-all of fixed-size records;
  2. gets: each owner runs the commit barrier and serves every requester's gets in one call
     (source-rank order, then batch order) -- a device index probe and one scatter launch that
     stores each hit straight into the requester's pool over NVLink ("p2p": peer pointers from
     CUDA IPC), or into contiguous rows sent back with NCCL send/recv ("nccl", the comparison
     transport);
  3. puts: each owner grants slab offsets in source-rank order; the clients gather their blocks
     straight into the owners' slabs (p2p) or send gathered rows that the owner writes into its
     slab (nccl); after every rank's copies (a stream-ordered barrier) the owners start host
     write-through. A grant that needs the host commit of a value still in flight ends the round;
     the next round grants the rest, so the directory sees the same sequence of prepares and
     forced commits as a single-process put of the same keys in the same order.

Errors (a put that can never fit) travel in the reply records, so every rank takes the same
collective steps; the affected ranks raise after the step.
"""

from __future__ import annotations

import ctypes as C
from typing import Any, Sequence

import numpy as np

from . import _native
from ._facade import Client, PagedLayout, Server, _stream_handle
from ._native import KvsError, check, load

_HDR = 4  # words at the head of every record


PLACEMENT_SLOTS = 4096


def fnv1a32_u64(keys: np.ndarray) -> np.ndarray:
    """fnv1a32 of each 64-bit key's 8 little-endian bytes (the hash the C ABI shards by)."""
    keys = np.ascontiguousarray(np.asarray(keys, dtype=np.uint64))
    b = keys.astype("<u8").view(np.uint8).reshape(-1, 8)
    h = np.full(keys.size, 2166136261, np.uint32)
    prime = np.uint32(16777619)
    for j in range(8):
        h ^= b[:, j]
        h *= prime
    return h


def placement_table(weights: Sequence[float]) -> np.ndarray:
    """Shard of each of PLACEMENT_SLOTS hash slots: contiguous slot ranges sized in proportion to
    the weights (largest remainder, ties to the lower shard), so shard s owns about
    weights[s] / sum(weights) of the keys."""
    w = np.asarray(weights, dtype=np.float64)
    if w.ndim != 1 or w.size == 0 or not np.all(np.isfinite(w)) or np.any(w <= 0):
        raise ValueError("placement weights must be positive and finite, one per shard")
    q = w / w.sum() * PLACEMENT_SLOTS
    n = np.floor(q).astype(np.int64)
    order = np.argsort(-(q - n), kind="stable")
    n[order[:PLACEMENT_SLOTS - int(n.sum())]] += 1
    return np.repeat(np.arange(w.size, dtype=np.int64), n)


def shard_of_u64(keys: np.ndarray, n_shards: int, table: np.ndarray | None = None) -> np.ndarray:
    """Owning shard of each 64-bit key: fnv1a32 of its 8 little-endian bytes mod n_shards, or,
    with a placement table, the table's shard for slot fnv1a32 mod PLACEMENT_SLOTS."""
    keys = np.ascontiguousarray(np.asarray(keys, dtype=np.uint64))
    if table is not None:
        return table[fnv1a32_u64(keys) % np.uint32(PLACEMENT_SLOTS)]
    if n_shards == 1:
        return np.zeros(keys.size, np.int64)
    return (fnv1a32_u64(keys) % np.uint32(n_shards)).astype(np.int64)


def request_words(cap: int) -> int:
    """int64 words of one request record: header + get keys, get ids, put keys, put ids."""
    return _HDR + 4 * cap


def reply_words(cap: int) -> int:
    """int64 words of one reply record: header + get found flags, put slab offsets."""
    return _HDR + 2 * cap


def pack_requests(world: int, cap: int, op: int, get_keys: np.ndarray, get_ids: np.ndarray,
                  put_keys: np.ndarray, put_ids: np.ndarray,
                  table: np.ndarray | None = None) -> tuple[np.ndarray, list, list]:
    """Request records [world, request_words(cap)] (record o goes to shard o) and, per owner, the
    batch positions of its gets and of its puts (in batch order). The keys of both kinds are
    hashed in one pass, then one stable sort by (kind, owner) places every key in its record."""
    rec = np.zeros((world, request_words(cap)), np.int64)
    rec[:, 2] = op
    gk = np.asarray(get_keys, np.uint64).reshape(-1)
    pk = np.asarray(put_keys, np.uint64).reshape(-1)
    ng = gk.size
    keys = np.concatenate([gk, pk])
    ids = np.concatenate([np.asarray(get_ids, np.int64).reshape(-1), np.asarray(put_ids, np.int64).reshape(-1)])
    own = shard_of_u64(keys, world, table)
    group = own.copy()
    group[ng:] += world  # gets of shard o are group o, puts of shard o group world + o
    order = np.argsort(group, kind="stable")
    counts = np.bincount(group, minlength=2 * world)
    if counts.size and counts.max() > cap:
        raise ValueError(f"sharded store: more than {cap} keys for one shard in a step")
    rec[:, 0], rec[:, 1] = counts[:world], counts[world:]
    starts = np.cumsum(counts) - counts
    g = group[order]
    slot = np.arange(order.size) - starts[g]
    o, kind = g % world, g // world
    base = _HDR + 2 * cap * kind + slot
    rec[o, base] = keys.view(np.int64)[order]
    rec[o, base + cap] = ids[order]
    ends = np.cumsum(counts)
    g_pos = [order[starts[i]:ends[i]] for i in range(world)]
    p_pos = [order[starts[world + i]:ends[world + i]] - ng for i in range(world)]
    return rec, g_pos, p_pos


def unpack_requests(recv: np.ndarray, cap: int):
    """Per source rank (in rank order): (get keys u64, get block ids, put keys u64, put block ids)."""
    out = []
    for r in recv:
        ng, npt = int(r[0]), int(r[1])
        out.append((
            r[_HDR:_HDR + ng].view(np.uint64).copy(),
            r[_HDR + cap:_HDR + cap + ng].copy(),
            r[_HDR + 2 * cap:_HDR + 2 * cap + npt].view(np.uint64).copy(),
            r[_HDR + 3 * cap:_HDR + 3 * cap + npt].copy(),
        ))
    return out


class DeviceEngine:
    """The shard and pool of this rank on its GPU, driven through the C ABI (include/kvs.h)."""

    def __init__(self, layout: PagedLayout, **server_cfg: Any) -> None:
        self.layout = layout
        self.device = layout.device
        self.value_len = layout.value_bytes()
        self.payload_per_block = int(sum(layout.member_block_bytes))
        self.server = Server(self.device, **server_cfg)
        self.client = Client(self.device, self.server)
        base, size = C.c_void_p(), C.c_uint64()
        check(load().kvs_server_slab(self.server._handle(), C.byref(base), C.byref(size)))
        self.slab_base, self.slab_bytes = base.value, size.value
        self._peer_slabs: list[int] = []
        self._peer_layouts = None
        self._opened: list[int] = []

    # ---- IPC set-up (collective through `all_gather_object`)
    def export(self) -> dict:
        out = {"slab": self._export_ptr(self.slab_base), "slab_bytes": self.slab_bytes, "members": []}
        for t in self.layout.members:
            out["members"].append(self._export_ptr(t.data_ptr()))
        out["member_block_bytes"] = list(self.layout.member_block_bytes)
        out["members_per_layer"] = self.layout.members_per_layer
        out["num_blocks"] = self.layout.num_blocks
        return out

    @staticmethod
    def _export_ptr(ptr: int) -> tuple[bytes, int]:
        h, off = _native.IpcHandle(), C.c_uint64()
        check(load().kvs_ipc_export(C.c_void_p(ptr), C.byref(h), C.byref(off)))
        return bytes(h.bytes), off.value

    def _open(self, handle: bytes, cache: dict) -> int:
        if handle not in cache:
            h = _native.IpcHandle()
            C.memmove(h.bytes, handle, 64)
            base = C.c_void_p()
            check(load().kvs_ipc_open(self.device, C.byref(h), C.byref(base)))
            cache[handle] = base.value
            self._opened.append(base.value)
        return cache[handle]

    def connect(self, exports: Sequence[dict], rank: int) -> None:
        world = len(exports)
        cache: dict[bytes, int] = {}
        self._slab_bytes = [e["slab_bytes"] for e in exports]
        self._peer_slabs = []
        layouts = (_native.BlockLayout * world)()
        self._keep = []
        for r, e in enumerate(exports):
            if r == rank:
                self._peer_slabs.append(self.slab_base)
                layouts[r] = self.layout.c
                continue
            if e["member_block_bytes"] != list(self.layout.member_block_bytes):
                raise ValueError(f"sharded store: rank {r} has a pool with other member sizes")
            self._peer_slabs.append(self._open(e["slab"][0], cache) + e["slab"][1])
            ptrs = (C.c_uint64 * len(e["members"]))(*[self._open(h, cache) + off for h, off in e["members"]])
            sizes = (C.c_uint64 * len(e["members"]))(*e["member_block_bytes"])
            self._keep += [ptrs, sizes]
            layouts[r] = _native.BlockLayout(len(e["members"]), e["members_per_layer"], ptrs, sizes, e["num_blocks"])
        self._peer_layouts = layouts

    def close_peers(self) -> None:
        for base in self._opened:
            load().kvs_ipc_close(self.device, C.c_void_p(base))
        self._opened = []

    def close(self) -> None:
        self.client.close()
        self.server.close()

    # ---- owner side
    def serve_gets(self, sets: np.ndarray, ids: np.ndarray, keys: np.ndarray) -> np.ndarray:
        n = keys.size
        found = np.zeros(n, np.uint8)
        s = np.ascontiguousarray(sets, np.uint32)
        b = np.ascontiguousarray(ids, np.int64)
        k = np.ascontiguousarray(keys, np.uint64)
        check(load().kvs_serve_gets(
            self.client._handle(), len(self._peer_layouts), self._peer_layouts, n, s.ctypes.data_as(_native._u32p),
            b.ctypes.data_as(_native._i64p), k.ctypes.data_as(_native._u64p), found.ctypes.data_as(_native._u8p),
            _stream_handle(self.device)))
        return found.astype(bool)

    def serve_gets_packed(self, keys: np.ndarray, rows) -> np.ndarray:
        n = keys.size
        found = np.zeros(n, np.uint8)
        k = np.ascontiguousarray(keys, np.uint64)
        check(load().kvs_serve_gets_packed(
            self.client._handle(), C.c_void_p(rows.data_ptr() if n else 0), self.value_len, n,
            k.ctypes.data_as(_native._u64p), found.ctypes.data_as(_native._u8p), _stream_handle(self.device)))
        return found.astype(bool)

    def grant_puts(self, keys: np.ndarray) -> tuple[np.ndarray, int, int]:
        """(slab offsets, number granted, error code)."""
        n = keys.size
        offs = np.zeros(n, np.uint64)
        ng = C.c_uint32()
        k = np.ascontiguousarray(keys, np.uint64)
        rc = load().kvs_grant_puts(self.client._handle(), n, k.ctypes.data_as(_native._u64p), self.value_len,
                                   offs.ctypes.data_as(_native._u64p), C.byref(ng))
        if rc != _native.OK:
            self.last_error = load().kvs_last_error().decode(errors="replace")
        return offs, ng.value, rc

    def puts_landed(self) -> None:
        check(load().kvs_puts_landed(self.client._handle(), _stream_handle(self.device)))

    def write_rows(self, rows, offsets: np.ndarray) -> None:
        """Owner (nccl transport): received value rows -> their slab offsets."""
        n = offsets.size
        if n == 0:
            return
        addrs = np.ascontiguousarray(np.asarray(offsets, np.uint64) + np.uint64(self.slab_base))
        check(load().kvs_copy_values(self.client._handle(), C.c_void_p(rows.data_ptr()), self.value_len, n,
                                     addrs.ctypes.data_as(_native._u64p), 0, _stream_handle(self.device)))

    # ---- client side
    def push_puts(self, ids: np.ndarray, owners: np.ndarray, offsets: np.ndarray) -> None:
        """Gather the blocks straight into the owners' slabs (P2P stores over NVLink)."""
        n = ids.size
        if n == 0:
            return
        slabs = np.asarray(self._peer_slabs, np.uint64)
        sizes = np.asarray(self._slab_bytes, np.uint64)
        offsets = np.asarray(offsets, np.uint64)
        if np.any(offsets + np.uint64(self.value_len) > sizes[owners]):
            raise KvsError(_native.E_INVAL, "sharded store: a granted offset lies outside the owner's slab")
        addrs = np.ascontiguousarray(slabs[owners] + offsets)
        b = np.ascontiguousarray(ids, np.int64)
        check(load().kvs_copy_blocks(self.client._handle(), C.byref(self.layout.c), n, b.ctypes.data_as(_native._i64p),
                                     addrs.ctypes.data_as(_native._u64p), 1, _stream_handle(self.device)))

    def _rows_copy(self, ids: np.ndarray, rows, to_blob: int, row_index: np.ndarray | None = None) -> None:
        n = ids.size
        if n == 0:
            return
        base = rows.data_ptr()
        r = np.arange(n, dtype=np.uint64) if row_index is None else np.asarray(row_index, np.uint64)
        addrs = np.ascontiguousarray(np.uint64(base) + r * np.uint64(self.value_len))
        b = np.ascontiguousarray(ids, np.int64)
        check(load().kvs_copy_blocks(self.client._handle(), C.byref(self.layout.c), n, b.ctypes.data_as(_native._i64p),
                                     addrs.ctypes.data_as(_native._u64p), to_blob, _stream_handle(self.device)))

    def gather_rows(self, ids: np.ndarray, rows) -> None:
        self._rows_copy(ids, rows, 1)

    def scatter_rows(self, ids: np.ndarray, rows, row_index: np.ndarray) -> None:
        """Rows row_index[i] -> pool block ids[i]."""
        self._rows_copy(ids, rows, 0, row_index)

    def flush(self) -> None:
        self.client.flush()

    def exists(self, keys: np.ndarray) -> np.ndarray:
        return self.client.exists_batch(keys) if keys.size else np.zeros(0, bool)

    def stats(self) -> dict:
        return self.server.stats()


class _GpuBucketing:
    """The step's request records built on the GPU (kvs_bucket_requests) of a store on NCCL ranks:
    keys and block ids go up in one pinned copy each, one kernel buckets them by owner into the
    all-to-all's send records, and the received records come back to the host in one copy together
    with this rank's batch positions per owner."""

    def __init__(self, store: "ShardedStore") -> None:
        torch = store._torch
        w, cap, dev = store.world, store.cap, store._dev
        self.store = store
        self.n_max = 2 * w * cap
        self.h_keys = torch.empty(self.n_max, dtype=torch.int64).pin_memory()
        self.h_ids = torch.empty(self.n_max, dtype=torch.int64).pin_memory()
        self.d_keys = torch.empty(self.n_max, dtype=torch.int64, device=dev)
        self.d_ids = torch.empty(self.n_max, dtype=torch.int64, device=dev)
        self.rec_words = request_words(cap)
        self.send = torch.empty(w * self.rec_words, dtype=torch.int64, device=dev)
        # one buffer comes back: received records, then back [w][2][cap] int32, counts [2][w] int32
        # and the overflow word (int32 views of its int64 tail)
        self.r_words = w * self.rec_words
        tail = (2 * w * cap + 2 * w + 2 + 1) // 2
        self.out = torch.zeros(self.r_words + tail, dtype=torch.int64, device=dev)
        t32 = self.out[self.r_words:].view(torch.int32)
        self.back = t32[:2 * w * cap]
        self.counts = t32[2 * w * cap:2 * w * cap + 2 * w]
        self.overflow = t32[2 * w * cap + 2 * w:2 * w * cap + 2 * w + 1]
        self.table = None
        if store.table is not None:
            self.table = torch.from_numpy(np.ascontiguousarray(store.table, dtype=np.int32)).to(dev)

    def exchange(self, op: int, gk: np.ndarray, gi: np.ndarray, pk: np.ndarray, pi: np.ndarray):
        st = self.store
        torch, w, cap = st._torch, st.world, st.cap
        ng, n = gk.size, gk.size + pk.size
        if n > self.n_max:
            raise ValueError(f"sharded store: more than {cap} keys for one shard in a step")
        hk, hi = self.h_keys.numpy(), self.h_ids.numpy()
        hk[:ng], hk[ng:n] = gk.view(np.int64), pk.view(np.int64)
        hi[:ng], hi[ng:n] = gi, pi
        if n:
            self.d_keys[:n].copy_(self.h_keys[:n], non_blocking=True)
            self.d_ids[:n].copy_(self.h_ids[:n], non_blocking=True)
        stream = torch.cuda.current_stream(st._dev).cuda_stream
        ptr = lambda t: C.c_void_p(t.data_ptr())
        check(load().kvs_bucket_requests(
            st.engine.device, ptr(self.d_keys), ptr(self.d_ids), n, ng,
            ptr(self.table) if self.table is not None else None, w, cap, op, ptr(self.send), ptr(self.back),
            ptr(self.counts), ptr(self.overflow), C.c_void_p(stream)))
        st.dist.all_to_all_single(self.out[:self.r_words], self.send, group=st.group)
        host = self.out.cpu().numpy()
        t32 = host[self.r_words:].view(np.int32)
        back = t32[:2 * w * cap].reshape(w, 2, cap)
        counts = t32[2 * w * cap:2 * w * cap + 2 * w].reshape(2, w)
        if t32[2 * w * cap + 2 * w]:
            raise ValueError(f"sharded store: more than {cap} keys for one shard in a step")
        reqs = unpack_requests(host[:self.r_words].reshape(w, self.rec_words), cap)
        g_pos = [back[o, 0, :counts[0, o]].astype(np.int64) for o in range(w)]
        p_pos = [back[o, 1, :counts[1, o]].astype(np.int64) for o in range(w)]
        return reqs, g_pos, p_pos


class ShardedStore:
    """Collective put / get / exists of paged KV blocks over a store sharded one shard per rank.

    Every rank calls every method with its own batch (possibly empty). `transport` "p2p" moves
    block bytes with copy kernels over NVLink peer memory; "nccl" moves contiguous rows with
    NCCL send/recv (the comparison transport)."""

    def __init__(self, engine: Any, *, max_batch: int = 256, transport: str = "p2p", group=None,
                 weights: Sequence[float] | None = None) -> None:
        import torch
        import torch.distributed as dist

        if transport not in ("p2p", "nccl"):
            raise ValueError(f"transport must be 'p2p' or 'nccl', not {transport!r}")
        self.dist = dist
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        # key placement: fnv1a32 mod world, or slots in proportion to per-shard weights (the same
        # on every rank, e.g. each GPU's device->host rate, which bounds its write-through)
        self.table = None
        if weights is not None:
            w = [float(x) for x in weights]
            if len(w) != self.world:
                raise ValueError(f"sharded store: {len(w)} placement weights for {self.world} shards")
            seen: list = [None] * self.world
            dist.all_gather_object(seen, w, group=group)
            if any(x != w for x in seen):
                raise ValueError("sharded store: placement weights differ between ranks")
            self.table = placement_table(w)
        self.engine = engine
        self.engine._rank = self.rank
        self.cap = int(max_batch)
        self.transport = transport
        self.value_len = engine.value_len
        self._cuda = dist.get_backend(group) == "nccl"
        self._dev = torch.device("cuda", engine.device) if self._cuda else torch.device("cpu")
        self._torch = torch
        if transport == "p2p":
            exports: list = [None] * self.world
            dist.all_gather_object(exports, engine.export(), group=group)
            engine.connect(exports, self.rank)
        self._token = torch.zeros(1, dtype=torch.int32, device=self._dev)
        self._rows_out = None
        self._rows_in = None
        self._bucket = _GpuBucketing(self) if self._cuda else None
        self.steps = 0
        # blocks moved by this rank: as a client (puts sent, gets found) and as an owner (gets
        # served); "remote" ones crossed to or from another GPU
        self.counters = dict(puts=0, puts_remote=0, gets=0, gets_found=0, served=0, served_remote=0,
                             grant_rounds=0)
        self.closed = False

    # ---- collectives
    def _requests(self, op: int, gk: np.ndarray, gi: np.ndarray, pk: np.ndarray, pi: np.ndarray):
        """Request records exchanged with every rank: per source rank (get keys, get ids, put keys,
        put ids), and per owner the batch positions of this rank's gets and puts. On GPUs the keys
        are bucketed on the device and the records go to the all-to-all from device memory; on CPU
        ranks pack_requests buckets them with numpy."""
        if self._bucket is not None:
            return self._bucket.exchange(op, gk, gi, pk, pi)
        send, g_pos, p_pos = pack_requests(self.world, self.cap, op, gk, gi, pk, pi, self.table)
        return unpack_requests(self._alltoall(send), self.cap), g_pos, p_pos

    def _alltoall(self, send: np.ndarray) -> np.ndarray:
        torch = self._torch
        s = torch.from_numpy(np.ascontiguousarray(send)).reshape(-1)
        if self._cuda:
            s = s.pin_memory().to(self._dev, non_blocking=True)
        r = torch.empty_like(s)
        self.dist.all_to_all_single(r, s, group=self.group)
        return r.cpu().numpy().reshape(send.shape)

    def _barrier(self) -> None:
        """Stream-ordered barrier: every rank's copies issued so far finish before later work."""
        if self._cuda:
            self.dist.all_reduce(self._token, group=self.group)
        else:
            self.dist.barrier(group=self.group)

    def _rows(self, which: str, n: int):
        torch = self._torch
        cur = getattr(self, which)
        if cur is None or cur.shape[0] < n:
            cur = torch.empty((max(n, 1), self.value_len), dtype=torch.uint8, device=self._dev)
            setattr(self, which, cur)
        return cur

    def _exchange_rows(self, send_rows, send_counts: Sequence[int], recv_rows, recv_counts: Sequence[int]) -> None:
        """Row blocks between ranks: rows [sum(send_counts[:p]) ...) go to rank p, rows from rank p
        land at [sum(recv_counts[:p]) ...)."""
        dist = self.dist
        so = np.concatenate([[0], np.cumsum(send_counts)]).astype(int)
        ro = np.concatenate([[0], np.cumsum(recv_counts)]).astype(int)
        ops = []
        for p in range(self.world):
            if p == self.rank:
                if send_counts[p]:
                    recv_rows[ro[p]:ro[p + 1]].copy_(send_rows[so[p]:so[p + 1]])
                continue
            if send_counts[p]:
                ops.append(dist.P2POp(dist.isend, send_rows[so[p]:so[p + 1]], p, group=self.group))
            if recv_counts[p]:
                ops.append(dist.P2POp(dist.irecv, recv_rows[ro[p]:ro[p + 1]], p, group=self.group))
        if ops:
            for w in dist.batch_isend_irecv(ops):
                w.wait()
            if self._cuda:
                # the work handles of a batched send/recv do not order this process's later
                # streams after the transfer (a copy launched next read the rows before they
                # arrived); a device synchronize does
                self._torch.cuda.synchronize(self._dev)

    # ---- public API
    def step(self, get_keys: Any = (), get_ids: Any = (), put_keys: Any = (), put_ids: Any = ()) -> np.ndarray:
        """Gets (against the state before this step's puts) then puts; returns the found flags of
        the gets in batch order."""
        gk = np.ascontiguousarray(np.asarray(get_keys, dtype=np.uint64).reshape(-1))
        gi = np.ascontiguousarray(np.asarray(get_ids, dtype=np.int64).reshape(-1))
        pk = np.ascontiguousarray(np.asarray(put_keys, dtype=np.uint64).reshape(-1))
        pi = np.ascontiguousarray(np.asarray(put_ids, dtype=np.int64).reshape(-1))
        if gk.size != gi.size or pk.size != pi.size:
            raise ValueError("sharded store: keys and block ids must have equal length")
        if self.closed:
            raise KvsError(_native.E_CLOSED, "sharded store is closed")
        world, cap, eng = self.world, self.cap, self.engine
        reqs, g_pos, p_pos = self._requests(0, gk, gi, pk, pi)
        # ---- owner: gets of every source, in source-rank order
        n_get = [r[0].size for r in reqs]
        g_keys = np.concatenate([r[0] for r in reqs]) if sum(n_get) else np.zeros(0, np.uint64)
        g_ids = np.concatenate([r[1] for r in reqs]) if sum(n_get) else np.zeros(0, np.int64)
        g_sets = np.repeat(np.arange(world, dtype=np.uint32), n_get)
        if self.transport == "p2p":
            found = eng.serve_gets(g_sets, g_ids, g_keys)
        else:
            out_rows = self._rows("_rows_out", g_keys.size)
            found = eng.serve_gets_packed(g_keys, out_rows[:g_keys.size])
        c = self.counters
        c["served"] += int(found.sum())
        c["served_remote"] += int(found[g_sets != self.rank].sum())
        # ---- owner: first round of put grants
        put_keys_by_src = [r[2] for r in reqs]
        put_ids_by_src = [r[3] for r in reqs]
        all_put = np.concatenate(put_keys_by_src) if sum(k.size for k in put_keys_by_src) else np.zeros(0, np.uint64)
        src_of_put = np.repeat(np.arange(world), [k.size for k in put_keys_by_src])
        cursor, status = 0, 0
        offs_all = np.zeros(all_put.size, np.uint64)

        def grant_round() -> tuple[np.ndarray, int]:
            nonlocal cursor, status
            if status != 0 or cursor >= all_put.size:
                return np.zeros(0, np.int64), 0
            offs, ng, rc = eng.grant_puts(all_put[cursor:])
            offs_all[cursor:cursor + ng] = offs[:ng]
            idx = np.arange(cursor, cursor + ng)
            cursor += ng
            if rc != _native.OK:
                status = rc
            return idx, int(cursor < all_put.size and status == 0)

        granted, more = grant_round()
        reply = np.zeros((world, reply_words(cap)), np.int64)
        base = np.concatenate([[0], np.cumsum(n_get)]).astype(int)
        for s in range(world):
            reply[s, 0] = status
            reply[s, 1] = more
            reply[s, _HDR:_HDR + n_get[s]] = found[base[s]:base[s + 1]]
        self._fill_grants(reply, granted, src_of_put, offs_all, put_keys_by_src)
        back = self._alltoall(reply)
        # ---- client: gets found flags (batch order)
        my_found = np.zeros(gk.size, bool)
        for o in range(world):
            my_found[g_pos[o]] = back[o, _HDR:_HDR + g_pos[o].size] != 0
        if self.transport == "nccl":
            send_counts = n_get  # rows served by this owner, per requester
            recv_counts = [g_pos[o].size for o in range(world)]
            in_rows = self._rows("_rows_in", gk.size)
            self._exchange_rows(out_rows, send_counts, in_rows, recv_counts)
            order = np.concatenate(g_pos) if gk.size else np.zeros(0, np.int64)
            # rows of misses hold nothing: scatter the hits only
            sel = np.flatnonzero(my_found[order])
            eng.scatter_rows(gi[order][sel], in_rows, sel)
        c["gets"] += gk.size
        c["gets_found"] += int(my_found.sum())
        c["puts"] += pk.size
        c["puts_remote"] += int(sum(p_pos[o].size for o in range(world) if o != self.rank))
        # ---- put rounds
        p_cursor = [0] * world  # per owner: puts of this rank granted so far
        while True:
            c["grant_rounds"] += 1
            ids, owners, offs, counts = [], [], [], [0] * world
            for o in range(world):
                ng = int(back[o, 2])
                if ng:
                    sel = p_pos[o][p_cursor[o]:p_cursor[o] + ng]
                    ids.append(pi[sel])
                    owners.append(np.full(ng, o, np.int64))
                    offs.append(back[o, _HDR + cap + p_cursor[o]:_HDR + cap + p_cursor[o] + ng].view(np.uint64))
                    p_cursor[o] += ng
                    counts[o] = ng
            ids_a = np.concatenate(ids) if ids else np.zeros(0, np.int64)
            own_a = np.concatenate(owners) if owners else np.zeros(0, np.int64)
            offs_a = np.concatenate(offs) if offs else np.zeros(0, np.uint64)
            if self.transport == "p2p":
                eng.push_puts(ids_a, own_a, offs_a)
                self._barrier()
            else:
                out_rows = self._rows("_rows_out", ids_a.size)
                eng.gather_rows(ids_a, out_rows[:ids_a.size])
                n_recv = granted.size
                recv_counts = [int(np.count_nonzero(src_of_put[granted] == s)) for s in range(world)]
                in_rows = self._rows("_rows_in", n_recv)
                self._exchange_rows(out_rows, counts, in_rows, recv_counts)
                eng.write_rows(in_rows[:n_recv], offs_all[granted])
            eng.puts_landed()
            if not np.any(back[:, 1]):
                break
            granted, more = grant_round()
            reply = np.zeros((world, reply_words(cap)), np.int64)
            reply[:, 0] = status
            reply[:, 1] = more
            self._fill_grants(reply, granted, src_of_put, offs_all, put_keys_by_src)
            back = self._alltoall(reply)
        self.steps += 1
        failed = [o for o in range(world) if p_cursor[o] < p_pos[o].size]
        if failed:
            raise KvsError(int(back[failed[0], 0]) or _native.E_NOSPACE,
                           f"sharded put: {sum(p_pos[o].size - p_cursor[o] for o in failed)} blocks were not "
                           f"stored (no device-cache space on shards {failed})")
        return my_found

    def _fill_grants(self, reply, granted, src_of_put, offs_all, put_keys_by_src) -> None:
        """Per source: the number granted this round (word 2) and their offsets, written after the
        ones granted in earlier rounds (the source keeps a cursor per owner)."""
        cap = self.cap
        starts = np.concatenate([[0], np.cumsum([k.size for k in put_keys_by_src])]).astype(int)
        for s in range(self.world):
            sel = granted[src_of_put[granted] == s] if granted.size else granted
            reply[s, 2] = sel.size
            if sel.size:
                pos = sel - starts[s]  # positions in this source's put list
                reply[s, _HDR + cap + pos] = offs_all[sel].view(np.int64)

    def put_blocks(self, keys: Any, block_ids: Any) -> None:
        self.step((), (), keys, block_ids)

    def get_blocks(self, keys: Any, block_ids: Any) -> np.ndarray:
        return self.step(keys, block_ids, (), ())

    def exists_batch(self, keys: Any) -> np.ndarray:
        """Collective exists of this rank's keys (commit barrier on every owner first)."""
        k = np.ascontiguousarray(np.asarray(keys, dtype=np.uint64).reshape(-1))
        world, cap = self.world, self.cap
        reqs, g_pos, _ = self._requests(1, k, np.zeros(k.size, np.int64), np.zeros(0, np.uint64),
                                        np.zeros(0, np.int64))
        n = [r[0].size for r in reqs]
        keys_all = np.concatenate([r[0] for r in reqs]) if sum(n) else np.zeros(0, np.uint64)
        found = self.engine.exists(keys_all)
        reply = np.zeros((world, reply_words(cap)), np.int64)
        base = np.concatenate([[0], np.cumsum(n)]).astype(int)
        for s in range(world):
            reply[s, _HDR:_HDR + n[s]] = found[base[s]:base[s + 1]]
        back = self._alltoall(reply)
        out = np.zeros(k.size, bool)
        for o in range(world):
            out[g_pos[o]] = back[o, _HDR:_HDR + g_pos[o].size] != 0
        return out

    def flush(self) -> None:
        """Commit every landed put of this rank's shard to the host tier."""
        self.engine.flush()

    def stats(self) -> dict:
        return self.engine.stats()

    def close(self) -> None:
        """Collective: unmap the peers' memory everywhere before any shard frees its slab."""
        if self.closed:
            return
        self.closed = True
        if self._cuda:
            self._torch.cuda.synchronize(self._dev)
        if hasattr(self.engine, "close_peers"):
            self.engine.close_peers()
        self.dist.barrier(group=self.group)
        self.engine.close()


def create(layout: PagedLayout, *, max_batch: int = 256, transport: str = "p2p", group=None,
           weights: Sequence[float] | None = None, **server_cfg: Any) -> ShardedStore:
    """A sharded store whose shard on this rank lives on the layout's GPU (collective)."""
    return ShardedStore(DeviceEngine(layout, **server_cfg), max_batch=max_batch, transport=transport, group=group,
                        weights=weights)
