"""ctypes bindings for the CPU oracle (test infrastructure only).

Every function forwards to oracle/kvs_oracle.c, which restates the reference's hot-path
algorithms (see its header for the citations). `build()` compiles the library with make.
"""

from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "_build" / "libkvs_oracle.so"
_lib = None

LOC_DEVICE, LOC_HOST, LOC_PENDING, ABSENT = 0, 1, 2, -1
BUCKET_EMPTY = 0xFFFFFFFF
MAGIC = 0x524B564E
UNIT_BYTES = 4288


def build() -> Path:
    subprocess.run(["make", "-s", "-C", str(_HERE)], check=True)
    return _LIB_PATH


class _Config(C.Structure):
    _fields_ = [
        ("max_keys", C.c_uint32),
        ("unit_bytes", C.c_uint32),
        ("heap_bytes", C.c_uint64),
        ("max_key_bytes", C.c_uint32),
        ("max_value_bytes", C.c_uint64),
        ("host_pool_bytes", C.c_uint64),
    ]


class _Stats(C.Structure):
    _fields_ = [
        (n, C.c_uint64)
        for n in (
            "live_device_bytes",
            "pending_device_bytes",
            "live_keys",
            "device_resident_keys",
            "allocation_calls",
            "allocation_successes",
            "allocation_failures",
            "victims_evicted",
            "catalog_replacements",
            "writes_through",
            "stale_commits",
            "host_serves",
            "admissions",
            "pool_values",
            "heap_values",
        )
    ] + [("epoch", C.c_uint32), ("issued", C.c_uint32), ("committed", C.c_uint32)]


class Run(C.Structure):
    _fields_ = [
        ("shard_index", C.c_uint32),
        ("device_byte_offset", C.c_uint32),
        ("num_bytes", C.c_uint32),
        ("host_byte_offset", C.c_uint64),
    ]


def lib():
    global _lib
    if _lib is None:
        if not _LIB_PATH.exists() or (
            os.path.getmtime(_HERE / "kvs_oracle.c") > os.path.getmtime(_LIB_PATH)
        ):
            build()
        L = C.CDLL(str(_LIB_PATH))
        P = C.c_void_p
        u32, u64, i64 = C.c_uint32, C.c_uint64, C.c_int64
        sig = {
            "kvo_last_error": (C.c_char_p, []),
            "kvo_fnv1a32": (u32, [P, u32]),
            "kvo_hash_num_buckets": (u32, [u32]),
            "kvo_buddy_order_for_units": (u32, [u32]),
            "kvo_header_words": (u32, [u32, P, P, u32]),
            "kvo_chunk_plan": (u64, [u32, u64, P, P, u32, P]),
            "kvo_gather": (C.c_int, [P, u32, u32, P, P, P, u32, P, P, u32, P, u64]),
            "kvo_scatter": (C.c_int, [P, u64, P, u32, u32, P, P, P, u32, P]),
            "kvo_chunk_slots": (C.c_int, [P, u64, u32, P, P]),
            "kvo_plan_tp_interleaved_runs": (
                C.c_int,
                [P, u64, P, P, P, u64, P, P, u64, i64, i64, i64, i64, i64, i64, P, u64, P],
            ),
            "kvo_apply_runs": (None, [P, u64, P, P, C.c_int]),
            "kvo_store_create": (P, [P]),
            "kvo_store_destroy": (None, [P]),
            "kvo_put": (C.c_int, [P, P, u32, P, u64, C.c_int]),
            "kvo_get": (C.c_int, [P, P, u32, P, u64, P, P]),
            "kvo_exists": (C.c_int, [P, P, u32, P]),
            "kvo_remove": (C.c_int, [P, P, u32, P]),
            "kvo_move_to_host": (C.c_int, [P, P, u32]),
            "kvo_move_to_device": (C.c_int, [P, P, u32]),
            "kvo_flush": (C.c_int, [P]),
            "kvo_location": (C.c_int, [P, P, u32, P]),
            "kvo_get_stats": (None, [P, P]),
            "kvo_index_lookup": (u32, [P, P, u32]),
            "kvo_buckets": (P, [P, P]),
            "kvo_lru_order": (u32, [P, P, u32]),
            "kvo_block_format": (u64, [u32, u32, P, P, u32, P, P]),
            "kvo_put_blocks": (C.c_int, [P, P, u32, u32, P, P, P, u32, C.c_int]),
            "kvo_get_blocks": (C.c_int, [P, P, u32, u32, P, P, P, u32, P, C.c_int]),
            "kvo_paged_fill_varlen": (C.c_int, [P, P, u32, u32, u32, P, u32, P, u32, P, P, P, u32, u32, P]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


class OracleError(RuntimeError):
    pass


def _check(rc: int) -> None:
    if rc != 0:
        raise OracleError(f"[{rc}] {lib().kvo_last_error().decode()}")


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def _u32(x) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(x, dtype=np.uint32))


def _u64(x) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(x, dtype=np.uint64))


def _i64(x) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(x, dtype=np.int64))


def _key(k) -> bytes:
    if isinstance(k, str):
        return k.encode()
    if isinstance(k, (int, np.integer)):
        return int(k).to_bytes(8, "little")
    return bytes(k)


def fnv1a32(data: bytes) -> int:
    b = bytes(data)
    return lib().kvo_fnv1a32(b, len(b))


def hash_num_buckets(max_keys: int) -> int:
    return lib().kvo_hash_num_buckets(max_keys)


def buddy_order_for_units(units: int) -> int:
    return lib().kvo_buddy_order_for_units(units)


def header_words(count: int, sizes) -> np.ndarray:
    sizes = _u32(sizes)
    out = np.zeros(count + 16, np.uint32)
    n = lib().kvo_header_words(count, _ptr(sizes), _ptr(out), out.size)
    return out[:n].copy()


def chunk_plan(n_layers: int, alloc: int):
    words = np.zeros(n_layers + 16, np.uint32)
    nw = C.c_uint32()
    rb = np.zeros(2 * n_layers, np.uint64)
    vlen = lib().kvo_chunk_plan(n_layers, alloc, _ptr(words), C.addressof(nw), words.size, _ptr(rb))
    return words[: nw.value].copy(), rb, int(vlen)


def _ptr_table(arrays) -> np.ndarray:
    return np.array([a.ctypes.data for a in arrays], dtype=np.uint64)


def gather(members, member_bytes, block_ids, region_bases, header, dst_bytes, dst=None):
    """members: list over ranks of list over members of uint8 arrays."""
    n_ranks, n_members = len(members), len(members[0])
    flat = [np.ascontiguousarray(members[r][m]) for r in range(n_ranks) for m in range(n_members)]
    tbl = _ptr_table(flat)
    mb, bid, rb, hdr = _u64(member_bytes), _u32(block_ids), _u64(region_bases), _u32(header)
    extent = _u64([min(flat[r * n_members + m].nbytes for r in range(n_ranks)) for m in range(n_members)])
    if dst is None:
        dst = np.zeros(dst_bytes, np.uint8)
    _check(
        lib().kvo_gather(_ptr(tbl), n_ranks, n_members, _ptr(mb), _ptr(extent), _ptr(bid), bid.size,
                         _ptr(rb), _ptr(hdr) if hdr.size else None, hdr.size, _ptr(dst), dst.nbytes)
    )
    return dst


def scatter(src, members, member_bytes, block_ids, region_bases):
    n_ranks, n_members = len(members), len(members[0])
    flat = [members[r][m] for r in range(n_ranks) for m in range(n_members)]
    for a in flat:
        assert a.flags.c_contiguous and a.dtype == np.uint8
    tbl = _ptr_table(flat)
    mb, bid, rb = _u64(member_bytes), _u32(block_ids), _u64(region_bases)
    extent = _u64([min(flat[r * n_members + m].nbytes for r in range(n_ranks)) for m in range(n_members)])
    src = np.ascontiguousarray(src, dtype=np.uint8)
    _check(
        lib().kvo_scatter(_ptr(src), src.nbytes, _ptr(tbl), n_ranks, n_members, _ptr(mb), _ptr(extent),
                          _ptr(bid), bid.size, _ptr(rb))
    )


def chunk_slots(slots, block_size: int):
    s = _i64(slots)
    fb, nb = C.c_uint64(), C.c_uint64()
    _check(lib().kvo_chunk_slots(_ptr(s) if s.size else None, s.size, block_size, C.addressof(fb), C.addressof(nb)))
    return int(fb.value), int(nb.value)


def plan_runs(slots, starts, ends, memobj_slots, member_alloc_bytes, region_bases, shard_block_bytes,
              block_bytes, block_size, dp_size, blocks_per_dp, tp_size, runs_cap=1 << 16):
    s, st, en, mo = _i64(slots), _i64(starts), _i64(ends), _i64(memobj_slots)
    ma, rb = _i64(member_alloc_bytes), _i64(region_bases)
    n_members = ma.size
    runs = (Run * (runs_cap * n_members))()
    counts = np.zeros(n_members, np.uint64)
    _check(
        lib().kvo_plan_tp_interleaved_runs(
            _ptr(s), s.size, _ptr(st), _ptr(en), _ptr(mo), mo.size, _ptr(ma), _ptr(rb), n_members,
            shard_block_bytes, block_bytes, block_size, dp_size, blocks_per_dp, tp_size,
            C.addressof(runs), runs_cap, _ptr(counts))
    )
    out = []
    for m in range(n_members):
        base = m * runs_cap
        out.append([
            (runs[base + i].shard_index, runs[base + i].device_byte_offset, runs[base + i].num_bytes,
             runs[base + i].host_byte_offset)
            for i in range(int(counts[m]))
        ])
    return out


def apply_runs(runs, shards, host, to_host: bool):
    arr = (Run * max(1, len(runs)))()
    for i, (si, do, nb, ho) in enumerate(runs):
        arr[i] = Run(si, do, nb, ho)
    tbl = _ptr_table(shards)
    lib().kvo_apply_runs(C.addressof(arr), len(runs), _ptr(tbl), _ptr(host), 1 if to_host else 0)


class Store:
    """The oracle store: reference directory, buddy heap, LRU and host tier on host memory."""

    def __init__(self, max_keys=1024, heap_bytes=64 << 20, unit_bytes=UNIT_BYTES, max_key_bytes=128,
                 max_value_bytes=64 << 20, host_pool_bytes=0):
        cfg = _Config(max_keys, unit_bytes, heap_bytes, max_key_bytes, max_value_bytes, host_pool_bytes)
        self._h = lib().kvo_store_create(C.addressof(cfg))
        if not self._h:
            raise OracleError(lib().kvo_last_error().decode())

    def close(self):
        if self._h:
            lib().kvo_store_destroy(self._h)
            self._h = None

    __del__ = close

    def put(self, key, value, sync_commit=False):
        k = _key(key)
        v = np.ascontiguousarray(np.frombuffer(bytes(value), np.uint8) if not isinstance(value, np.ndarray) else value.view(np.uint8).reshape(-1))
        _check(lib().kvo_put(self._h, k, len(k), _ptr(v), v.nbytes, 1 if sync_commit else 0))

    def get(self, key, out: np.ndarray):
        k = _key(key)
        found, vlen = C.c_int(), C.c_uint64()
        _check(lib().kvo_get(self._h, k, len(k), _ptr(out), out.nbytes, C.addressof(found), C.addressof(vlen)))
        return bool(found.value)

    def get_bytes(self, key, capacity=64 << 20):
        out = np.zeros(capacity, np.uint8)
        k = _key(key)
        found, vlen = C.c_int(), C.c_uint64()
        _check(lib().kvo_get(self._h, k, len(k), _ptr(out), out.nbytes, C.addressof(found), C.addressof(vlen)))
        return bytes(out[: vlen.value]) if found.value else None

    def exists(self, key):
        k = _key(key)
        f = C.c_int()
        _check(lib().kvo_exists(self._h, k, len(k), C.addressof(f)))
        return bool(f.value)

    def remove(self, key):
        k = _key(key)
        f = C.c_int()
        _check(lib().kvo_remove(self._h, k, len(k), C.addressof(f)))
        return bool(f.value)

    delete = remove

    def move_to_host(self, key):
        k = _key(key)
        _check(lib().kvo_move_to_host(self._h, k, len(k)))

    def move_to_device(self, key):
        k = _key(key)
        _check(lib().kvo_move_to_device(self._h, k, len(k)))

    def flush(self):
        _check(lib().kvo_flush(self._h))

    def location(self, key):
        k = _key(key)
        off = C.c_uint64()
        loc = lib().kvo_location(self._h, k, len(k), C.addressof(off))
        return loc, int(off.value)

    def index_lookup(self, key):
        k = _key(key)
        return lib().kvo_index_lookup(self._h, k, len(k))

    def stats(self) -> dict:
        st = _Stats()
        lib().kvo_get_stats(self._h, C.addressof(st))
        return {n: getattr(st, n) for n, _ in _Stats._fields_}

    def buckets(self) -> np.ndarray:
        n = C.c_uint32()
        p = lib().kvo_buckets(self._h, C.addressof(n))
        return np.ctypeslib.as_array(C.cast(p, C.POINTER(C.c_uint32)), shape=(n.value, 2)).copy()

    def lru_order(self, cap=1 << 20):
        out = np.zeros(cap, np.uint32)
        n = lib().kvo_lru_order(self._h, _ptr(out), cap)
        return out[:n].copy()

    def put_blocks(self, members, member_bytes, keys, block_ids, members_per_layer=2, n_threads=1):
        tbl = _ptr_table(members)
        mb, k, b = _u64(member_bytes), _u64(keys), _u32(block_ids)
        _check(lib().kvo_put_blocks(self._h, _ptr(tbl), len(members), members_per_layer, _ptr(mb), _ptr(k), _ptr(b),
                                    k.size, n_threads))

    def get_blocks(self, members, member_bytes, keys, block_ids, members_per_layer=2, n_threads=1):
        tbl = _ptr_table(members)
        mb, k, b = _u64(member_bytes), _u64(keys), _u32(block_ids)
        found = np.zeros(k.size, np.uint8)
        _check(lib().kvo_get_blocks(self._h, _ptr(tbl), len(members), members_per_layer, _ptr(mb), _ptr(k), _ptr(b),
                                    k.size, _ptr(found), n_threads))
        return found.astype(bool)


def block_format(member_bytes, members_per_layer=2):
    """(header words, region bases, value length) of one block value."""
    mb = _u64(member_bytes)
    words = np.zeros(mb.size + 16, np.uint32)
    nw = C.c_uint32()
    rb = np.zeros(mb.size, np.uint64)
    vlen = lib().kvo_block_format(mb.size, members_per_layer, _ptr(mb), _ptr(words), words.size, C.addressof(nw), _ptr(rb))
    if not vlen:
        raise OracleError("members must be whole layers")
    return words[: nw.value].copy(), rb, int(vlen)


def paged_fill_varlen(k_fill, v_fill, cu_seqlens, page_table, start_positions, cache_k, cache_v):
    """Token-granular moreh_paged_fill_cache_varlen on numpy arrays, caches updated in place.

    k_fill / v_fill: (heads, total_tokens, head_dim) of any dtype; caches: (num_blocks, heads,
    block_size, head_dim) of the same dtype; cu_seqlens (batch + 1,), page_table (batch,
    max_blocks_per_seq) and start_positions (batch,) int32. Returns the out-of-range token count."""
    heads, total, dim = k_fill.shape
    nb, h2, bs, d2 = cache_k.shape
    assert (h2, d2) == (heads, dim) and v_fill.shape == k_fill.shape and cache_v.shape == cache_k.shape
    for a in (k_fill, v_fill, cache_k, cache_v):
        assert a.flags.c_contiguous and a.dtype == k_fill.dtype
    cu = np.ascontiguousarray(cu_seqlens, np.int32)
    pt = np.ascontiguousarray(page_table, np.int32)
    sp = np.ascontiguousarray(start_positions, np.int32)
    oor = C.c_uint64()
    _check(lib().kvo_paged_fill_varlen(_ptr(k_fill), _ptr(v_fill), heads, total, dim * k_fill.itemsize, _ptr(cu),
                                       pt.shape[0], _ptr(pt), pt.shape[1], _ptr(sp), _ptr(cache_k), _ptr(cache_v),
                                       nb, bs, C.addressof(oor)))
    return int(oor.value)
