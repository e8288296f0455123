"""The oracle against the reference's own directory and planner code, compiled from its sources.

oracle/build_ref.py compiles, from the reference checkout, the helper functions of
dram_worker_kernel.cpp (FNV-1a index with backward-shift delete, buddy heap, residency LRU,
catalog slots, victim selection, eviction, allocation) and the raw-byte run planner into
oracle/_ref/libkvs_ref.so. These tests drive the same operation sequences through that library
and through the oracle and require identical directory state after every operation.
"""

import ctypes as C
from pathlib import Path

import numpy as np
import pytest

from oracle import kvs_oracle as O

LIB = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "libkvs_ref.so"
U = O.UNIT_BYTES

pytestmark = pytest.mark.skipif(not LIB.exists(), reason="oracle/_ref not built (needs the reference checkout)")


@pytest.fixture(scope="module")
def ref():
    L = C.CDLL(str(LIB))
    P = C.c_void_p
    sig = {
        "ref_store_create": (P, [C.c_uint32, C.c_uint32, C.c_uint32]),
        "ref_store_destroy": (None, [P]),
        "ref_fnv1a": (C.c_uint32, [P, C.c_uint32]),
        "ref_store_put": (C.c_int, [P, P, C.c_uint32, C.c_uint32]),
        "ref_store_get": (C.c_int, [P, P, C.c_uint32]),
        "ref_store_remove": (C.c_int, [P, P, C.c_uint32]),
        "ref_store_move_to_host": (None, [P, P, C.c_uint32]),
        "ref_store_move_to_device": (None, [P, P, C.c_uint32]),
        "ref_store_barrier": (None, [P]),
        "ref_store_location": (C.c_int, [P, P, C.c_uint32, P]),
        "ref_store_buckets": (None, [P, P]),
        "ref_store_num_buckets": (C.c_uint32, [P]),
        "ref_store_lru": (C.c_uint32, [P, P, C.c_uint32]),
        "ref_store_counters": (None, [P, P, P, P]),
        "ref_assert_failures": (C.c_ulonglong, []),
        "ref_plan_tp_interleaved_runs": (
            C.c_longlong,
            [P, C.c_uint64, P, P, P, C.c_uint64, P, P, C.c_uint64] + [C.c_int64] * 6 + [P, C.c_uint64, P],
        ),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    return L


def test_fnv1a_matches_reference(ref):
    rng = np.random.default_rng(0)
    for n in [1, 7, 8, 64, 128]:
        for _ in range(50):
            k = rng.integers(0, 256, n, dtype=np.uint8).tobytes()
            assert ref.ref_fnv1a(k, n) == O.fnv1a32(k)


class RefStore:
    def __init__(self, lib, max_keys, heap_bytes):
        self.L = lib
        self.h = lib.ref_store_create(max_keys, heap_bytes, 128)
        assert self.h

    def location(self, key):
        off = C.c_uint32()
        loc = self.L.ref_store_location(self.h, key, len(key), C.byref(off))
        return loc, off.value

    def buckets(self):
        nb = self.L.ref_store_num_buckets(self.h)
        out = np.zeros((nb, 2), np.uint32)
        self.L.ref_store_buckets(self.h, out.ctypes.data)
        return out

    def lru(self, cap=4096):
        out = np.zeros(cap, np.uint32)
        n = self.L.ref_store_lru(self.h, out.ctypes.data, cap)
        return out[:n].tolist()

    def counters(self):
        a, b, c = C.c_uint32(), C.c_uint32(), C.c_uint32()
        self.L.ref_store_counters(self.h, C.byref(a), C.byref(b), C.byref(c))
        return a.value, b.value, c.value


def _compare(o, r, keys):
    for k in keys:
        lo, oo = o.location(k)
        lr, orf = r.location(k)
        assert lo == lr, (k, lo, lr)
        if lo != O.ABSENT and lo != O.LOC_HOST:
            assert oo == orf, (k, oo, orf)
    ob, rb = o.buckets(), r.buckets()
    assert np.array_equal(ob[:, 1], rb[:, 1])
    live = ob[:, 1] != O.BUCKET_EMPTY
    assert np.array_equal(ob[live, 0], rb[live, 0])
    assert o.lru_order().tolist() == r.lru()
    st = o.stats()
    assert (st["live_device_bytes"], st["pending_device_bytes"], st["epoch"]) == r.counters()
    assert r.L.ref_assert_failures() == 0


@pytest.mark.parametrize("seed", range(6))
def test_directory_matches_reference_helpers(ref, seed):
    rng = np.random.default_rng(seed)
    max_keys = int(rng.choice([8, 24, 64]))
    heap_units = int(rng.choice([16, 40, 100]))
    o = O.Store(max_keys=max_keys, heap_bytes=heap_units * U, host_pool_bytes=1 << 20)
    r = RefStore(ref, max_keys, heap_units * U)
    keys = [f"k{i}".encode() for i in range(int(max_keys * 1.5))]
    for step in range(400):
        op = rng.choice(["put", "put", "put", "get", "get", "del", "mth", "mtd", "flush"])
        k = keys[int(rng.integers(len(keys)))]
        if op == "put":
            n = int(rng.choice([1, 100, U, U + 1, 2 * U, 3 * U + 5, 7 * U]))
            rc = ref.ref_store_put(r.h, k, len(k), n)
            try:
                o.put(k, bytes(n))
                assert rc == 0
            except O.OracleError:
                assert rc == -3
        elif op == "get":
            got = o.get_bytes(k, 16 * U) is not None
            assert got == bool(ref.ref_store_get(r.h, k, len(k)))
        elif op == "del":
            assert o.remove(k) == bool(ref.ref_store_remove(r.h, k, len(k)))
        elif op == "mth":
            o.move_to_host(k)
            ref.ref_store_move_to_host(r.h, k, len(k))
        elif op == "mtd":
            o.move_to_device(k)
            ref.ref_store_move_to_device(r.h, k, len(k))
        else:
            o.flush()
            ref.ref_store_barrier(r.h)
        _compare(o, r, keys)
    ref.ref_store_destroy(r.h)


def _ref_plan(ref, slots, starts, ends, mo, ma, rb, sbb, bb, bs, dp, bpd, tp, cap=4096):
    arrs = [np.ascontiguousarray(np.asarray(x, np.int64)) for x in (slots, starts, ends, mo, ma, rb)]
    n_members = len(ma)
    out = np.zeros(5 * n_members * cap, np.uint32)
    counts = np.zeros(n_members, np.uint64)
    rc = ref.ref_plan_tp_interleaved_runs(
        arrs[0].ctypes.data, arrs[0].size, arrs[1].ctypes.data, arrs[2].ctypes.data, arrs[3].ctypes.data, arrs[3].size,
        arrs[4].ctypes.data, arrs[5].ctypes.data, n_members, sbb, bb, bs, dp, bpd, tp, out.ctypes.data, cap,
        counts.ctypes.data)
    if rc < 0:
        return None
    o = out.reshape(n_members, cap, 5)
    return [[(int(x[0]), int(x[1]), int(x[2]), int(x[3]) | (int(x[4]) << 32)) for x in o[m, : int(counts[m])]]
            for m in range(n_members)]


def test_run_planner_matches_reference(ref):
    rng = np.random.default_rng(3)
    checked = invalid = 0
    for trial in range(300):
        tp = int(rng.choice([1, 2, 4]))
        dp = int(rng.choice([1, 2]))
        bs = int(rng.choice([16, 32, 128]))
        bpd = int(rng.integers(4, 12))
        sbb = int(rng.choice([64, 2048, 1088 * 4]))
        bb = sbb * tp
        n_chunks = int(rng.integers(1, 4))
        n_members = int(rng.choice([2, 4, 6]))
        max_blocks = int(rng.integers(1, 4))
        slots, starts, ends = [], [], []
        for c in range(n_chunks):
            nb = int(rng.integers(1, max_blocks + 1))
            first_block = int(rng.integers(0, dp * bpd - nb + 1))
            toks = int(rng.integers(1, nb * bs + 1))
            seq = list(range(first_block * bs, first_block * bs + toks))
            if rng.random() < 0.15 and len(seq) > 1:  # break the slot sequence sometimes
                seq[int(rng.integers(1, len(seq)))] += 1
            starts.append(len(slots))
            slots += seq
            ends.append(len(slots))
        ma = [max_blocks * bb] * n_members
        rb = [m * (n_chunks * max_blocks * bb) for m in range(n_members)]
        mo = list(range(n_chunks))
        exp = _ref_plan(ref, slots, starts, ends, mo, ma, rb, sbb, bb, bs, dp, bpd, tp)
        try:
            got = O.plan_runs(slots, starts, ends, mo, ma, rb, sbb, bb, bs, dp, bpd, tp)
        except O.OracleError:
            got = None
        assert got == exp, trial
        checked += exp is not None
        invalid += exp is None
    assert checked > 100 and invalid > 5
