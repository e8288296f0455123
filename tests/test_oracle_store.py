"""Store semantics of the oracle: the reference's put / get / exists / remove / move contract,
eviction policy and hash index invariants (patch 0003 design.md sections 5-7)."""

import numpy as np
import pytest

from oracle import kvs_oracle as O

U = O.UNIT_BYTES


def val(i, n):
    return bytes((i + off) % 256 for off in range(n))  # product_device_smoke.py payload pattern


def test_put_get_exists_delete_roundtrip():
    s = O.Store(max_keys=16, heap_bytes=64 * U)
    s.put(b"a", val(1, 1000))
    assert s.location(b"a")[0] == O.LOC_PENDING  # landed, write-through outstanding
    assert s.exists(b"a")
    assert s.location(b"a")[0] == O.LOC_DEVICE  # EXISTS fused the commit barrier
    assert s.get_bytes(b"a") == val(1, 1000)
    assert not s.exists(b"b")
    assert s.get_bytes(b"b") is None
    assert s.remove(b"a") and not s.exists(b"a") and not s.remove(b"a")


def test_miss_leaves_output_unchanged_and_small_output_fails_before_touching():
    s = O.Store(max_keys=16, heap_bytes=64 * U)
    s.put("k", val(3, 500), sync_commit=True)
    out = np.full(100, 0xA5, np.uint8)
    assert not s.get("missing", out)
    assert (out == 0xA5).all()
    epoch = s.stats()["epoch"]
    with pytest.raises(O.OracleError, match="smaller than the stored value"):
        s.get("k", out)
    assert (out == 0xA5).all()
    assert s.stats()["epoch"] == epoch  # no access stamp for an undersized output


def test_key_validation():
    s = O.Store(max_keys=4, heap_bytes=16 * U)
    with pytest.raises(O.OracleError, match="key must be non-empty"):
        s.put(b"", b"x")
    with pytest.raises(O.OracleError, match="exceeds Server max_key_bytes"):
        s.exists(b"x" * 129)
    with pytest.raises(O.OracleError, match="value_len_bytes must be > 0"):
        s.put(b"k", b"")


def test_move_to_host_and_back_keeps_bytes():
    s = O.Store(max_keys=8, heap_bytes=32 * U)
    s.put("m", val(9, 3 * U + 5), sync_commit=True)
    s.move_to_host("m")
    assert s.location("m")[0] == O.LOC_HOST
    assert s.get_bytes("m") == val(9, 3 * U + 5)  # host serve + read-through admission
    assert s.location("m")[0] == O.LOC_DEVICE
    s.move_to_host("m")
    s.move_to_device("m")
    assert s.location("m")[0] == O.LOC_DEVICE
    assert s.get_bytes("m") == val(9, 3 * U + 5)


def test_lru_evicts_oldest_committed_device_copy_only():
    # heap of 8 units, 2-unit values: 4 fit
    s = O.Store(max_keys=16, heap_bytes=8 * U)
    for i in range(4):
        s.put(i, val(i, 2 * U - 7), sync_commit=True)
    assert s.get_bytes(0) == val(0, 2 * U - 7)  # touch 0: 1 is now the LRU
    s.put(4, val(4, 2 * U - 7), sync_commit=True)
    assert s.location(1)[0] == O.LOC_HOST  # evicted device copy, key retained
    assert all(s.location(k)[0] == O.LOC_DEVICE for k in (0, 2, 3, 4))
    assert s.exists(1) and s.get_bytes(1) == val(1, 2 * U - 7)
    st = s.stats()
    assert st["victims_evicted"] >= 1 and st["live_keys"] == 5


def test_pending_entries_are_pinned_and_force_commits():
    s = O.Store(max_keys=16, heap_bytes=4 * U)
    s.put(1, val(1, 2 * U))
    s.put(2, val(2, 2 * U))  # both pending, heap full
    assert s.stats()["pending_device_bytes"] == 4 * U
    s.put(3, val(3, 2 * U))  # must commit the FIFO head, then evict it
    assert s.location(1)[0] == O.LOC_HOST
    assert s.location(3)[0] == O.LOC_PENDING
    assert s.get_bytes(1) == val(1, 2 * U)


def test_same_key_put_replaces_value():
    s = O.Store(max_keys=8, heap_bytes=16 * U)
    s.put("x", val(1, 100))
    s.put("x", val(2, 5000))  # finds the pending entry: commit, then replace
    assert s.get_bytes("x") == val(2, 5000)
    assert s.stats()["live_keys"] == 1


def test_catalog_replacement_drops_oldest_key():
    s = O.Store(max_keys=3, heap_bytes=64 * U)
    for k in ("a", "b", "c"):
        s.put(k, val(ord(k), 64), sync_commit=True)
    assert s.get_bytes("a")  # a is now most recently accessed
    s.put("d", val(4, 64), sync_commit=True)  # catalog full: replaces b (oldest access epoch)
    assert not s.exists("b")
    assert all(s.exists(k) for k in ("a", "c", "d"))
    assert s.stats()["catalog_replacements"] == 1


def test_hash_index_backward_shift_keeps_lookups_exact():
    rng = np.random.default_rng(0)
    s = O.Store(max_keys=64, heap_bytes=4096 * U)
    keys = [int(x) for x in rng.integers(1, 2**63, 60)]
    for k in keys:
        s.put(k, val(k % 251, 64))
    s.flush()
    live = set(keys)
    for k in rng.permutation(keys)[:40]:
        assert s.remove(int(k))
        live.discard(int(k))
        b = s.buckets()
        # no tombstones; every live key reachable; absent keys miss
        assert not (b[:, 1] == 0xFFFFFFFE).any()
        for q in keys:
            assert (s.index_lookup(q) != O.BUCKET_EMPTY) == (q in live)
    assert (s.buckets()[:, 1] != O.BUCKET_EMPTY).sum() == len(live)


def test_host_pool_first_fit_and_heap_fallback():
    s = O.Store(max_keys=8, heap_bytes=64 * U, host_pool_bytes=4 * U)
    s.put(1, val(1, 3 * U), sync_commit=True)  # 3 units in the pool
    s.put(2, val(2, 2 * U), sync_commit=True)  # does not fit the 1 free unit: heap copy
    st = s.stats()
    assert st["pool_values"] == 1 and st["heap_values"] == 1
    s.remove(1)
    s.put(3, val(3, 4 * U), sync_commit=True)  # the freed extent coalesced to 4 units
    assert s.stats()["pool_values"] == 2
    for k, n in ((2, 2 * U), (3, 4 * U)):
        s.move_to_host(k)
        assert s.get_bytes(k) == val(k, n)


def test_block_put_get_roundtrip_multithreaded():
    rng = np.random.default_rng(5)
    n_layers, seg, pool = 2, 4096, 64
    members = [rng.integers(0, 256, pool * seg, dtype=np.uint8) for _ in range(2 * n_layers)]
    s = O.Store(max_keys=128, heap_bytes=512 * U)
    keys = rng.integers(1, 2**63, 16, dtype=np.uint64)
    src = rng.permutation(pool)[:16]
    s.put_blocks(members, [seg] * 4, keys, src, n_threads=4)
    out = [np.zeros_like(m) for m in members]
    dst = rng.permutation(pool)[:16]
    miss = rng.integers(1, 2**63, 4, dtype=np.uint64)
    found = s.get_blocks(out, [seg] * 4, np.concatenate([keys, miss]), np.concatenate([dst, dst[:4]]), n_threads=4)
    assert found[:16].all() and not found[16:].any()
    for m in range(4):
        for i in range(16):
            assert np.array_equal(out[m][dst[i] * seg:(dst[i] + 1) * seg], members[m][src[i] * seg:(src[i] + 1) * seg])


def test_block_path_under_eviction_serves_host_tier_bytes():
    """get_blocks with host-tier hits and read-through admissions that evict in the same batch."""
    seg, pool = 2 * 16 * 64 * 2, 96
    mb = [seg] * 4
    _, _, vlen = O.block_format(mb)
    units = -(-vlen // U)
    heap = 12 * (1 << (units - 1).bit_length()) * U
    s = O.Store(max_keys=128, heap_bytes=heap, host_pool_bytes=64 << 20)
    rng = np.random.default_rng(7)
    host = [rng.integers(0, 256, pool * seg, dtype=np.uint8) for _ in range(4)]
    keys = rng.integers(1, 2**63, 48, dtype=np.uint64)
    truth = {}
    for r in range(6):
        idx = rng.choice(48, 8, replace=False)
        src = rng.choice(48, 8, replace=False)
        s.put_blocks(host, mb, keys[idx], src)
        for k, b in zip(idx, src):
            truth[int(k)] = [h[b * seg:(b + 1) * seg].copy() for h in host]
        g = rng.choice(48, 12, replace=False)
        dst = 48 + rng.choice(48, 12, replace=False)
        found = s.get_blocks(host, mb, keys[g], dst, n_threads=3)
        for k, d, f in zip(g, dst, found):
            assert f == (int(k) in truth)
            if f:
                for m in range(4):
                    assert np.array_equal(host[m][d * seg:(d + 1) * seg], truth[int(k)][m])
    st = s.stats()
    assert st["admissions"] > 0 and st["victims_evicted"] > 0


def test_forced_commit_lands_the_host_copy_before_its_block_is_reused():
    """A put batch larger than the slab: the forced commit's host copy must be complete before the
    retry evicts that value and reuses its block for the next put of the batch."""
    seg, pool = 1024, 8
    mb = [seg] * 2
    _, _, vlen = O.block_format(mb)
    units = -(-vlen // U)
    s = O.Store(max_keys=16, heap_bytes=2 * (1 << (units - 1).bit_length()) * U, host_pool_bytes=1 << 20)
    rng = np.random.default_rng(3)
    host = [rng.integers(0, 256, pool * seg, dtype=np.uint8) for _ in range(2)]
    keys = np.array([11, 22, 33], np.uint64)
    s.put_blocks(host, mb, keys, [0, 1, 2])  # the third put forces a commit of the first and evicts it
    assert s.location(11)[0] == 1  # host only
    found = s.get_blocks(host, mb, keys[:1], [5])
    assert found.all()
    for m in range(2):
        assert np.array_equal(host[m][5 * seg:6 * seg], host[m][0:seg])
