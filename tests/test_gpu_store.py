"""The B200 store (CUDA path through the C ABI) against the oracle, bit-exact.

Covers the reference's put / get / exists / delete / move contract (tests/product_device_smoke.py
and tests/device/*.py of the reference), the batched paged-block path on the config-1 shape, the
directory policy (residency, LRU order, hash buckets) under eviction pressure, and the host tier.
"""

import numpy as np
import pytest
import torch

from kvcache_manager import Client, KvsError, PagedLayout, Server, codec
from oracle import kvs_oracle as O

pytestmark = [pytest.mark.gpu, pytest.mark.usefixtures("copy_engine")]

U = 4288
LOC = {0: "device", 1: "host", 2: "pending", -1: "absent"}


def payload(i, n):
    return bytes((i + off) % 256 for off in range(n))


def dev_bytes(b: bytes, pad=0):
    t = torch.frombuffer(bytearray(b) + bytearray(pad), dtype=torch.uint8)
    return t.cuda()


def kv_pool(n_layers, heads, bs, dim, n_blocks, dtype=torch.bfloat16, seed=0):
    g = torch.Generator().manual_seed(seed)
    layers = []
    for _ in range(n_layers):
        pair = []
        for _ in range(2):
            x = torch.randn((n_blocks, heads, bs, dim), generator=g, dtype=torch.float32).to(dtype)
            pair.append(x.cuda())
        layers.append(tuple(pair))
    return layers


@pytest.fixture
def store():
    made = []

    def make(**kw):
        kw.setdefault("max_keys", 256)
        kw.setdefault("heap_bytes", 256 * U)
        kw.setdefault("host_pool_bytes", 64 << 20)
        s = Server(0, **kw)
        c = Client(0, s)
        made.append((c, s))
        return c, s

    yield make
    for c, s in made:
        c.close()
        s.close()


def test_product_smoke_sequence(store):
    """put / exists / get / move_to_host / get / move_to_device / get / delete (product smoke)."""
    c, s = store()
    assert c.ping(bytes(range(64))) == bytes(range(64))
    for it, n in enumerate([1, 31, 4288, 4289, 65536 + 7, 3 * 4288 + 1]):
        key = f"smoke-{it}".encode()
        data = payload(it, n)
        val = dev_bytes(data)
        out = torch.zeros(n + 100, dtype=torch.uint8, device="cuda")
        sync = it % 2 == 1
        c.put(key, val, n, sync_commit=sync)
        if not sync:
            c.flush()
        assert c.exists(key)
        assert c.get(key, out) and out[:n].cpu().numpy().tobytes() == data
        assert not out[n:].any(), "bytes past the value must stay unchanged"
        c.move_to_host(key)
        assert s.location(key)[0] == 1
        out.zero_()
        assert c.get(key, out) and out[:n].cpu().numpy().tobytes() == data
        c.move_to_host(key)
        c.move_to_device(key)
        assert s.location(key)[0] == 0
        out.zero_()
        assert c.get(key, out) and out[:n].cpu().numpy().tobytes() == data
        assert c.delete(key) and not c.exists(key)


def test_errors_match_reference_messages(store):
    c, s = store()
    v = dev_bytes(b"x" * 64)
    with pytest.raises(KvsError, match="key must be non-empty"):
        c.exists(b"")
    with pytest.raises(KvsError, match="exceeds Server max_key_bytes"):
        c.exists(b"x" * 129)
    with pytest.raises(KvsError, match="value_len_bytes must be > 0"):
        c.put(b"k", v, 0)
    with pytest.raises(RuntimeError, match="must use DEVICE storage"):
        c.put(b"k", torch.zeros(8, dtype=torch.uint8), 8)
    with pytest.raises(RuntimeError, match="exceeds tensor packed bytes"):
        c.put(b"k", v, 65)
    c.put(b"k", v, 64, sync_commit=True)
    small = torch.full((16,), 0xA5, dtype=torch.uint8, device="cuda")
    with pytest.raises(KvsError, match="smaller than the stored value"):
        c.get(b"k", small)
    assert (small == 0xA5).all()
    assert not c.get(b"missing", small) and (small == 0xA5).all()
    assert c.ping(b"after-invalid") == b"after-invalid"
    assert c.exists("k") and c.exists(b"k")  # str and bytes name the same key


def test_exists_waits_for_async_put_commit(store):
    c, s = store()
    c.put(b"delayed-commit", dev_bytes(payload(1, 256)), 256, sync_commit=False)
    issued, committed = s._test_put_drain_progress()
    assert issued != committed
    assert c.exists(b"delayed-commit")
    assert s._test_put_drain_progress() == (issued, issued)


def test_config1_block_roundtrip(store):
    """2 layers x 8 heads x 128 dim bf16, 32-token blocks, 1024-block pool; 64 blocks put, exists on
    64 hits + 64 misses, get into 64 fresh slots, bit-exact."""
    c, s = store(max_keys=1024, heap_bytes=64 * 16 * 4288 * 4, host_pool_bytes=64 << 20)
    kv = kv_pool(2, 8, 32, 128, 1024, seed=1)
    layout = PagedLayout.from_kv_caches(kv)
    rng = np.random.default_rng(1)
    perm = rng.permutation(1024)
    src, dst = perm[:64], perm[64:128]
    keys = codec.chained_block_hashes(1234, 64)
    c.put_blocks(layout, keys, src)
    misses = codec.chained_block_hashes(999, 64)
    found = c.exists_batch(list(keys) + list(misses))
    assert found[:64].all() and not found[64:].any()
    snapshot = [t.clone() for pair in kv for t in pair]
    got = c.get_blocks(layout, keys, dst)
    assert got.all()
    members = [t for pair in kv for t in pair]
    untouched = torch.as_tensor(np.setdiff1d(np.arange(1024), dst), device="cuda")
    for m, t in enumerate(members):
        bits, ref = t.view(torch.int16), snapshot[m].view(torch.int16)  # bitwise, not float compare
        assert torch.equal(bits[torch.as_tensor(dst, device="cuda")], ref[torch.as_tensor(src, device="cuda")])
        assert torch.equal(bits[untouched], ref[untouched])
    # the stored value is the reference blob of one block: check against the oracle's gather
    seg = 8 * 32 * 128 * 2
    words, rb, vlen = O.chunk_plan(2, seg)
    assert vlen == layout.value_bytes()
    out = torch.zeros(vlen, dtype=torch.uint8, device="cuda")
    assert c.get(int(keys[5]), out)
    host = [[t.view(torch.uint8).reshape(-1).cpu().numpy() for t in snapshot]]
    ref = O.gather(host, [seg] * 4, [int(src[5])], rb, words, vlen)
    assert np.array_equal(out.cpu().numpy(), ref)


def test_get_blocks_miss_leaves_blocks_untouched(store):
    c, s = store()
    kv = kv_pool(2, 2, 16, 64, 32, seed=3)
    layout = PagedLayout.from_kv_caches(kv)
    before = [t.clone() for p in kv for t in p]
    found = c.get_blocks(layout, [11, 12, 13], [0, 1, 2])
    assert not found.any()
    assert all(torch.equal(a, b) for a, b in zip(before, [t for p in kv for t in p]))


@pytest.mark.parametrize("n_keys", [1, 6])
def test_get_blocks_of_a_value_of_another_length_is_a_format_error(store, n_keys):
    """A key whose stored value is not one block of the layout: get_blocks reports it and writes
    nothing for it (n_keys = 1 takes the one-launch probe+scatter path)."""
    c, s = store()
    kv = kv_pool(2, 2, 16, 64, 32, seed=4)
    layout = PagedLayout.from_kv_caches(kv)
    c.put(5, dev_bytes(payload(5, 1000)), 1000, sync_commit=True)
    before = [t.clone() for p in kv for t in p]
    keys = [5] + list(range(100, 100 + n_keys - 1))
    with pytest.raises(KvsError, match="block layout needs"):
        c.get_blocks(layout, keys, list(range(n_keys)))
    assert all(torch.equal(a, b) for a, b in zip(before, [t for p in kv for t in p]))


def test_fp8_with_per_block_scales_roundtrip(store):
    """Config-5 style layout: per layer K, V fp8 e4m3 (16-token blocks) plus one fp32 scale per block."""
    c, s = store(max_keys=512, heap_bytes=2048 * U)
    n_layers, nb = 8, 512
    g = torch.Generator().manual_seed(5)
    members = []
    for _ in range(n_layers):
        for _ in range(2):
            members.append(torch.randn((nb, 8, 16, 128), generator=g).to(torch.float8_e4m3fn).cuda())
        members.append(torch.rand((nb,), generator=g).cuda())
    layout = PagedLayout(members, members_per_layer=3)
    rng = np.random.default_rng(5)
    perm = rng.permutation(nb)
    src, dst = perm[:100], perm[100:200]
    keys = codec.chained_block_hashes(55, 100)
    c.put_blocks(layout, keys, src)
    snap = [t.clone() for t in members]
    assert c.get_blocks(layout, keys, dst).all()
    for a, b in zip(members, snap):
        ab, bb = a.view(torch.uint8).reshape(nb, -1), b.view(torch.uint8).reshape(nb, -1)
        assert torch.equal(ab[torch.as_tensor(dst).cuda()], bb[torch.as_tensor(src).cuda()])
    # value format against the oracle
    mb = layout.member_block_bytes
    words, rb, vlen = O.block_format(mb, 3)
    assert vlen == layout.value_bytes()
    out = torch.zeros(vlen, dtype=torch.uint8, device="cuda")
    assert c.get(int(keys[0]), out)
    o = O.Store(max_keys=16, heap_bytes=4096 * U)
    host = [t.view(torch.uint8).reshape(-1).cpu().numpy() for t in snap]
    o.put_blocks(host, mb, [keys[0]], [int(src[0])], members_per_layer=3)
    assert o.get_bytes(keys[0], vlen) == out.cpu().numpy().tobytes()


def _compare_state(o, s, keys):
    for k in keys:
        lo, _ = o.location(k)
        ls, _ = s.location(k)
        assert LOC[lo] == LOC[ls], (k, LOC[lo], LOC[ls])
    so, ss = o.stats(), s.stats()
    for f in ("live_device_bytes", "pending_device_bytes", "live_keys", "device_resident_keys", "victims_evicted",
              "catalog_replacements", "writes_through", "stale_commits", "admissions", "epoch", "issued",
              "committed", "allocation_calls", "allocation_successes", "allocation_failures"):
        assert so[f] == ss[f], (f, so[f], ss[f])


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_directory_policy_matches_oracle_under_pressure(store, seed):
    """Random put / get / exists / delete / move sequences on a small slab and catalog: every key's
    residency, the counters, the LRU order and the hash buckets match the oracle after every op."""
    rng = np.random.default_rng(seed)
    cfg = dict(max_keys=24, heap_bytes=40 * U, host_pool_bytes=48 * U)
    c, s = store(**cfg)
    o = O.Store(max_keys=24, heap_bytes=40 * U, host_pool_bytes=48 * U)
    keys = [f"key-{i}".encode() for i in range(32)]
    vals = {}
    out = torch.zeros(8 * U, dtype=torch.uint8, device="cuda")
    for step in range(220):
        op = rng.choice(["put", "put", "put", "get", "get", "exists", "delete", "mth", "mtd", "flush", "sput"])
        k = keys[int(rng.integers(len(keys)))]
        if op in ("put", "sput"):
            n = int(rng.choice([1, 100, U, U + 1, 2 * U, 3 * U + 5, 5 * U]))
            data = payload(step, n)
            o.put(k, data, sync_commit=op == "sput")
            c.put(k, dev_bytes(data), n, sync_commit=op == "sput")
            vals[k] = data
        elif op == "get":
            out.fill_(0x5A)
            exp = o.get_bytes(k, 8 * U)
            got = c.get(k, out)
            assert got == (exp is not None)
            if got:
                assert out[: len(exp)].cpu().numpy().tobytes() == exp
        elif op == "exists":
            assert c.exists(k) == o.exists(k)
        elif op == "delete":
            assert c.delete(k) == o.remove(k)
        elif op == "mth":
            o.move_to_host(k)
            c.move_to_host(k)
        elif op == "mtd":
            o.move_to_device(k)
            c.move_to_device(k)
        else:
            o.flush()
            c.flush()
        _compare_state(o, s, keys)
    # LRU order (slots, MRU first) and the hash buckets (slot words) agree, and the device index
    # replica matches the host catalog once a device lookup has run
    c.exists_batch([1])
    assert s.lru_order() == o.lru_order().tolist()
    host_b, dev_b = s.index_snapshot()
    ob = o.buckets()
    assert np.array_equal(host_b[:, 1], ob[:, 1])
    live = host_b[:, 1] != 0xFFFFFFFF
    assert np.array_equal(host_b[live, 0], ob[live, 0])
    assert np.array_equal(dev_b[:, 1], host_b[:, 1]) and np.array_equal(dev_b[live, 0], host_b[live, 0])


@pytest.mark.parametrize("get_n", [12, 3])
@pytest.mark.parametrize("repeat_keys", [False, True])
def test_block_path_eviction_and_host_tier_matches_oracle(store, repeat_keys, get_n):
    """Blocks under a slab that holds a quarter of them: LRU eviction, host-tier serves and
    read-through admissions on get_blocks, compared with the oracle's sequential semantics. With
    repeat_keys a get batch names some keys more than once (a host-tier key admitted by its first
    get is read from its new block by the later ones). get_n = 3 takes the one-launch
    probe+scatter path of small gets."""
    n_layers, heads, bs, dim, pool = 2, 2, 16, 64, 96
    kv = kv_pool(n_layers, heads, bs, dim, pool, seed=7)
    layout = PagedLayout.from_kv_caches(kv)
    vlen = layout.value_bytes()
    units = -(-vlen // U)
    order_units = 1 << (units - 1).bit_length()
    heap = 12 * order_units * U
    c, s = store(max_keys=128, heap_bytes=heap, host_pool_bytes=64 << 20)
    o = O.Store(max_keys=128, heap_bytes=heap, host_pool_bytes=64 << 20)
    members = [t for p in kv for t in p]
    host = [t.view(torch.uint8).reshape(-1).cpu().numpy() for t in members]
    mb = layout.member_block_bytes
    rng = np.random.default_rng(7)
    keys = np.array(codec.chained_block_hashes(77, 48), dtype=np.uint64)
    for r in range(6):
        idx = rng.choice(48, 8, replace=False)
        src = rng.choice(48, 8, replace=False)
        c.put_blocks(layout, keys[idx], src)
        o.put_blocks(host, mb, keys[idx], src)
        g = rng.choice(48, get_n, replace=repeat_keys)
        dst = 48 + rng.choice(48, get_n, replace=False)
        fo = o.get_blocks(host, mb, keys[g], dst)
        fs = c.get_blocks(layout, keys[g], dst)
        assert np.array_equal(fo, fs)
        for m in range(len(members)):
            exp = host[m].reshape(pool, -1)[dst]
            assert np.array_equal(members[m].view(torch.uint8).reshape(pool, -1)[torch.as_tensor(dst).cuda()].cpu().numpy(), exp)
        _compare_state(o, s, [int(k) for k in keys])
    assert s.stats()["victims_evicted"] > 0 and s.stats()["admissions"] > 0


def test_small_gets_once_the_index_is_in_sync_match_oracle(store):
    """Gets of at most 8 blocks whose shard has no index updates pending and whose layout is on the
    device already launch without any host-to-device copy (keys and block ids in the kernel
    parameters): device hits, a host-tier hit, a miss and a repeated key against the oracle, with
    gets that must upload (pending index updates, another layout) in between."""
    n_layers, heads, bs, dim, pool = 2, 2, 16, 64, 64
    kv = kv_pool(n_layers, heads, bs, dim, pool, seed=12)
    layout = PagedLayout.from_kv_caches(kv)
    units = -(-layout.value_bytes() // U)
    heap = 32 * (1 << (units - 1).bit_length()) * U
    c, s = store(max_keys=64, heap_bytes=heap, host_pool_bytes=32 << 20)
    o = O.Store(max_keys=64, heap_bytes=heap, host_pool_bytes=32 << 20)
    members = [t for p in kv for t in p]
    host = [t.view(torch.uint8).reshape(-1).cpu().numpy() for t in members]
    mb = layout.member_block_bytes
    keys = np.array(codec.chained_block_hashes(91, 16), dtype=np.uint64)
    c.put_blocks(layout, keys[:12], np.arange(12))
    o.put_blocks(host, mb, keys[:12], np.arange(12))
    c.move_to_host(int(keys[3]))
    o.move_to_host(int(keys[3]))
    other = PagedLayout.from_kv_caches(kv_pool(n_layers, heads, bs, dim, 8, seed=13))
    c.get_blocks(other, keys[:1], [0])  # another layout: uploads, and applies the pending updates
    steps = [([0], [40]),                      # the layout the next gets reuse
             ([3, 1, 14, 1], [41, 42, 43, 44]),  # host-tier hit (admitted), device hit, miss, repeat
             ([2], [45]),                      # pending updates after the admission: uploads
             ([5, 6], [46, 47]), ([7], [48]), ([8, 9, 10, 11], [49, 50, 51, 52])]
    o.get_blocks([h.copy() for h in host], mb, keys[:1], [0])  # the same get (its pool is not compared)
    for idx, dst in steps:
        fo = o.get_blocks(host, mb, keys[idx], np.array(dst))
        fs = c.get_blocks(layout, keys[idx], dst)
        assert np.array_equal(fo, fs), (idx, fo, fs)
        for m in range(len(members)):
            got = members[m].view(torch.uint8).reshape(pool, -1)[torch.as_tensor(dst).cuda()].cpu().numpy()
            assert np.array_equal(got, host[m].reshape(pool, -1)[dst]), (idx, m)
        _compare_state(o, s, [int(k) for k in keys])


@pytest.mark.parametrize("slab_blocks", [1400, 300])
def test_put_of_more_than_512_blocks_matches_oracle(store, slab_blocks):
    """A put of 1100 blocks launches its gather in pieces of 512 while the host prepares the rest;
    with a slab of 300 blocks the pieces interleave with evictions and forced commits. The catalog,
    the restored blocks and the found flags equal the oracle's."""
    n_layers, heads, bs, dim, pool = 2, 2, 16, 32, 2304
    kv = kv_pool(n_layers, heads, bs, dim, pool, seed=21)
    layout = PagedLayout.from_kv_caches(kv)
    units = -(-layout.value_bytes() // U)
    heap = slab_blocks * (1 << (units - 1).bit_length()) * U
    cfg = dict(max_keys=2048, heap_bytes=heap, host_pool_bytes=1200 * units * U)
    c, s = store(**cfg)
    o = O.Store(**cfg)
    members = [t for p in kv for t in p]
    host = [t.view(torch.uint8).reshape(-1).cpu().numpy() for t in members]
    mb = layout.member_block_bytes
    keys = np.array(codec.chained_block_hashes(123, 1100), dtype=np.uint64)
    src = np.random.default_rng(4).permutation(1100)
    c.put_blocks(layout, keys, src)
    o.put_blocks(host, mb, keys, src)
    dst = np.arange(1152, 1152 + 1100)
    fo = o.get_blocks(host, mb, keys, dst)
    fs = c.get_blocks(layout, keys, dst)
    assert np.array_equal(fo, fs) and fs.all()
    for m in range(len(members)):
        got = members[m].view(torch.uint8).reshape(pool, -1)[1152:2252].cpu().numpy()
        assert np.array_equal(got, host[m].reshape(pool, -1)[1152:2252])
    _compare_state(o, s, [int(k) for k in keys[::7]])


def test_put_batch_and_get_parallel(store):
    c, s = store()
    c2 = Client(0, s)
    try:
        vals = [payload(i, 300 + i) for i in range(4)]
        c.put_batch([f"b{i}" for i in range(4)], [dev_bytes(v) for v in vals], [len(v) for v in vals], sync_commit=True)
        out = torch.zeros(2 * 512, dtype=torch.uint8, device="cuda")
        found = Client.get_parallel([c, c2], ["b1", "nope"], out)
        assert found == [True, False]
        assert out[: len(vals[1])].cpu().numpy().tobytes() == vals[1]
        assert not out[512:].any()
    finally:
        c2.close()


def test_profiles_and_counters(store):
    c, s = store()
    c.put(b"p", dev_bytes(payload(2, 5000)), 5000, sync_commit=True)
    c.move_to_host(b"p")
    c.move_to_device(b"p")
    assert s.moves_completed() >= 2
    mp = s.move_profile()
    assert mp["to_host_count"] == 1 and mp["to_device_count"] == 1 and mp["to_host_read_bytes"] == 5000
    ap = s.allocator_profile()
    assert ap["allocation_calls"] >= 2 and ap["allocation_successes"] >= 2
    pp = c.put_profile()
    assert pp["count"] == 1 and pp["total_ns"] > 0
    assert s.is_ready() and c.is_established()
    c.close()
    assert not c.is_established()
    with pytest.raises(KvsError, match="closed"):
        c.exists(b"p")


def test_put_blocks_with_a_key_twice_in_one_batch_matches_oracle(store):
    """A batch that puts one key twice: the second put waits for the first to commit (forced
    commit), then replaces it; the stored value is the second block, state as the oracle's."""
    n_layers, heads, bs, dim, pool = 2, 2, 16, 64, 32
    kv = kv_pool(n_layers, heads, bs, dim, pool, seed=3)
    layout = PagedLayout.from_kv_caches(kv)
    c, s = store(max_keys=64, heap_bytes=64 * U, host_pool_bytes=8 << 20)
    o = O.Store(max_keys=64, heap_bytes=64 * U, host_pool_bytes=8 << 20)
    members = [t for p in kv for t in p]
    host = [t.view(torch.uint8).reshape(-1).cpu().numpy() for t in members]
    mb = layout.member_block_bytes
    keys = np.array([7, 8, 7, 9, 8], dtype=np.uint64)
    src = np.array([0, 1, 2, 3, 4])
    c.put_blocks(layout, keys, src)
    o.put_blocks(host, mb, keys, src)
    dst = np.array([20, 21, 22])
    fo = o.get_blocks(host, mb, np.array([7, 8, 9], np.uint64), dst)
    fs = c.get_blocks(layout, np.array([7, 8, 9], np.uint64), dst)
    assert fo.all() and fs.all()
    for m in range(len(members)):
        got = members[m].view(torch.uint8).reshape(pool, -1)[20:23].cpu().numpy()
        assert np.array_equal(got, host[m].reshape(pool, -1)[20:23])
        assert np.array_equal(got[0], host[m].reshape(pool, -1)[2]) and np.array_equal(got[1], host[m].reshape(pool, -1)[4])
    _compare_state(o, s, [7, 8, 9])
