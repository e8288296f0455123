"""Expiry path of the bulk-copy engine's bounded waits, on the GPU, without a fault.

The engine bounds every wait on a tile load. kvs_set_copy_wait_limit(0) makes each CTA's first
wait expire at once, while the loads it already issued still land normally (the CTA waits for
them, with the full limit, before it exits). These tests check what a caller sees then:
  * the asynchronous chunk gather reports the expiry through kvs_copy_engine_status after the
    stream is synchronised, and no CTA exits with a load in flight (unsafe_exits stays 0);
  * a store client returns KVS_E_TIMEOUT from its next synchronising call and KVS_E_QUARANTINED
    from every call after it (the reference's Quarantined state,
    src/client_operations_adapter.cpp:54-59), while a fresh client on the same shard still
    restores earlier puts bit-exactly.
The copies stay on the bulk engine (the one-wave engine has no waits), and both limits are
restored after each test.
"""

import ctypes as C

import numpy as np
import pytest
import torch

from kvcache_manager import Client, KvsError, PagedLayout, Server, codec, ops
from kvcache_manager import _native
from oracle import kvs_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture
def lib():
    lib = _native.load()
    # the bounded waits belong to the bulk engine: keep these small copies off the one-wave engine
    assert lib.kvs_set_small_copy_limit(0) == 0
    yield lib
    assert lib.kvs_set_copy_wait_limit(-1) == 0
    assert lib.kvs_set_small_copy_limit(-1) == 0


def _status(lib, device=0):
    expired, unsafe = C.c_uint32(), C.c_uint32()
    _native.check(lib.kvs_copy_engine_status(device, C.byref(expired), C.byref(unsafe)))
    return expired.value, unsafe.value


def test_chunk_gather_reports_expired_waits(lib):
    g = torch.Generator().manual_seed(31)
    sbb, pool, n_members = 96 * 1024, 8, 4
    members = [torch.randint(0, 256, (pool * sbb,), dtype=torch.uint8, generator=g).cuda() for _ in range(n_members)]
    block_ids = [5, 1, 6]
    alloc = len(block_ids) * sbb
    header = list(O.header_words(n_members, [alloc] * n_members))
    region_bases = [4 * len(header) + m * alloc for m in range(n_members)]
    blob_bytes = region_bases[-1] + alloc
    e0, u0 = _status(lib)

    assert lib.kvs_set_copy_wait_limit(0) == 0
    cut = torch.zeros(blob_bytes, dtype=torch.uint8, device="cuda")
    ops.pack_local_shards(members, cut, block_ids, sbb, region_bases, header)  # synchronises the stream
    e1, u1 = _status(lib)
    assert e1 > e0, "a zero-poll wait limit must expire the copy engine's waits"
    assert u1 == u0, "a CTA exited with a tile load still in flight"
    # no tile store follows an expired wait: the payload regions stay as they were
    assert not cut[region_bases[0]:].any()

    assert lib.kvs_set_copy_wait_limit(-1) == 0
    full = torch.zeros(blob_bytes, dtype=torch.uint8, device="cuda")
    ops.pack_local_shards(members, full, block_ids, sbb, region_bases, header)
    assert _status(lib) == (e1, u1), "waits expired under the default limit"
    host = [t.cpu().numpy() for t in members]
    want = O.gather([host], [sbb] * n_members, block_ids, region_bases, header, blob_bytes)
    assert full.cpu().numpy().tobytes() == bytes(want)


def test_store_client_times_out_then_stays_quarantined(lib):
    g = torch.Generator().manual_seed(32)
    kv = [tuple(torch.randn((16, 8, 32, 128), generator=g).to(torch.bfloat16).cuda() for _ in range(2))
          for _ in range(2)]
    layout = PagedLayout.from_kv_caches(kv)
    keys_a = np.array(codec.chained_block_hashes(71, 4), np.uint64)
    keys_b = np.array(codec.chained_block_hashes(72, 4), np.uint64)
    with Server(0, max_keys=64, heap_bytes=64 << 20, host_pool_bytes=32 << 20) as server:
        c = Client(0, server)
        c.put_blocks(layout, keys_a, [0, 1, 2, 3], sync_commit=True)
        snap = [t.clone() for p in kv for t in p]
        e0, u0 = _status(lib)

        assert lib.kvs_set_copy_wait_limit(0) == 0
        c.put_blocks(layout, keys_b, [4, 5, 6, 7])  # returns at landed: nothing synchronised yet
        with pytest.raises(KvsError) as err:
            c.get_blocks(layout, keys_a, [8, 9, 10, 11])
        assert err.value.code == _native.E_TIMEOUT
        assert lib.kvs_set_copy_wait_limit(-1) == 0
        with pytest.raises(KvsError) as err:
            c.exists_batch(keys_a)
        assert err.value.code == _native.E_QUARANTINED
        with pytest.raises(KvsError) as err:
            c.get_blocks(layout, keys_a, [8, 9, 10, 11])
        assert err.value.code == _native.E_QUARANTINED
        e1, u1 = _status(lib)
        assert e1 > e0 and u1 == u0
        c.close()

        # the shard still serves the complete values of the earlier put to a fresh client
        with Client(0, server) as fresh:
            assert fresh.get_blocks(layout, keys_a, [12, 13, 14, 15]).all()
        for a, b in zip([t for p in kv for t in p], snap):
            assert torch.equal(a[12:16], b[0:4])
        assert _status(lib) == (e1, u1)
