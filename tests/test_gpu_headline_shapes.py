"""Bit-exact put / get at the block shapes the benchmark is quoted on, against the oracle.

* Qwen3-32B-shaped blocks: 64 layers x (K, V) of 8 KV heads x 64 tokens x 128 dims in bf16, so a
  value is 16 MiB of payload in 128 member regions of 128 KiB (buddy blocks of 4096 units). The
  kernels are shape-generic, but this is the shape of every headline number, so it is checked as
  itself: every restored block of every member byte for byte, and one stored value against the
  oracle's gather of the same block.
* The fine-grained fp8 layout: 80 layers x (K, V fp8 e4m3 of 8 heads x 16 tokens x 128 dims, one
  fp32 scale per block), 240 members per block, at batches of 1 and 4096 blocks: payload and
  scale bytes of every restored block, and one stored value against the oracle.
The byte layout follows the reference's scatter / gather (patch 0003 lines 8028-8247) and its
raw-byte blob (patch 0005 lines 12258-12310).
"""

import numpy as np
import pytest
import torch

from kvcache_manager import Client, PagedLayout, Server, codec
from oracle import kvs_oracle as O

pytestmark = [pytest.mark.gpu, pytest.mark.usefixtures("copy_engine")]

U = 4288


def _bits(t):
    return t.contiguous().view(torch.uint8)


def _check_restored(members, src, dst, snapshot=None):
    si = None if snapshot is not None else torch.as_tensor(np.asarray(src), device="cuda")
    di = torch.as_tensor(np.asarray(dst), device="cuda")
    for m, t in enumerate(members):
        want = snapshot[m] if snapshot is not None else t.index_select(0, si)
        assert torch.equal(_bits(t.index_select(0, di)), _bits(want)), f"member {m}: restored blocks differ"


def _check_value_against_oracle(client, layout, members, key, block, members_per_layer):
    mb = layout.member_block_bytes
    words, rb, vlen = O.block_format(mb, members_per_layer)
    assert vlen == layout.value_bytes()
    out = torch.zeros(vlen, dtype=torch.uint8, device="cuda")
    assert client.get(int(key), out)
    # the oracle store puts the same block from host copies of that block of every member
    host = [_bits(t[block:block + 1]).reshape(-1).cpu().numpy() for t in members]
    units = -(-vlen // U)
    o = O.Store(max_keys=16, heap_bytes=2 * (1 << (units - 1).bit_length()) * U, host_pool_bytes=0)
    try:
        o.put_blocks(host, mb, [int(key)], [0], members_per_layer=members_per_layer)
        assert o.get_bytes(int(key), vlen) == out.cpu().numpy().tobytes()
    finally:
        o.close()


def test_qwen3_32b_shaped_blocks_bit_exact():
    layers, heads, bt, dim, pool, n = 64, 8, 64, 128, 48, 16
    g = torch.Generator(device="cuda").manual_seed(2026)
    kv = []
    for _ in range(layers):
        kv.append(tuple(torch.empty((pool, heads, bt, dim), dtype=torch.bfloat16, device="cuda").normal_(generator=g)
                        for _ in range(2)))
    layout = PagedLayout.from_kv_caches(kv)
    members = layout.members
    assert sum(layout.member_block_bytes) == 16 << 20
    vlen = layout.value_bytes()
    units = -(-vlen // U)
    block_units = 1 << (units - 1).bit_length()
    assert block_units == 4096
    rng = np.random.default_rng(20)
    perm = rng.permutation(pool)
    src, dst = perm[:n], perm[n:2 * n]
    keys = np.array(codec.chained_block_hashes(2026, n), np.uint64)
    with Server(0, max_keys=64, heap_bytes=(n + 4) * block_units * U, host_pool_bytes=(n + 4) * units * U) as s, \
            Client(0, s) as c:
        c.put_blocks(layout, keys, src)
        found = c.get_blocks(layout, keys, dst)
        assert found.all()
        _check_restored(members, src, dst)
        _check_value_against_oracle(c, layout, members, keys[3], int(src[3]), 2)
        # misses leave their blocks untouched
        before = [t.index_select(0, torch.as_tensor(perm[2 * n:2 * n + 2], device="cuda")) for t in members]
        miss = np.array(codec.chained_block_hashes(99, 2), np.uint64)
        assert not c.get_blocks(layout, miss, perm[2 * n:2 * n + 2]).any()
        _check_restored(members, None, perm[2 * n:2 * n + 2], snapshot=before)


@pytest.fixture(scope="module")
def fp8_store():
    layers, heads, bt, dim, pool = 80, 8, 16, 128, 8192 + 64
    g = torch.Generator(device="cuda").manual_seed(5)
    members = []
    for _ in range(layers):
        for _ in range(2):
            t = torch.empty((pool, heads, bt, dim), dtype=torch.uint8, device="cuda")
            t.random_(0, 256, generator=g)
            members.append(t.view(torch.float8_e4m3fn))
        members.append(torch.rand((pool,), generator=g, device="cuda"))
    layout = PagedLayout(members, members_per_layer=3)
    vlen = layout.value_bytes()
    units = -(-vlen // U)
    block_units = 1 << (units - 1).bit_length()
    s = Server(0, max_keys=8192, heap_bytes=(4096 + 8) * block_units * U, host_pool_bytes=(4096 + 8) * units * U)
    c = Client(0, s)
    yield layout, members, c, pool
    c.close()
    s.close()


@pytest.mark.parametrize("batch", [1, 4096])
def test_fp8_scales_layout_bit_exact(fp8_store, batch):
    layout, members, c, pool = fp8_store
    assert len(members) == 240 and layout.member_block_bytes[2] == 4
    rng = np.random.default_rng(batch)
    perm = rng.permutation(pool)
    src, dst = perm[:batch], perm[batch:2 * batch]
    keys = np.array(codec.chained_block_hashes(5000 + batch, batch), np.uint64)
    c.put_blocks(layout, keys, src)
    assert c.get_blocks(layout, keys, dst).all()
    _check_restored(members, src, dst)  # payload and scales
    j = batch // 2
    _check_value_against_oracle(c, layout, members, keys[j], int(src[j]), 3)
    for k in keys:  # keep the catalog bounded for the next case
        c.delete(int(k))
