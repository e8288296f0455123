"""kvs_gather_chunk_noalloc: the chunk gather for callers that must not allocate device memory.

Serving engines that give almost all HBM to their paged KV pool, and restore paths that cannot
afford an allocation's device synchronisation, call this entry point instead of kvs_gather_chunk:
it stages its metadata in a fixed array compiled into the library. This test calls both entry
points through the C ABI on the same inputs, twice in a row with different inputs (the shared
array is overwritten between the calls), and requires byte-identical blobs. It runs alone in a
fresh process as well as after the rest of the suite.
"""

import ctypes as C

import numpy as np
import pytest
import torch

from kvcache_manager import _native

pytestmark = pytest.mark.gpu


def _arrays(n_ranks, n_members, sbb, pool, seed):
    g = torch.Generator().manual_seed(seed)
    members = [[torch.randint(0, 256, (pool * sbb,), dtype=torch.uint8, generator=g).cuda() for _ in range(n_members)]
               for _ in range(n_ranks)]
    flat = [members[r][m] for r in range(n_ranks) for m in range(n_members)]
    ptrs = (C.c_uint64 * len(flat))(*[t.data_ptr() for t in flat])
    sizes = (C.c_uint64 * n_members)(*([sbb] * n_members))
    extent = (C.c_uint64 * n_members)(*([pool * sbb] * n_members))
    return members, ptrs, sizes, extent


def _gather(fn, ptrs, n_ranks, n_members, sizes, extent, block_ids, region_bases, header, blob):
    lib = _native.load()
    ids = (C.c_uint32 * len(block_ids))(*block_ids)
    rb = (C.c_uint64 * n_members)(*region_bases)
    hw = (C.c_uint32 * max(1, len(header)))(*header)
    stream = torch.cuda.current_stream().cuda_stream
    rc = fn(ptrs, n_ranks, n_members, sizes, extent, ids, len(block_ids), rb, hw, len(header),
            C.c_void_p(blob.data_ptr()), blob.numel(), C.c_void_p(stream))
    assert rc == 0, lib.kvs_last_error().decode()


@pytest.mark.parametrize("call", [0, 1])
def test_noalloc_gather_matches_gather_on_consecutive_calls(call):
    lib = _native.load()
    shapes = [(3, 6, 2048, 4, [1, 2]), (2, 5, 64 * 1024 + 4096, 6, [5, 0, 3])]
    # two calls in a row with different inputs, each checked against the allocating entry point
    for k, (n_ranks, n_members, sbb, pool, block_ids) in enumerate(shapes):
        members, ptrs, sizes, extent = _arrays(n_ranks, n_members, sbb, pool, seed=100 * call + k)
        alloc = len(block_ids) * sbb * n_ranks
        header = [0x524B564E, n_members] + [alloc] * n_members
        header += [0] * ((-len(header)) % 8)
        region_bases = [4 * len(header) + m * alloc for m in range(n_members)]
        blob_bytes = region_bases[-1] + alloc
        ref = torch.full((blob_bytes,), 0xA5, dtype=torch.uint8, device="cuda")
        got = torch.full((blob_bytes,), 0x5A, dtype=torch.uint8, device="cuda")
        _gather(lib.kvs_gather_chunk, ptrs, n_ranks, n_members, sizes, extent, block_ids, region_bases, header, ref)
        _gather(lib.kvs_gather_chunk_noalloc, ptrs, n_ranks, n_members, sizes, extent, block_ids, region_bases,
                header, got)
        torch.cuda.synchronize()
        assert torch.equal(got, ref), f"call {k}: the no-alloc gather differs from kvs_gather_chunk"
        # and both hold the member blocks where the layout says
        for r in range(n_ranks):
            for m in range(n_members):
                for cb, b in enumerate(block_ids):
                    off = region_bases[m] + cb * sbb * n_ranks + r * sbb
                    assert torch.equal(got[off:off + sbb], members[r][m][b * sbb:(b + 1) * sbb])


def test_noalloc_rejects_metadata_beyond_its_scratch():
    lib = _native.load()
    n_members = 4096  # 24 B per member alone is 96 KiB > 64 KiB
    ptrs = (C.c_uint64 * n_members)(*([1] * n_members))
    sizes = (C.c_uint64 * n_members)(*([32] * n_members))
    extent = (C.c_uint64 * n_members)(*([1 << 20] * n_members))
    ids = (C.c_uint32 * 1)(0)
    rb = (C.c_uint64 * n_members)(*[32 * (m + 1) for m in range(n_members)])
    rc = lib.kvs_gather_chunk_noalloc(ptrs, 1, n_members, sizes, extent, ids, 1, rb, None, 0, C.c_void_p(1), 1 << 30,
                                      None)
    assert rc == _native.E_INVAL
    msg = lib.kvs_last_error().decode()
    assert "65536-byte scratch" in msg and "kvs_gather_chunk" in msg
