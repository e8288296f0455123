"""kvs_gather_chunk_noalloc: the chunk gather for callers that must not allocate device memory.

Serving engines that give almost all HBM to their paged KV pool, and restore paths that cannot
afford an allocation's device synchronisation, call this entry point instead of kvs_gather_chunk:
it keeps its metadata in a fixed array compiled into the library. These tests call both entry
points through the C ABI on the same inputs, twice in a row with different inputs (the shared
array is overwritten between the calls), and require byte-identical blobs; check that many calls
leave the device's free memory unchanged; and run the comparison once more in a fresh Python
process, where the first call on the device also does the array's set-up. This file is collected
last, so a run that stops at the first failure has run every other test before it.
"""

import ctypes as C
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

from kvcache_manager import _native

pytestmark = pytest.mark.gpu

# (ranks, members, block bytes, pool blocks, block ids): the last one's 4000 block ids need more
# metadata than one staging launch carries, so its metadata goes in two
SHAPES = [(3, 6, 2048, 4, [1, 2]), (2, 5, 64 * 1024 + 4096, 6, [5, 0, 3]),
          (1, 2, 1024, 4096, [(7 * i) % 4096 for i in range(4000)])]


def _arrays(n_ranks, n_members, sbb, pool, seed):
    g = torch.Generator().manual_seed(seed)
    members = [[torch.randint(0, 256, (pool * sbb,), dtype=torch.uint8, generator=g).cuda() for _ in range(n_members)]
               for _ in range(n_ranks)]
    flat = [members[r][m] for r in range(n_ranks) for m in range(n_members)]
    ptrs = (C.c_uint64 * len(flat))(*[t.data_ptr() for t in flat])
    sizes = (C.c_uint64 * n_members)(*([sbb] * n_members))
    extent = (C.c_uint64 * n_members)(*([pool * sbb] * n_members))
    return members, ptrs, sizes, extent


class _Case:
    def __init__(self, n_ranks, n_members, sbb, pool, block_ids, seed):
        self.n_ranks, self.n_members, self.sbb, self.block_ids = n_ranks, n_members, sbb, block_ids
        self.members, self.ptrs, self.sizes, self.extent = _arrays(n_ranks, n_members, sbb, pool, seed)
        alloc = len(block_ids) * sbb * n_ranks
        header = [0x524B564E, n_members] + [alloc] * n_members
        self.header = header + [0] * ((-len(header)) % 8)
        self.region_bases = [4 * len(self.header) + m * alloc for m in range(n_members)]
        self.blob_bytes = self.region_bases[-1] + alloc
        self.ids = (C.c_uint32 * len(block_ids))(*block_ids)
        self.rb = (C.c_uint64 * n_members)(*self.region_bases)
        self.hw = (C.c_uint32 * len(self.header))(*self.header)

    def gather(self, fn, blob):
        stream = torch.cuda.current_stream().cuda_stream
        rc = fn(self.ptrs, self.n_ranks, self.n_members, self.sizes, self.extent, self.ids, len(self.block_ids),
                self.rb, self.hw, len(self.header), C.c_void_p(blob.data_ptr()), blob.numel(), C.c_void_p(stream))
        assert rc == 0, _native.load().kvs_last_error().decode()


def _compare_consecutive_calls(seed_base):
    lib = _native.load()
    # calls in a row with different inputs, each checked against the allocating entry point
    for k, shape in enumerate(SHAPES):
        case = _Case(*shape, seed=seed_base + k)
        ref = torch.full((case.blob_bytes,), 0xA5, dtype=torch.uint8, device="cuda")
        got = torch.full((case.blob_bytes,), 0x5A, dtype=torch.uint8, device="cuda")
        case.gather(lib.kvs_gather_chunk, ref)
        case.gather(lib.kvs_gather_chunk_noalloc, got)
        torch.cuda.synchronize()
        assert torch.equal(got, ref), f"call {k}: the no-alloc gather differs from kvs_gather_chunk"
        # and both hold the member blocks where the layout says
        sbb, n_ranks = case.sbb, case.n_ranks
        for r in range(n_ranks):
            for m in range(case.n_members):
                for cb, b in list(enumerate(case.block_ids))[:8]:
                    off = case.region_bases[m] + cb * sbb * n_ranks + r * sbb
                    assert torch.equal(got[off:off + sbb], case.members[r][m][b * sbb:(b + 1) * sbb])


@pytest.mark.parametrize("call", [0, 1])
def test_noalloc_gather_matches_gather_on_consecutive_calls(call):
    _compare_consecutive_calls(100 * call)


def test_noalloc_gather_leaves_device_memory_unchanged():
    lib = _native.load()
    case = _Case(*SHAPES[1], seed=7)
    blob = torch.zeros(case.blob_bytes, dtype=torch.uint8, device="cuda")
    case.gather(lib.kvs_gather_chunk_noalloc, blob)  # first call: module load and the array's set-up
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    reserved0 = torch.cuda.memory_reserved()
    for _ in range(200):
        case.gather(lib.kvs_gather_chunk_noalloc, blob)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, f"device free memory moved by {free0 - free1} bytes over 200 calls"
    assert torch.cuda.memory_reserved() == reserved0


def test_noalloc_gather_in_a_fresh_process():
    if os.environ.get("KVS_NOALLOC_CHILD"):
        pytest.skip("already the fresh process")
    root = Path(__file__).resolve().parents[1]
    env = dict(os.environ, KVS_NOALLOC_CHILD="1")
    code = ("import sys; sys.path[:0] = [{!r}, {!r}, {!r}]\n"
            "import test_zz_no_alloc as t; t._compare_consecutive_calls(500); print('fresh-process ok')"
            ).format(str(root), str(root / "tt-infinity_b200"), str(root / "tests"))
    res = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env, timeout=600)
    assert res.returncode == 0 and "fresh-process ok" in res.stdout, res.stdout[-2000:] + res.stderr[-2000:]


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
