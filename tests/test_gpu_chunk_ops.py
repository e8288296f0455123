"""GPU chunk gather / scatter ops against the golden blob and the oracle (bit-exact)."""

import hashlib
import json

import numpy as np
import pytest
import torch

from oracle import kvs_oracle as O

pytestmark = [pytest.mark.gpu, pytest.mark.usefixtures("copy_engine")]


def _members(seed0, n_members, chips, wpm):
    out = []
    for m in range(n_members):
        g = torch.Generator().manual_seed(seed0 + m)
        out.append(torch.randint(0, 2**31 - 1, (chips, wpm), dtype=torch.int32, generator=g))
    return out


@pytest.fixture(scope="module")
def ops():
    from kvcache_manager import ops as ops_mod

    return ops_mod


def test_gather_golden_three_ranks_one_gpu_then_scatter(golden_dir, ops):
    fx = json.loads((golden_dir / "gather_roundtrip.json").read_text())
    expected = (golden_dir / "gather_roundtrip_expected.bin").read_bytes()
    sbb, nm, ranks = fx["SHARD_BLOCK_BYTES"], fx["N_MEMBERS"], fx["rank_indices"]
    wpm = fx["BLOCKS"] * sbb // 4
    host = _members(fx["member_seed0"], nm, fx["chips"], wpm)
    # every chip's shard becomes its own device tensor (ranks live on one GPU here)
    dev = [[host[m][chip].clone().cuda() for m in range(nm)] for chip in range(fx["chips"])]
    blob = torch.zeros(fx["value_len"], dtype=torch.uint8, device="cuda")
    ops.gather_tp_shards_to_chip([dev[r] for r in ranks], blob, fx["CHUNK_BLOCKS"], sbb, fx["region_bases"],
                                 fx["header_words"])
    got = blob.cpu().numpy().tobytes()
    assert hashlib.sha256(got).hexdigest() == fx["expected_sha256"]
    assert got == expected
    for chip in range(fx["chips"]):
        for t in dev[chip]:
            t.zero_()
    ops.scatter_chunk_from_chip(blob, [dev[r] for r in ranks], fx["CHUNK_BLOCKS"], sbb, fx["region_bases"])
    for chip in range(fx["chips"]):
        for m in range(nm):
            now = dev[chip][m].cpu()
            for blk in range(fx["BLOCKS"]):
                lo, hi = blk * sbb // 4, (blk + 1) * sbb // 4
                if chip in ranks and blk in fx["CHUNK_BLOCKS"]:
                    assert torch.equal(now[lo:hi], host[m][chip][lo:hi]), (chip, m, blk)
                else:
                    assert int(now[lo:hi].abs().sum()) == 0, f"chip {chip} member {m}: spilled into block {blk}"


def test_pack_unpack_local_shards_match_oracle(golden_dir, ops):
    fx = json.loads((golden_dir / "perchip_roundtrip.json").read_text())
    sbb, nm = fx["SHARD_BLOCK_BYTES"], fx["N_MEMBERS"]
    plan = fx["shard_plans"][str(len(fx["CHUNK_BLOCKS"]))]
    host = _members(1000, nm, fx["chips"], fx["BLOCKS"] * sbb // 4)
    for chip in range(fx["chips"]):
        members = [host[m][chip].clone().cuda() for m in range(nm)]
        blob = torch.zeros(plan["value_len"], dtype=torch.uint8, device="cuda")
        ops.pack_local_shards(members, blob, fx["CHUNK_BLOCKS"], sbb, plan["region_bases"], plan["header_words"])
        ref = O.gather([[host[m][chip].view(torch.uint8).numpy() for m in range(nm)]], [sbb] * nm, fx["CHUNK_BLOCKS"],
                       plan["region_bases"], plan["header_words"], plan["value_len"])
        assert np.array_equal(blob.cpu().numpy(), ref)
        for t in members:
            t.zero_()
        ops.unpack_local_shards(blob, members, fx["CHUNK_BLOCKS"], sbb, plan["region_bases"])
        for m in range(nm):
            for blk in fx["CHUNK_BLOCKS"]:
                lo, hi = blk * sbb // 4, (blk + 1) * sbb // 4
                assert torch.equal(members[m].cpu()[lo:hi], host[m][chip][lo:hi])


@pytest.mark.parametrize("seed,n_ranks,n_members,sbb,n_blocks,pool", [
    (1, 1, 4, 65536, 8, 32),       # config-1 segments
    (2, 2, 6, 4096, 5, 16),
    (3, 3, 3, 48, 7, 20),          # tiny, 16-byte multiples
    (4, 1, 2, 36, 3, 9),           # 4-byte multiple only: word path
    (5, 4, 2, 131072 + 4096, 3, 6),  # multi-tile segments with a ragged tail tile
])
def test_random_chunks_match_oracle(ops, seed, n_ranks, n_members, sbb, n_blocks, pool):
    rng = np.random.default_rng(seed)
    host = [[rng.integers(0, 256, pool * sbb, dtype=np.uint8) for _ in range(n_members)] for _ in range(n_ranks)]
    block_ids = [int(b) for b in rng.permutation(pool)[:n_blocks]]
    words = O.header_words(n_members, [n_blocks * sbb * n_ranks] * n_members).tolist()
    hdr = 4 * len(words)
    region = (n_blocks * sbb * n_ranks + 32 + 31) // 32 * 32  # 32-aligned regions with gaps between
    rb = [hdr + m * region for m in range(n_members)]
    blob_bytes = rb[-1] + n_blocks * sbb * n_ranks + 64
    ref = O.gather(host, [sbb] * n_members, block_ids, rb, words, blob_bytes)
    dev = [[torch.from_numpy(a).cuda() for a in r] for r in host]
    blob = torch.zeros(blob_bytes, dtype=torch.uint8, device="cuda")
    ops.gather_tp_shards_to_chip(dev, blob, block_ids, sbb, rb, words)
    assert np.array_equal(blob.cpu().numpy(), ref)
    cleared = [[np.zeros_like(a) for a in r] for r in host]
    O.scatter(ref, cleared, [sbb] * n_members, block_ids, rb)
    dclear = [[torch.zeros_like(t) for t in r] for r in dev]
    ops.scatter_chunk_from_chip(blob, dclear, block_ids, sbb, rb)
    for r in range(n_ranks):
        for m in range(n_members):
            assert np.array_equal(dclear[r][m].cpu().numpy(), cleared[r][m])


def test_validation_errors_before_any_access(ops):
    from kvcache_manager import KvsError

    m = [torch.zeros(64, dtype=torch.int32, device="cuda")]
    blob = torch.zeros(1024, dtype=torch.uint8, device="cuda")
    with pytest.raises(KvsError, match="header must be 32-byte aligned"):
        ops.pack_local_shards(m, blob, [0], 32, [32], [0] * 4)
    with pytest.raises(KvsError, match="overlaps the"):
        ops.pack_local_shards(m, blob, [0], 32, [0], [0] * 8)
    with pytest.raises(KvsError, match="reaches past member"):
        ops.pack_local_shards(m, blob, [8], 32, [32], [0] * 8)
    with pytest.raises(KvsError, match="past the"):
        ops.pack_local_shards(m, blob, [0], 32, [1024], [0] * 8)
    with pytest.raises(KvsError, match="region base .* 32-byte aligned"):
        ops.pack_local_shards(m, blob, [0], 32, [48], [0] * 8)
    assert not blob.any()
