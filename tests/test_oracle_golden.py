"""Pin the CPU oracle against golden vectors produced by the reference's own code.

The fixtures in tests/golden/ come from tests/golden/make_golden.py, which imports the
reference's device-test helpers (_gathered_plan, _make_members, _expected_gathered_bytes,
_shard_plan) and its connector modules (tt_raw_byte.py, tt_kv_serde.py). These tests never read
the reference.
"""

import hashlib
import json

import numpy as np
import pytest
import torch

from oracle import kvs_oracle as O


def _load(golden_dir, name):
    return json.loads((golden_dir / name).read_text())


def _members(seed0, n_members, chips, words_per_member):
    """Same torch.randint calls as the reference tests' _make_members."""
    out = []
    for m in range(n_members):
        g = torch.Generator().manual_seed(seed0 + m)
        out.append(torch.randint(0, 2**31 - 1, (chips, words_per_member), dtype=torch.int32, generator=g))
    return out


def _sha(t):
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


@pytest.fixture(scope="module")
def gather_case(golden_dir):
    fx = _load(golden_dir, "gather_roundtrip.json")
    wpm = fx["BLOCKS"] * fx["SHARD_BLOCK_BYTES"] // 4
    host = _members(fx["member_seed0"], fx["N_MEMBERS"], fx["chips"], wpm)
    expected = (golden_dir / "gather_roundtrip_expected.bin").read_bytes()
    return fx, host, expected


def test_member_generation_matches_reference_helpers(gather_case):
    fx, host, _ = gather_case
    assert [_sha(h) for h in host] == fx["member_sha256"]


def test_header_and_region_plan_match_reference(gather_case):
    fx, _, _ = gather_case
    n_ranks = len(fx["rank_indices"])
    alloc = len(fx["CHUNK_BLOCKS"]) * n_ranks * fx["SHARD_BLOCK_BYTES"]
    words = O.header_words(fx["N_MEMBERS"], [alloc] * fx["N_MEMBERS"])
    assert words.tolist() == fx["header_words"]
    hdr = 4 * len(words)
    assert [hdr + m * alloc for m in range(fx["N_MEMBERS"])] == fx["region_bases"]
    assert hdr + fx["N_MEMBERS"] * alloc == fx["value_len"]


def test_oracle_gather_is_byte_exact_against_reference_expected_blob(gather_case):
    fx, host, expected = gather_case
    ranks = fx["rank_indices"]
    sbb = fx["SHARD_BLOCK_BYTES"]
    members = [[host[m][r].contiguous().view(torch.uint8).numpy() for m in range(fx["N_MEMBERS"])] for r in ranks]
    blob = O.gather(members, [sbb] * fx["N_MEMBERS"], fx["CHUNK_BLOCKS"], fx["region_bases"], fx["header_words"],
                    fx["value_len"])
    assert hashlib.sha256(blob.tobytes()).hexdigest() == fx["expected_sha256"]
    assert blob.tobytes() == expected


def test_oracle_scatter_restores_owned_blocks_and_leaves_the_rest_zero(gather_case):
    fx, host, expected = gather_case
    ranks, sbb, n_members = fx["rank_indices"], fx["SHARD_BLOCK_BYTES"], fx["N_MEMBERS"]
    cleared = [[np.zeros(fx["BLOCKS"] * sbb, np.uint8) for _ in range(n_members)] for _ in range(fx["chips"])]
    src = np.frombuffer(expected, np.uint8).copy()
    O.scatter(src, [cleared[r] for r in ranks], [sbb] * n_members, fx["CHUNK_BLOCKS"], fx["region_bases"])
    for chip in range(fx["chips"]):
        for m in range(n_members):
            orig = host[m][chip].contiguous().view(torch.uint8).numpy()
            now = cleared[chip][m]
            for blk in range(fx["BLOCKS"]):
                lo, hi = blk * sbb, (blk + 1) * sbb
                if chip in ranks and blk in fx["CHUNK_BLOCKS"]:
                    assert np.array_equal(now[lo:hi], orig[lo:hi]), (chip, m, blk)
                else:
                    assert not now[lo:hi].any(), f"chip {chip} member {m}: scatter spilled into block {blk}"


def test_perchip_shard_plans_match_reference(golden_dir):
    fx = _load(golden_dir, "perchip_roundtrip.json")
    sbb = fx["SHARD_BLOCK_BYTES"]
    for n_blocks, plan in fx["shard_plans"].items():
        alloc = int(n_blocks) * sbb
        words = O.header_words(fx["N_MEMBERS"], [alloc] * fx["N_MEMBERS"])
        assert words.tolist() == plan["header_words"]
        hdr = 4 * len(words)
        assert [hdr + i * alloc for i in range(fx["N_MEMBERS"])] == plan["region_bases"]
        assert hdr + fx["N_MEMBERS"] * alloc == plan["value_len"]
    wpm = fx["BLOCKS"] * sbb // 4
    for seed0, shas in fx["member_sha256"].items():
        assert [_sha(h) for h in _members(int(seed0), fx["N_MEMBERS"], fx["chips"], wpm)] == shas


def test_chunk_plans_match_raw_byte_codec(golden_dir):
    fx = _load(golden_dir, "raw_byte_plans.json")
    assert fx["magic"] == O.MAGIC
    for case in fx["cases"]:
        g = case["geometry"]
        n_blocks = -(-g["n_slots"] // g["block_size"])
        for plan, sbb in ((case["chunk_plan"], g["shard_block_bytes"] * g["tp_size"]),
                          (case["shard_plan"], g["shard_block_bytes"])):
            words, rb, vlen = O.chunk_plan(g["n_layers"], n_blocks * sbb)
            assert words.tolist() == plan["header_words"]
            assert rb.tolist() == plan["region_bases"]
            assert vlen == plan["value_len"]
            assert plan["member_bytes"] == n_blocks * sbb
        first_block = g["first_slot"] // g["block_size"]
        local = first_block % g["blocks_per_dp"]
        assert case["chunk_plan"]["block_ids"] == list(range(local, local + n_blocks))


def test_chunk_slots_accept_and_reject_like_the_codec(golden_dir):
    fx = _load(golden_dir, "raw_byte_plans.json")
    for case in fx["chunk_slots_rejects"]:
        with pytest.raises(O.OracleError) as err:
            O.chunk_slots(case["slots"], 32)
        key = case["message"].split("(")[0].split(". The")[0].strip()
        assert key in str(err.value)
    for case in fx["chunk_slots_accepts"]:
        _, nb = O.chunk_slots(case["slots"], 32)
        assert nb == case["n_blocks"]


def test_fnv1a32_published_vectors():
    # FNV-1a 32-bit test vectors published with the algorithm (Fowler/Noll/Vo)
    assert O.fnv1a32(b"") == 0x811C9DC5
    assert O.fnv1a32(b"a") == 0xE40C292C
    assert O.fnv1a32(b"foobar") == 0xBF9CF968


def test_hash_num_buckets_and_buddy_orders():
    assert O.hash_num_buckets(1024) == 2048
    assert O.hash_num_buckets(1000) == 2048
    assert O.hash_num_buckets(0) == 2
    assert O.hash_num_buckets(65536) == 131072
    assert [O.buddy_order_for_units(u) for u in (1, 2, 3, 4, 5, 3913, 4096, 4097)] == [0, 1, 2, 2, 3, 12, 12, 13]
