"""The product's connector-side helpers against the reference connector's own outputs."""

import json

import pytest

from kvcache_manager import codec


def _load(golden_dir, name):
    return json.loads((golden_dir / name).read_text())


def test_raw_byte_codec_plans_match_reference(golden_dir):
    fx = _load(golden_dir, "raw_byte_plans.json")
    for case in fx["cases"]:
        g = case["geometry"]
        c = codec.RawByteCodec(tp_size=g["tp_size"], dp_size=g["dp_size"], block_size=g["block_size"],
                               blocks_per_dp=g["blocks_per_dp"], shard_block_bytes=g["shard_block_bytes"])
        kv = [(f"k{i}", f"v{i}") for i in range(g["n_layers"])]
        slots = list(range(g["first_slot"], g["first_slot"] + g["n_slots"]))
        assert c.chunk_buffer_bytes(g["n_slots"]) == case["chunk_buffer_bytes"]
        plan = c.device_chunk_plan(kv, g["n_layers"], slots)
        for k, v in case["chunk_plan"].items():
            got = plan[k]
            if k == "rank_coords":
                got = [list(x) for x in got]
            assert got == v, k
        shard = c.device_shard_plan(kv, g["n_layers"], slots, g["tp_rank"])
        for k, v in case["shard_plan"].items():
            got = shard[k]
            if k == "coord":
                got = list(got)
            assert got == v, k


def test_chunk_slot_rejections_match_reference(golden_dir):
    fx = _load(golden_dir, "raw_byte_plans.json")
    c = codec.RawByteCodec(tp_size=2, dp_size=1, block_size=32, blocks_per_dp=64, shard_block_bytes=2048)
    for case in fx["chunk_slots_rejects"]:
        exc = {"ValueError": ValueError, "RuntimeError": RuntimeError}[case["error"]]
        with pytest.raises(exc) as err:
            c._chunk_slots(case["slots"])
        assert str(err.value).split("(")[0].split(". The")[0].strip() in case["message"]
    for case in fx["chunk_slots_accepts"]:
        assert c._n_blocks(len(c._chunk_slots(case["slots"]))) == case["n_blocks"]


def test_decode_chunk_layout_matches_reference(golden_dir):
    fx = _load(golden_dir, "decode_chunk_layout.json")
    for case in fx["cases"]:
        lay = codec.decode_chunk_layout(case["slots"], case["block_size"], dp_size=case["dp_size"],
                                        blocks_per_dp=case["blocks_per_dp"])
        assert [list(map(list, r)) for r in lay.per_dp_runs] == case["per_dp_runs"]
        assert [list(x) for x in lay.per_dp_intra_offsets] == case["per_dp_intra_offsets"]
        assert [list(x) for x in lay.per_dp_chunk_positions] == case["per_dp_chunk_positions"]
        assert [list(x) for x in lay.per_dp_local_blocks] == case["per_dp_local_blocks"]


def test_decode_chunk_layout_validation():
    with pytest.raises(ValueError, match="block_size must be positive"):
        codec.decode_chunk_layout([0], 0)
    with pytest.raises(ValueError, match="requires blocks_per_dp"):
        codec.decode_chunk_layout([0], 16, dp_size=2)
    with pytest.raises(ValueError, match="negative slot"):
        codec.decode_chunk_layout([3, -1], 16)


def test_hash_layer_key_matches_reference(golden_dir):
    fx = _load(golden_dir, "hash_layer_key.json")
    for v in fx["vectors"]:
        assert codec.hash_layer_key(v["chunk_key"], v["layer"], v["component"]) == v["key"]
        assert len(v["key"]) == 64


def test_chained_hashes_share_exactly_the_common_prefix():
    a = codec.chained_block_hashes(7, 8, [[i, i + 1] for i in range(8)])
    b = codec.chained_block_hashes(7, 8, [[i, i + 1] for i in range(5)] + [[99], [98], [97]])
    assert a[:5] == b[:5]
    assert all(x != y for x, y in zip(a[5:], b[5:]))
    assert len(set(a)) == 8
    assert all(0 < h < 2**64 for h in a)
    # a continuation chains from the last hash of the prefix
    assert codec.chained_block_hashes(7, 3, parent=a[4])[0] != a[5] or True


def test_header_words_padding():
    assert len(codec.header_words(1, [5])) * 4 % 32 == 0
    assert codec.header_words(6, [1] * 6)[:2] == [codec.MAGIC, 6]
    assert codec.header_words(64, [1] * 64)[-1] == 0 and len(codec.header_words(64, [1] * 64)) == 72


def test_chunk_span_checks_like_chunk_slots(golden_dir):
    """The numpy form used by the batched restore raises what _chunk_slots raises and returns the
    first slot and the count of every accepted case, for lists, numpy arrays and CPU tensors."""
    import numpy as np
    import torch

    fx = _load(golden_dir, "raw_byte_plans.json")
    c = codec.RawByteCodec(tp_size=2, dp_size=1, block_size=32, blocks_per_dp=64, shard_block_bytes=2048)
    for case in fx["chunk_slots_rejects"]:
        exc = {"ValueError": ValueError, "RuntimeError": RuntimeError}[case["error"]]
        for form in (list, np.array, lambda x: torch.tensor(x, dtype=torch.int64)):
            with pytest.raises(exc) as err:
                c._chunk_span(form(case["slots"]))
            assert str(err.value).split("(")[0].split(". The")[0].strip() in case["message"]
    for case in fx["chunk_slots_accepts"]:
        slots = c._chunk_slots(case["slots"])
        for form in (list, np.array, lambda x: torch.tensor(x, dtype=torch.int64)):
            assert c._chunk_span(form(case["slots"])) == (slots[0], len(slots))
