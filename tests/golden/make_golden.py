"""Generate the golden fixtures in tests/golden/ from the reference's own Python code.

This script runs only where the reference checkout is present (default
/root/reference, or $KVS_REFERENCE). It imports, unmodified:

  * tests/device/test_kvcache_manager_gather_roundtrip.py  (_gathered_plan, _make_members,
    _expected_gathered_bytes) with a stand-in `ttnn` whose from_torch returns its input;
  * tests/device/test_kvcache_manager_perchip_roundtrip.py (_shard_plan, _make_members);
  * the connector modules tt_raw_byte.py, tt_paged_slice.py and tt_kv_serde.py, which the
    reference keeps as new-file hunks of third_party/tt-metal/patches/0005-*.patch; they are
    extracted to a temporary directory and imported with a stand-in `lmcache.logging`.

The outputs are small JSON/binary files committed next to this script. Tests never read the
reference; they only read these fixtures.
"""

from __future__ import annotations

import hashlib
import importlib
import json
import os
import sys
import tempfile
import types
from pathlib import Path

import torch

REF = Path(os.environ.get("KVS_REFERENCE", "/root/reference"))
OUT = Path(__file__).resolve().parent
P5 = REF / "third_party/tt-metal/patches/0005-lmcache-t3knic-connector.patch"


def extract_new_file(patch: Path, path_in_patch: str) -> str:
    """Return the text of a new-file hunk (`--- /dev/null`, `+++ b/<path>`) of a patch."""
    lines = patch.read_text().splitlines()
    for i, line in enumerate(lines):
        if line == f"+++ b/{path_in_patch}":
            hunk = lines[i + 1]
            assert hunk.startswith("@@ -0,0 +1"), hunk
            count = int(hunk.split("+1,")[1].split(" ")[0])
            body = lines[i + 2 : i + 2 + count]
            assert all(b.startswith("+") for b in body)
            return "\n".join(b[1:] for b in body) + "\n"
    raise KeyError(path_in_patch)


def stub_modules() -> None:
    ttnn = types.ModuleType("ttnn")
    ttnn.ROW_MAJOR_LAYOUT = "ROW_MAJOR"
    ttnn.DRAM_MEMORY_CONFIG = "DRAM"
    ttnn.from_torch = lambda t, **kw: t
    ttnn.ShardTensorToMesh = lambda *a, **kw: None
    ttnn.ReplicateTensorToMesh = lambda *a, **kw: None
    sys.modules["ttnn"] = ttnn
    lm = types.ModuleType("lmcache")
    lml = types.ModuleType("lmcache.logging")

    class _Log:
        def __getattr__(self, name):
            return lambda *a, **k: None

    lml.init_logger = lambda name: _Log()
    lm.logging = lml
    sys.modules["lmcache"] = lm
    sys.modules["lmcache.logging"] = lml


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


def gather_roundtrip() -> None:
    sys.path.insert(0, str(REF / "tests"))
    g = importlib.import_module("device.test_kvcache_manager_gather_roundtrip")
    chips = 8  # the 2x4 model submesh of kvcache_manager_gather_2d_setup
    rank_indices = [0, 1, 2]
    members, host = g._make_members(object(), chips)
    words, region_bases, value_len = g._gathered_plan(g.N_MEMBERS, len(g.CHUNK_BLOCKS), len(rank_indices))
    expected = g._expected_gathered_bytes(host, words, rank_indices)
    assert len(expected) == value_len
    (OUT / "gather_roundtrip_expected.bin").write_bytes(expected)
    fixture = {
        "source": "tests/device/test_kvcache_manager_gather_roundtrip.py",
        "SHARD_BLOCK_BYTES": g.SHARD_BLOCK_BYTES,
        "BLOCKS": g.BLOCKS,
        "N_MEMBERS": g.N_MEMBERS,
        "CHUNK_BLOCKS": g.CHUNK_BLOCKS,
        "chips": chips,
        "rank_indices": rank_indices,
        "member_seed0": 3000,
        "header_words": [int(w) for w in words],
        "region_bases": [int(r) for r in region_bases],
        "value_len": int(value_len),
        "member_sha256": [sha(h) for h in host],
        "expected_sha256": hashlib.sha256(expected).hexdigest(),
    }
    (OUT / "gather_roundtrip.json").write_text(json.dumps(fixture, indent=1) + "\n")

    p = importlib.import_module("device.test_kvcache_manager_perchip_roundtrip")
    chips_pc = 4
    plans = {}
    for n_blocks in (1, 2, 3):
        w, rb, vl = p._shard_plan(p.N_MEMBERS, n_blocks)
        plans[str(n_blocks)] = {"header_words": [int(x) for x in w], "region_bases": [int(x) for x in rb],
                                "value_len": int(vl)}
    seeds = {}
    for seed0 in (1000, 2000):
        _, host = p._make_members(object(), chips_pc, seed0=seed0)
        seeds[str(seed0)] = [sha(h) for h in host]
    (OUT / "perchip_roundtrip.json").write_text(json.dumps({
        "source": "tests/device/test_kvcache_manager_perchip_roundtrip.py",
        "SHARD_BLOCK_BYTES": p.SHARD_BLOCK_BYTES, "BLOCKS": p.BLOCKS, "N_MEMBERS": p.N_MEMBERS,
        "CHUNK_BLOCKS": p.CHUNK_BLOCKS, "chips": chips_pc, "shard_plans": plans, "member_sha256": seeds,
    }, indent=1) + "\n")


def connector_modules() -> dict:
    tmp = Path(tempfile.mkdtemp(prefix="kvs_golden_"))
    mods = {}
    for name in ("tt_raw_byte", "tt_paged_slice", "tt_kv_serde"):
        src = extract_new_file(P5, f"lmcache-t3knic/lmcache_t3knic/t3knic_lmcache/{name}.py")
        (tmp / f"{name}.py").write_text(src)
    sys.path.insert(0, str(tmp))
    for name in ("tt_raw_byte", "tt_paged_slice", "tt_kv_serde"):
        mods[name] = importlib.import_module(name)
    return mods


def raw_byte_plans(rb) -> None:
    cases = []
    geoms = [
        # (tp, dp, block_size, blocks_per_dp, shard_block_bytes, n_layers, first_slot, n_slots, tp_rank)
        (1, 1, 32, 1024, 65536, 2, 0, 32, 0),
        (1, 1, 32, 1024, 65536, 2, 64, 96, 0),
        (1, 1, 64, 4096, 131072, 64, 128, 64, 0),
        (1, 1, 16, 65536, 16384, 80, 16 * 7, 16, 0),
        (4, 2, 128, 256, 1088 * 4, 3, 128 * 300, 256, 2),
        (8, 1, 128, 512, 1088 * 8, 64, 128 * 5, 100, 7),
    ]
    for tp, dp, bs, bpd, sbb, nl, first, n, rank in geoms:
        codec = rb.RawByteCodec(tp_size=tp, dp_size=dp, block_size=bs, blocks_per_dp=bpd, shard_block_bytes=sbb)
        kv = [(f"k{layer}", f"v{layer}") for layer in range(nl)]
        slots = list(range(first, first + n))
        plan = codec.device_chunk_plan(kv, nl, slots)
        shard = codec.device_shard_plan(kv, nl, slots, rank)
        cases.append({
            "geometry": {"tp_size": tp, "dp_size": dp, "block_size": bs, "blocks_per_dp": bpd,
                         "shard_block_bytes": sbb, "n_layers": nl, "first_slot": first, "n_slots": n,
                         "tp_rank": rank},
            "chunk_buffer_bytes": codec.chunk_buffer_bytes(n),
            "chunk_plan": {k: plan[k] for k in ("rank_coords", "dp", "region_bases", "block_ids", "header_words",
                                                "value_len", "member_bytes")},
            "shard_plan": {k: shard[k] for k in ("coord", "shard_index", "region_bases", "block_ids",
                                                 "header_words", "value_len", "member_bytes")},
        })
    rejects = []
    codec = rb.RawByteCodec(tp_size=2, dp_size=1, block_size=32, blocks_per_dp=64, shard_block_bytes=2048)
    for slots in ([], [5, 6, 7], [32, 33, 35], [64, 65, 66, 64]):
        try:
            codec._chunk_slots(slots)
            rejects.append({"slots": slots, "error": None})
        except (ValueError, RuntimeError) as e:
            rejects.append({"slots": slots, "error": type(e).__name__, "message": str(e)})
    accepts = []
    for slots in ([0], list(range(32, 64)), list(range(96, 150))):
        t = codec._chunk_slots(slots)
        accepts.append({"slots": slots, "n_blocks": codec._n_blocks(int(t.numel()))})
    (OUT / "raw_byte_plans.json").write_text(json.dumps({
        "source": "patch 0005 lmcache_t3knic/t3knic_lmcache/tt_raw_byte.py",
        "magic": rb.RawByteCodec._MAGIC, "header_align": rb.RawByteCodec.HEADER_ALIGN,
        "cases": cases, "chunk_slots_rejects": rejects, "chunk_slots_accepts": accepts,
    }, indent=1) + "\n")


def paged_slice(ps) -> None:
    cases = []
    inputs = [
        (list(range(0, 64)), 32, 1, None),
        (list(range(96, 160)) + [7, 8], 32, 1, None),
        ([3, 1, 2, 40, 41, 90], 16, 2, 4),
        (list(range(256, 300)) + [1000], 64, 2, 8),
    ]
    for slots, bs, dp, bpd in inputs:
        lay = ps.decode_chunk_layout(slots, bs, dp_size=dp, blocks_per_dp=bpd)
        cases.append({"slots": slots, "block_size": bs, "dp_size": dp, "blocks_per_dp": bpd,
                      "per_dp_runs": [list(map(list, r)) for r in lay.per_dp_runs],
                      "per_dp_intra_offsets": [list(x) for x in lay.per_dp_intra_offsets],
                      "per_dp_chunk_positions": [list(x) for x in lay.per_dp_chunk_positions],
                      "per_dp_local_blocks": [list(x) for x in lay.per_dp_local_blocks]})
    (OUT / "decode_chunk_layout.json").write_text(json.dumps({
        "source": "patch 0005 lmcache_t3knic/t3knic_lmcache/tt_paged_slice.py", "cases": cases}, indent=1) + "\n")


def layer_keys(serde) -> None:
    vecs = []
    for chunk_key in ("vllm@qwen3-32b@8@0@deadbeef", "model@1@0@0123456789abcdef", ""):
        for layer in (0, 1, 63):
            for comp in ("kv", "k", "v", "raw"):
                vecs.append({"chunk_key": chunk_key, "layer": layer, "component": comp,
                             "key": serde.hash_layer_key(chunk_key, layer, comp)})
    (OUT / "hash_layer_key.json").write_text(json.dumps({
        "source": "patch 0005 lmcache_t3knic/t3knic_lmcache/tt_kv_serde.py", "vectors": vecs}, indent=1) + "\n")


def main() -> None:
    stub_modules()
    gather_roundtrip()
    mods = connector_modules()
    raw_byte_plans(mods["tt_raw_byte"])
    paged_slice(mods["tt_paged_slice"])
    layer_keys(mods["tt_kv_serde"])
    print("golden fixtures written to", OUT)


if __name__ == "__main__":
    main()
