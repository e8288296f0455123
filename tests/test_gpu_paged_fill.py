"""The sm_100a token-granular paged fill (kvcache_manager.ops.paged_fill_cache_varlen, through
kvs_paged_fill_varlen) against the oracle, which tests/test_paged_fill_oracle.py pins to the
reference's own moreh_paged_fill_cache_varlen kernels: tile-aligned and unaligned requests, null
and negative page-table entries, -1-padded cu_seqlens, 1/2/4-byte dtypes, out-of-range entries,
a Qwen3-sized layer, and the reference's validation errors. Bit-exact."""

import numpy as np
import pytest
import torch

from kvcache_manager import ops
from oracle import kvs_oracle as O
from test_paged_fill_oracle import random_case

pytestmark = pytest.mark.gpu

VIEW = {1: torch.uint8, 2: torch.int16, 4: torch.int32}


def run_gpu(k, v, cu, pt, sp, ck, cv, dtype, oor=None):
    """numpy uint16 inputs reinterpreted as `dtype` bytes; returns the caches as numpy uint16."""
    def dev(a):
        return torch.from_numpy(a.view(np.uint8).copy()).cuda().view(dtype)

    kd, vd = dev(k).reshape(1, *k.shape[:2], -1), dev(v).reshape(1, *v.shape[:2], -1)
    ckd, cvd = dev(ck).reshape(*ck.shape[:3], -1), dev(cv).reshape(*cv.shape[:3], -1)
    i32 = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.int32)).cuda()
    ops.paged_fill_cache_varlen(kd, vd, i32(cu), i32(pt), i32(sp), ckd, cvd, out_of_range=oor)
    torch.cuda.synchronize()
    back = lambda t: t.view(torch.uint8).cpu().numpy().view(np.uint16).reshape(ck.shape)
    return back(ckd), back(cvd)


@pytest.mark.parametrize("seed", range(8))
@pytest.mark.parametrize("aligned", [True, False])
def test_paged_fill_matches_oracle(seed, aligned):
    rng = np.random.default_rng(100 + seed)
    heads = int(rng.choice([1, 2, 8]))
    dim = int(rng.choice([32, 64, 128]))
    block_size = int(rng.choice([16, 32, 64])) if not aligned else int(rng.choice([32, 64]))
    batch = int(rng.integers(1, 6))
    k, v, cu, pt, sp, ck, cv, _ = random_case(rng, heads, dim, block_size, batch, aligned=aligned,
                                              pad_batch=int(rng.integers(0, 3)))
    exp_k, exp_v = ck.copy(), cv.copy()
    O.paged_fill_varlen(k, v, cu, pt, sp, exp_k, exp_v)
    dtype = [torch.bfloat16, torch.float8_e4m3fn, torch.float32][seed % 3]
    got_k, got_v = run_gpu(k, v, cu, pt, sp, ck, cv, dtype)
    assert np.array_equal(got_k, exp_k) and np.array_equal(got_v, exp_v)


@pytest.mark.parametrize("case", ["many_requests", "one_head_consecutive_blocks", "row_192B", "row_16KiB", "row_17KiB"])
def test_paged_fill_edge_cases(case):
    """32 or more requests (the binary-search lookup instead of the in-register one), one KV head
    over physically consecutive blocks, and rows of 192 B, 16 KiB and 17 KiB."""
    import zlib

    rng = np.random.default_rng(zlib.crc32(case.encode()))
    heads, dim, bs, batch = {"many_requests": (2, 64, 32, 37), "one_head_consecutive_blocks": (1, 128, 16, 4),
                             "row_192B": (2, 96, 16, 5), "row_16KiB": (1, 8192, 16, 2),
                             "row_17KiB": (1, 8704, 16, 2)}[case]
    long_requests = case in ("many_requests", "one_head_consecutive_blocks")  # 32-token multiples
    k, v, cu, pt, sp, ck, cv, _ = random_case(rng, heads, dim, bs, batch, aligned=long_requests, pad_batch=1)
    if case == "one_head_consecutive_blocks":
        pt = np.where(pt != 0, np.arange(1, pt.size + 1).reshape(pt.shape) % ck.shape[0], 0).astype(np.int32)
    exp_k, exp_v = ck.copy(), cv.copy()
    n_oor = O.paged_fill_varlen(k, v, cu, pt, sp, exp_k, exp_v)
    oor = torch.zeros(1, dtype=torch.int32, device="cuda")
    got_k, got_v = run_gpu(k, v, cu, pt, sp, ck, cv, torch.bfloat16, oor)
    assert np.array_equal(got_k, exp_k) and np.array_equal(got_v, exp_v)
    assert int(oor.item()) == n_oor


@pytest.mark.parametrize("n_layers", [1, 3, 70])
def test_paged_fill_layers_matches_oracle_per_layer(n_layers):
    """The all-layers fill (one launch per 64 layers) gives every layer the oracle's single-layer
    result, and counts each out-of-range token once."""
    rng = np.random.default_rng(40 + n_layers)
    k, v, cu, pt, sp, ck, cv, _ = random_case(rng, 2, 64, 16, 4, aligned=True, pad_batch=1)
    pt = pt.copy()
    r = int(np.argmax(np.diff(cu[:5]) > 0))  # a request with tokens: its last block is out of range
    pt[r, (int(sp[r]) + int(cu[r + 1] - cu[r]) - 1) // 16] = ck.shape[0] + 3
    dev = lambda a: torch.from_numpy(a.view(np.uint8).copy()).cuda().view(torch.bfloat16)
    i32 = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.int32)).cuda()
    ks, vs, cks, cvs, exp = [], [], [], [], []
    n_oor = None
    for layer in range(n_layers):
        lk, lv = (rng.integers(0, 1 << 16, k.shape, dtype=np.uint16) for _ in range(2))
        lck, lcv = (rng.integers(0, 1 << 16, ck.shape, dtype=np.uint16) for _ in range(2))
        ek, ev = lck.copy(), lcv.copy()
        n = O.paged_fill_varlen(lk, lv, cu, pt, sp, ek, ev)
        n_oor = n if n_oor is None else n_oor
        exp.append((ek, ev))
        ks.append(dev(lk).reshape(1, *k.shape))
        vs.append(dev(lv).reshape(1, *v.shape))
        cks.append(dev(lck).reshape(ck.shape))
        cvs.append(dev(lcv).reshape(cv.shape))
    oor = torch.zeros(1, dtype=torch.int32, device="cuda")
    ops.paged_fill_cache_varlen_layers(ks, vs, i32(cu), i32(pt), i32(sp), cks, cvs, out_of_range=oor)
    torch.cuda.synchronize()
    for layer, (ek, ev) in enumerate(exp):
        got_k = cks[layer].view(torch.uint8).cpu().numpy().view(np.uint16).reshape(ck.shape)
        got_v = cvs[layer].view(torch.uint8).cpu().numpy().view(np.uint16).reshape(cv.shape)
        assert np.array_equal(got_k, ek) and np.array_equal(got_v, ev), f"layer {layer}"
    assert int(oor.item()) == n_oor


def test_paged_fill_layers_validation():
    z = lambda *s, dt=torch.bfloat16: torch.zeros(*s, dtype=dt, device="cuda")
    i32 = lambda *s: torch.zeros(*s, dtype=torch.int32, device="cuda")
    k, c = [z(1, 2, 32, 64), z(1, 2, 32, 64)], [z(4, 2, 32, 64), z(4, 2, 32, 64)]
    ops.paged_fill_cache_varlen_layers(k, k, i32(2), i32(1, 2), i32(1), c, c)
    with pytest.raises(RuntimeError, match="same layers"):
        ops.paged_fill_cache_varlen_layers(k, k[:1], i32(2), i32(1, 2), i32(1), c, c)
    c5 = [c[0], z(5, 2, 32, 64)]
    with pytest.raises(RuntimeError, match="first layer's shapes"):
        ops.paged_fill_cache_varlen_layers(k, k, i32(2), i32(1, 2), i32(1), c5, c5)
    with pytest.raises(RuntimeError, match="must match cache_k dtype"):
        ops.paged_fill_cache_varlen_layers(k, k, i32(2), i32(1, 2), i32(1), [c[0], z(4, 2, 32, 64, dt=torch.float32)], c)


def test_paged_fill_out_of_range_is_skipped_and_counted():
    rng = np.random.default_rng(9)
    k, v, cu, pt, sp, ck, cv, _ = random_case(rng, 2, 64, 32, 3, aligned=True)
    cu = np.array([0, 96, 96 + int(cu[2] - cu[1]), 96 + int(cu[3] - cu[1])], np.int32)  # request 0: 96 tokens
    k = np.ascontiguousarray(np.concatenate([k, k], axis=1)[:, : max(k.shape[1], int(cu[3]) + 32)])
    v = np.ascontiguousarray(np.concatenate([v, v], axis=1)[:, : k.shape[1]])
    pt = np.concatenate([pt, np.zeros((pt.shape[0], 4), np.int32)], axis=1)
    pt[0, :] = ck.shape[0] + 5  # every block of request 0 is past the cache: skipped, not written
    pt[1:, :] = np.where(pt[1:, :] >= ck.shape[0], 0, pt[1:, :])
    sp = sp.copy()
    sp[1:] = 0
    exp_k, exp_v = ck.copy(), cv.copy()
    n_oor = O.paged_fill_varlen(k, v, cu, pt, sp, exp_k, exp_v)
    assert n_oor == 96
    oor = torch.zeros(1, dtype=torch.int32, device="cuda")
    got_k, got_v = run_gpu(k, v, cu, pt, sp, ck, cv, torch.bfloat16, oor)
    assert np.array_equal(got_k, exp_k) and np.array_equal(got_v, exp_v)
    assert int(oor.item()) == 96


def test_paged_fill_qwen3_layer():
    """8192 tokens of 4 requests, 8 KV heads x 128 bf16, 64-token blocks, chunked-prefill starts."""
    rng = np.random.default_rng(3)
    lens = [3072, 2048, 1024, 2048]
    starts = [0, 512, 4096, 64]
    bs, heads, dim = 64, 8, 128
    max_blocks = max((s + n + bs - 1) // bs for s, n in zip(starts, lens))
    nb = 4 * max_blocks + 1
    pt = rng.permutation(np.arange(1, nb))[: 4 * max_blocks].reshape(4, max_blocks).astype(np.int32)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    sp = np.array(starts, np.int32)
    k = rng.integers(0, 1 << 16, (heads, 8192, dim), dtype=np.uint16)
    v = rng.integers(0, 1 << 16, (heads, 8192, dim), dtype=np.uint16)
    ck = np.zeros((nb, heads, bs, dim), np.uint16)
    cv = np.zeros_like(ck)
    exp_k, exp_v = ck.copy(), cv.copy()
    assert O.paged_fill_varlen(k, v, cu, pt, sp, exp_k, exp_v) == 0
    got_k, got_v = run_gpu(k, v, cu, pt, sp, ck, cv, torch.bfloat16)
    assert np.array_equal(got_k, exp_k) and np.array_equal(got_v, exp_v)


def test_paged_fill_validation_errors():
    z = lambda *s, dt=torch.bfloat16: torch.zeros(*s, dtype=dt, device="cuda")
    i32 = lambda *s: torch.zeros(*s, dtype=torch.int32, device="cuda")
    args = dict(k_fill_value=z(1, 2, 32, 64), v_fill_value=z(1, 2, 32, 64), cu_seqlens=i32(2), page_table=i32(1, 2),
                start_positions=i32(1), cache_k=z(4, 2, 32, 64), cache_v=z(4, 2, 32, 64))
    ops.paged_fill_cache_varlen(**args)
    bad = [("k_fill_value", z(2, 2, 32, 64), "first dim must be 1"),
           ("cache_k", z(4, 2, 32, 64, dt=torch.float32), "must match cache_k dtype"),
           ("page_table", i32(1, 5), "must be <= max_num_blocks"),
           ("start_positions", i32(2), "must match batch_size"),
           ("cu_seqlens", z(2), "must be INT32"),
           ("cache_v", z(4, 2, 32, 64).cpu(), "must be on device")]
    for name, t, msg in bad:
        with pytest.raises(RuntimeError, match=msg):
            ops.paged_fill_cache_varlen(**dict(args, **{name: t}))
