"""The token-granular paged KV fill of the oracle against the reference's own
moreh_paged_fill_cache_varlen reader and writer kernels, compiled from patch 0002 by
oracle/build_ref.py and run on host buffers, for tile-aligned random geometries (where the
reference's 32-token tiles and single tokens give the same result); plus the oracle's behaviour
on its own for unaligned requests, null / negative page-table entries and -1-padded cu_seqlens."""

import ctypes as C
from pathlib import Path

import numpy as np
import pytest

from oracle import kvs_oracle as O

LIB = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "libkvs_ref.so"
T = 32  # tile edge


def random_case(rng, heads, dim, block_size, batch, aligned=True, pad_batch=0):
    unit = T if aligned else 1
    lens = [int(rng.integers(0, 5)) * unit + (0 if aligned else int(rng.integers(0, 7))) for _ in range(batch)]
    starts = [int(rng.integers(0, 4)) * (T if aligned else 1) * (1 if aligned else int(rng.integers(1, 40)))
              for _ in range(batch)]
    valid = sum(lens)
    total = (valid + T - 1) // T * T + T * int(rng.integers(0, 2))  # tile-padded, maybe an extra tile
    total = max(total, T)
    max_blocks = max(1, max((s + n + block_size - 1) // block_size for s, n in zip(starts, lens)))
    n_blocks = batch * max_blocks + 3
    phys = rng.permutation(np.arange(1, n_blocks))[: batch * max_blocks].reshape(batch, max_blocks).astype(np.int32)
    mask = rng.random(phys.shape)
    phys[mask < 0.1] = 0    # vLLM's null block
    phys[mask > 0.92] = -1  # unused / other DP group
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    full_batch = batch + pad_batch
    cu = np.concatenate([cu, -np.ones(pad_batch, np.int32)])
    pt = np.concatenate([phys, np.zeros((pad_batch, max_blocks), np.int32)])
    sp = np.array(starts + [0] * pad_batch, np.int32)
    k = rng.integers(0, 1 << 16, (heads, total, dim), dtype=np.uint16)
    v = rng.integers(0, 1 << 16, (heads, total, dim), dtype=np.uint16)
    ck = rng.integers(0, 1 << 16, (n_blocks, heads, block_size, dim), dtype=np.uint16)
    cv = rng.integers(0, 1 << 16, (n_blocks, heads, block_size, dim), dtype=np.uint16)
    return k, v, cu, pt, sp, ck, cv, full_batch


def tilize(a):
    """(..., rows, cols) -> (..., rows/32, cols/32, 32, 32): 32 x 32 tiles, row-major inside."""
    *lead, r, c = a.shape
    t = a.reshape(*lead, r // T, T, c // T, T)
    return np.moveaxis(t, -2, -3).copy()  # always a new array, never a view of `a`


def untilize(t):
    *lead, rt, ct, _, _ = t.shape
    return np.moveaxis(t, -3, -2).copy().reshape(*lead, rt * T, ct * T)


@pytest.mark.skipif(not LIB.exists(), reason="oracle/_ref not built (needs the reference checkout)")
@pytest.mark.parametrize("seed", range(12))
def test_token_fill_matches_reference_kernels_on_tile_aligned_inputs(seed):
    rng = np.random.default_rng(seed)
    heads = int(rng.choice([1, 2, 4]))
    dim = int(rng.choice([32, 64, 128]))
    block_size = int(rng.choice([32, 64]))
    batch = int(rng.integers(1, 5))
    k, v, cu, pt, sp, ck, cv, full = random_case(rng, heads, dim, block_size, batch, pad_batch=int(rng.integers(0, 3)))
    exp_k, exp_v = ck.copy(), cv.copy()
    oor = O.paged_fill_varlen(k, v, cu, pt, sp, exp_k, exp_v)
    assert oor == 0
    ref = C.CDLL(str(LIB))
    ref.ref_paged_fill_varlen.restype = C.c_int
    kt, vt = tilize(k), tilize(v)
    ckt, cvt = tilize(ck), tilize(cv)
    P = lambda a: a.ctypes.data_as(C.c_void_p)
    rc = ref.ref_paged_fill_varlen(P(kt), P(vt), heads, k.shape[1], dim, T * T * 2, P(cu), full, P(pt), pt.shape[1],
                                   P(sp), P(ckt), P(cvt), ck.shape[0], block_size)
    assert rc == 0
    assert np.array_equal(untilize(ckt), exp_k)
    assert np.array_equal(untilize(cvt), exp_v)
    assert not np.array_equal(exp_k, ck) or cu[batch] == 0  # something was written


def test_token_fill_unaligned_and_skips():
    rng = np.random.default_rng(5)
    k, v, cu, pt, sp, ck, cv, full = random_case(rng, 2, 16, 16, 4, aligned=False, pad_batch=2)
    exp_k = ck.copy()
    exp_v = cv.copy()
    O.paged_fill_varlen(k, v, cu, pt, sp, exp_k, exp_v)
    # restate the expected result directly, token by token
    want_k, want_v = ck.copy(), cv.copy()
    valid = int(cu[: full + 1][cu[: full + 1] >= 0].max())
    for t in range(min(valid, k.shape[1])):
        r = max(i for i in range(full + 1) if 0 <= cu[i] <= t)
        pos = t - cu[r] + sp[r]
        b = pt[r, pos // 16]
        if b <= 0:
            continue
        want_k[b, :, pos % 16] = k[:, t]
        want_v[b, :, pos % 16] = v[:, t]
    assert np.array_equal(exp_k, want_k) and np.array_equal(exp_v, want_v)
