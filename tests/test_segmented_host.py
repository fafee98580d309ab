"""Segmented-sort oracle on CPU: the per-segment C++ oracle and the numpy
lexsort restatement agree on segmentations with empty segments, gaps,
unordered segments and partial bit ranges; positions outside every segment
keep the prefilled output.  Also: the C ABI size query needs no GPU and does
not depend on the offsets."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from oracle import oracle as O
from tests import datagen as D


def random_segments(n, rng, max_len, gap_p=0.2, shuffle=True):
    begins, ends, pos = [], [], 0
    while pos < n:
        if rng.random() < gap_p:
            pos += int(rng.integers(1, 5))
            continue
        m = int(rng.integers(0, max_len + 1))
        e = min(n, pos + m)
        begins.append(pos)
        ends.append(e)
        pos = e
    order = rng.permutation(len(begins)) if shuffle else np.arange(len(begins))
    return np.array(begins, dtype=np.int64)[order], np.array(ends, dtype=np.int64)[order]


@pytest.mark.parametrize("kt", ["u8", "i16", "f32", "i64", "f64"])
@pytest.mark.parametrize("desc", [False, True])
@pytest.mark.parametrize("max_len", [3, 40, 2000])
def test_segmented_oracles_agree(kt, desc, max_len):
    rng = np.random.default_rng(max_len + (7 if desc else 0))
    n = 20_000
    keys = D.special_floats(kt, n, seed=3) if kt.startswith("f") else D.uniform_bits(kt, n, seed=3)
    vals = np.arange(n, dtype=np.uint32)
    b, e = random_segments(n, rng, max_len)
    pre_k = D.uniform_bits(kt, n, seed=99)
    pre_v = np.full(n, 0xFFFFFFFF, dtype=np.uint32)
    bb, eb = (3, 8 * keys.dtype.itemsize - 1) if kt != "u8" else (0, 8)
    k1, v1 = O.oracle_segmented_sort(kt, keys, vals, b, e, bb, eb, desc, pre_k, pre_v)
    k2, v2 = O.numpy_segmented_sort(kt, keys, vals, b, e, bb, eb, desc, pre_k, pre_v)
    assert np.array_equal(k1.view(np.uint8), k2.view(np.uint8)) and np.array_equal(v1, v2)
    covered = np.zeros(n, dtype=bool)
    for x, y in zip(b, e):
        covered[x:max(x, y)] = True
    assert np.array_equal(v1[~covered], pre_v[~covered])
    # every segment holds a permutation of its own items
    for x, y in zip(b.tolist(), e.tolist()):
        if y > x:
            assert np.array_equal(np.sort(v1[x:y]), np.arange(x, y, dtype=np.uint32))


def test_segmented_size_query_needs_no_gpu():
    from libcusort_b200 import _capi
    lib = _capi.load()
    nb = C.c_size_t(0)
    rc = lib.cusort_segmented_sort_pairs(None, C.byref(nb), _capi.KEY_TYPES["u32"], None, None, 4, None, None,
                                         1 << 20, 1000, None, None, 0, 32, 0, None)
    assert rc == 0 and nb.value > 0
    nk = C.c_size_t(0)
    assert lib.cusort_segmented_sort_keys(None, C.byref(nk), _capi.KEY_TYPES["u32"], None, None, 1 << 20, 5,
                                          None, None, 0, 32, 0, None) == 0
    assert 0 < nk.value < nb.value
    bad = lib.cusort_segmented_sort_keys(None, C.byref(nk), _capi.KEY_TYPES["u32"], None, None, 10, 1, None, None,
                                         0, 33, 0, None)
    assert bad != 0
