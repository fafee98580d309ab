"""CPU tests of the oracle (no GPU): the C++ restatement against an independent
numpy restatement, exhaustive twiddle checks, and the committed golden
vectors produced by running the reference library itself."""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O
from tests import datagen as D

GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.mark.parametrize("kt", D.KEY_TYPES)
@pytest.mark.parametrize("desc", [False, True])
def test_oracle_matches_numpy(kt, desc):
    n = 20_000
    keys = D.special_floats(kt, n, seed=3, frac=0.02) if kt.startswith("f") else D.uniform_bits(kt, n, seed=3)
    vals = D.values_for(n, 4)
    kb = keys.dtype.itemsize
    for begin, end in [(0, 8 * kb), (1, 8 * kb - 1), (0, 1), (8 * kb - 5, 8 * kb)]:
        ok, ov = O.oracle_sort(kt, keys, vals, begin, end, desc)
        nk, nv = O.numpy_sort(kt, keys, vals, begin, end, desc)
        assert np.array_equal(ok.view(np.uint8), nk.view(np.uint8))
        assert np.array_equal(ov, nv)


@pytest.mark.parametrize("kt", ["u8", "i8", "u16", "i16"])
def test_twiddle_exhaustive_small(kt):
    kb = 1 if kt.endswith("8") else 2
    allv = np.arange(1 << (8 * kb), dtype=O.NP_UINT[kb]).view(O.NP_DTYPE[kt])
    for desc in (False, True):
        ok, _ = O.oracle_sort(kt, allv, None, 0, 8 * kb, desc)
        # full-width sort of every value is a plain numeric sort
        expect = np.sort(allv)[::-1] if desc else np.sort(allv)
        assert np.array_equal(ok, expect)


def test_float_total_order():
    v = np.array([1.0, -0.0, 0.0, np.inf, -np.inf, -1.0, np.nan, 2.5e-45, -2.5e-45], dtype=np.float32)
    u = v.view(np.uint32).copy()
    u[6] = 0x7FC00000
    neg_nan = np.array([0xFFC00000], dtype=np.uint32)
    keys = np.concatenate([u, neg_nan]).view(np.float32)
    ok, _ = O.oracle_sort("f32", keys)
    bits = ok.view(np.uint32).tolist()
    assert bits == [0xFFC00000, 0xFF800000, 0xBF800000, 0x80000002, 0x80000000, 0x00000000, 0x00000002,
                    0x3F800000, 0x7F800000, 0x7FC00000]


def test_descending_keeps_equal_keys_in_input_order():
    keys = np.array([3, 1, 3, 2, 1, 3], dtype=np.int32)
    vals = np.arange(6, dtype=np.uint32)
    ok, ov = O.oracle_sort("i32", keys, vals, descending=True)
    assert ok.tolist() == [3, 3, 3, 2, 1, 1]
    assert ov.tolist() == [0, 2, 5, 3, 1, 4]


def test_histogram_matches_numpy():
    keys = D.uniform_bits("f64", 5000, seed=2)
    h = O.oracle_histogram("f64", keys, 3, 61, True)
    dk = O.numpy_digit_keys("f64", keys, 0, 64, True)
    for p in range(h.shape[0]):
        sh = 3 + 8 * p
        w = min(8, 61 - sh)
        d = (dk >> np.uint64(sh)) & np.uint64((1 << w) - 1)
        assert np.array_equal(h[p], np.bincount(d.astype(np.int64), minlength=256))


def _golden_cases():
    if not (GOLDEN / "index.json").exists():
        return []
    return json.loads((GOLDEN / "index.json").read_text())["cases"]


@pytest.mark.parametrize("case", _golden_cases(), ids=lambda c: c["name"])
def test_oracle_against_reference_golden(case):
    """Golden vectors were produced by the reference libcusort on a B200."""
    z = np.load(GOLDEN / case["file"])
    kt = case["key_type"]
    keys = z["keys_in"]
    vals = z["values_in"] if "values_in" in z.files else None
    ok, ov = O.oracle_sort(kt, keys, vals, case["begin_bit"], case["end_bit"], case["descending"])
    assert np.array_equal(ok.view(np.uint8), z["keys_out"].view(np.uint8))
    if vals is not None:
        assert np.array_equal(ov.view(np.uint8), z["values_out"].view(np.uint8))


def test_golden_vectors_present():
    assert _golden_cases(), "tests/golden/index.json missing: the oracle is not pinned to the reference"
