"""Bit-exact parity of the 64-bit offset kernels, which sorts of 2^30 items
and more select (reference: libcusort.cuh:2955-2960), on inputs small enough
for the CPU oracle: the test hook CUSORT_WIDE_OFFSETS=1 makes every sort use
them.  Every key width with every value width, skewed keys (the tiles of
these kernels were re-sized so that the 32-bit warp counters fit), descending
order, partial bit ranges, the DoubleBuffer form, the one-digit paths of
1- and 2-byte keys and the multi-tile segments of the segmented sort.  At
every shape the onesweep kernel keeps two CTAs on each SM.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from libcusort_b200 import _capi  # noqa: E402
from oracle import oracle as O  # noqa: E402
from tests import datagen as D  # noqa: E402
from tests.gpu_helpers import run_ours, same_bits  # noqa: E402

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("no CUDA device", allow_module_level=True)

CORES = os.cpu_count() or 1
N = 1_500_000


@pytest.fixture(autouse=True)
def wide(monkeypatch):
    monkeypatch.setenv("CUSORT_WIDE_OFFSETS", "1")


def _keys(kt, n, seed):
    return D.special_floats(kt, n, seed=seed) if kt.startswith("f") else D.uniform_bits(kt, n, seed=seed)


def _check(kt, keys, vals, begin=0, end=None, desc=False, api="raw"):
    ek, ev = O.oracle_sort(kt, keys, vals, begin, end, desc, threads=CORES)
    ko, vo, _ = run_ours(kt, keys, vals, begin, end, desc, api=api)
    where = f"{kt} vb={0 if vals is None else vals.dtype.itemsize} bits=[{begin},{end}) desc={desc} api={api}"
    assert same_bits(ko, ek), f"keys differ: {where}"
    if vals is not None:
        assert same_bits(vo, ev), f"values differ: {where}"


@pytest.mark.parametrize("kt", ["u8", "i16", "u32", "f32", "i64", "f64"])
@pytest.mark.parametrize("vb", [0, 1, 2, 4, 8, 16])
def test_wide_offsets_every_width(kt, vb):
    lib = _capi.load()
    off, grid = C.c_int(0), C.c_int(0)
    kid = _capi.KEY_TYPES[kt]
    bits = 8 * _capi.KEY_BYTES[kt]
    if vb == 0 and bits <= 16:
        bits -= 1  # the full range of 1- and 2-byte keys counts and fills instead (no onesweep)
    assert lib.cusort_query_plan(kid, vb, 1 << 26, 0, bits, None, None, C.byref(grid), None, C.byref(off)) == 0
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    assert off.value == 8 and grid.value == 2 * sms, "two onesweep CTAs per SM"
    keys = _keys(kt, N, seed=40 + vb)
    _check(kt, keys, D.values_for(N, vb) if vb else None)


@pytest.mark.parametrize("vb", [0, 1, 2, 4, 16])
def test_wide_offsets_skewed_u32(vb):
    keys = D.zipf_table("u32", N, seed=41, distinct=4096, s=1.1)
    _check("u32", keys, D.values_for(N, vb) if vb else None)


@pytest.mark.parametrize("kt", ["i32", "u64", "f64"])
def test_wide_offsets_descending_and_bit_ranges(kt):
    keys = _keys(kt, N, seed=42)
    vals = D.values_for(N, 4)
    bits = 8 * keys.dtype.itemsize
    _check(kt, keys, vals, desc=True)
    _check(kt, keys, vals, 3, bits - 5)
    _check(kt, keys, vals, 0, 13, desc=True)


@pytest.mark.parametrize("kt,vb", [("u32", 4), ("u64", 8), ("u16", 0), ("f32", 0)])
def test_wide_offsets_double_buffer(kt, vb):
    keys = _keys(kt, N, seed=43)
    _check(kt, keys, D.values_for(N, vb) if vb else None, api="db")


@pytest.mark.parametrize("kt", ["u8", "i8", "u16", "i16"])
def test_wide_offsets_one_digit_paths(kt):
    # full-range keys-only sorts of 1- and 2-byte keys count and fill with 64-bit counts
    keys = _keys(kt, N, seed=44)
    keys[: N // 4] = keys[7]  # one heavy value
    for desc in (False, True):
        _check(kt, keys, None, desc=desc)


def test_wide_offsets_segmented():
    from tests.test_segmented_gpu import lengths_segments, run_segmented
    rng = np.random.default_rng(45)
    lengths = np.exp(rng.uniform(0, np.log(60_000), size=80)).astype(np.int64)
    lengths[:3] = [0, 90_000, 150_000]  # multi-tile segments take the onesweep passes
    b, e, n = lengths_segments(lengths.tolist(), gap=2)
    for kt, vb in (("i32", 4), ("u32", 0), ("f64", 16)):
        keys = _keys(kt, n, seed=46)
        vals = D.values_for(n, vb) if vb else None
        ko, vo, ek, ev = run_segmented(kt, keys, vals, b, e)
        assert same_bits(ko, ek)
        if vb:
            assert same_bits(vo, ev)
