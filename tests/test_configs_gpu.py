"""Bit-exact parity at the exact sizes and distributions of every single-GPU
benchmark configuration, so the tile shapes, skew behaviour and short-circuit
paths that those sizes select are the ones checked:

  configs[0]  2^20 uint32 keys-only, uniform over all 32 bits, ascending
  configs[1]  2^26 int32 keys uniform (and low-entropy a & b & c) + uint32
              index values, SortPairs ascending, in/out and DoubleBuffer forms
  configs[2]  2^26 keys-only dtype sweep, ascending and descending: int8..int64
              uniform over the full width; float/double N(0, 1e3) with 0.1 %
              each of -0.0, +0.0, +inf, -inf and quiet NaN
  configs[3]  2^26 double keys N(0, 1) + 16-byte values (i, ~i); 2^26 uint32
              keys over bits [0, 20) drawn Zipf(1.1) from 65,536 seeded values
              spanning all 32 bits + uint32 index values, and the companion
              whose table values are < 2^16 (a pass whose digit is constant)

Each case is compared bit for bit with (a) the CPU oracle (a parallel stable
sort on the masked twiddled key) and (b) the reference library built from the
unmodified libcusort.cuh on the same inputs through its own public API
(libcusort.cuh:2972-3104), when that build is present.  Values carry the
original index, so equality with the oracle also proves stability.
"""
from __future__ import annotations

import gc
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import oracle as O  # noqa: E402
from tests import datagen as D  # noqa: E402
from tests.gpu_helpers import run_ours, run_ref, same_bits  # noqa: E402

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("no CUDA device", allow_module_level=True)

N26 = 1 << 26
CORES = os.cpu_count() or 1
HAVE_REF = O.ref_available()


def parity(kt, keys, values=None, begin=0, end=None, desc=False, apis=("raw",)):
    """Ours (each API form) == oracle == reference, bit for bit."""
    ek, ev = O.oracle_sort(kt, keys, values, begin, end, desc, threads=CORES)
    for api in apis:
        ko, vo, info = run_ours(kt, keys, values, begin, end, desc, api=api)
        where = f"{kt} n={len(keys)} bits=[{begin},{end}) desc={desc} api={api}"
        assert same_bits(ko, ek), f"keys differ from the oracle: {where}"
        if values is not None:
            assert same_bits(vo, ev), f"values differ from the oracle: {where}"
        del ko, vo
        if HAVE_REF:
            rk, rv, rinfo = run_ref(kt, keys, values, begin, end, desc, api=api)
            assert same_bits(rk, ek), f"reference keys differ: {where}"
            if values is not None:
                assert same_bits(rv, ev), f"reference values differ: {where}"
            if api == "db":
                assert info["ksel"] == rinfo["ksel"] and (values is None or info["vsel"] == rinfo["vsel"])
            del rk, rv
        gc.collect()


def test_config0_u32_keys_2p20():
    keys = D.uniform_bits("u32", 1 << 20, seed=1)
    parity("u32", keys, apis=("raw", "db"))


@pytest.mark.parametrize("dist", ["uniform", "low_entropy"])
def test_config1_i32_u32_pairs_2p26(dist):
    keys = D.uniform_bits("i32", N26, seed=2) if dist == "uniform" else D.low_entropy("i32", N26, seed=3)
    vals = D.values_for(N26, 4)
    parity("i32", keys, vals, apis=("raw", "db"))


@pytest.mark.parametrize("kt", ["i8", "i16", "i32", "i64", "f32", "f64"])
def test_config2_dtype_sweep_2p26(kt):
    keys = D.special_floats(kt, N26, seed=5, scale=1e3) if kt.startswith("f") else D.uniform_bits(kt, N26, seed=4)
    if kt.startswith("f"):
        bits = keys.view(O.NP_UINT[keys.dtype.itemsize])
        # the specials are present: +-0, +-inf and NaN
        assert np.isnan(keys).any() and np.isinf(keys).any() and (bits == (1 << (8 * keys.dtype.itemsize - 1))).any()
    for desc in (False, True):
        parity(kt, keys, None, desc=desc)


def test_config3_f64_keys_16B_values_2p26():
    rng = np.random.default_rng(6)
    keys = rng.standard_normal(N26)
    vals = D.values_for(N26, 16)  # (index, ~index)
    parity("f64", keys, vals)


@pytest.mark.parametrize("below", [None, 16])
def test_config3_u32_zipf_bits_0_20_2p26(below):
    keys = D.zipf_table("u32", N26, seed=7, distinct=65536, s=1.1, below=below)
    if below is None:
        assert (keys >> 20).any(), "bits above the sorted range must vary (and be carried through)"
    else:
        assert (keys >> 16).max() == 0  # digit of the third pass (bits 16..19) is constant
    vals = D.values_for(N26, 4)
    parity("u32", keys, vals, 0, 20)
