"""GPU parity of the segmented sort (cusort_segmented_sort_keys/_pairs)
against the CPU oracle, bit-exact: every length class (one warp, one CTA,
multi-tile onesweep segments), empty segments, gaps and unordered segments,
partial bit ranges, both directions, key/value widths, and positions outside
every segment left as they were."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from libcusort_b200 import _capi  # noqa: E402
from oracle import oracle as O  # noqa: E402
from tests import datagen as D  # noqa: E402
from tests.gpu_helpers import DevBuf, same_bits  # noqa: E402
from tests.test_segmented_host import random_segments  # noqa: E402

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("no CUDA device", allow_module_level=True)


def run_segmented(kt, keys, values, begins, ends, begin_bit=0, end_bit=None, desc=False):
    lib = _capi.load()
    n = keys.shape[0]
    end_bit = 8 * keys.dtype.itemsize if end_bit is None else end_bit
    vb = 0 if values is None else values.dtype.itemsize * int(np.prod(values.shape[1:], dtype=np.int64))
    pre_k = D.uniform_bits(kt, n, seed=1234)
    pre_v = None if values is None else np.full(values.shape, 0x5A, dtype=values.dtype)
    kin, kout = DevBuf.from_array(keys), DevBuf.from_array(pre_k)
    vin = DevBuf.from_array(values) if vb else None
    vout = DevBuf.from_array(pre_v) if vb else None
    b_d = torch.from_numpy(np.asarray(begins, dtype=np.int64)).cuda()
    e_d = torch.from_numpy(np.asarray(ends, dtype=np.int64)).cuda()
    S = len(begins)
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    nb = C.c_size_t(0)
    P = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    kid = _capi.KEY_TYPES[kt]

    def call(temp):
        if vb:
            return lib.cusort_segmented_sort_pairs(temp, C.byref(nb), kid, kin.ptr, kout.ptr, vb, vin.ptr, vout.ptr,
                                                   n, S, P(b_d), P(e_d), begin_bit, end_bit, int(desc), stream)
        return lib.cusort_segmented_sort_keys(temp, C.byref(nb), kid, kin.ptr, kout.ptr, n, S, P(b_d), P(e_d),
                                              begin_bit, end_bit, int(desc), stream)

    assert call(None) == 0
    temp = DevBuf(nb.value)
    assert call(temp.ptr) == 0
    torch.cuda.synchronize()
    st = C.c_uint32(0)
    assert lib.cusort_read_device_status(temp.ptr, C.byref(st), stream) == 0 and st.value == 0
    assert all(x.guards_ok() for x in (kin, kout, temp) + ((vin, vout) if vb else ()))
    ko = kout.to_array(keys)
    vo = vout.to_array(values) if vb else None
    ek, ev = O.oracle_segmented_sort(kt, keys, values, begins, ends, begin_bit, end_bit, desc, pre_k, pre_v)
    return ko, vo, ek, ev


def lengths_segments(lengths, gap=0):
    b, e, pos = [], [], 0
    for m in lengths:
        b.append(pos)
        e.append(pos + m)
        pos += m + gap
    return np.array(b, dtype=np.int64), np.array(e, dtype=np.int64), pos


@pytest.mark.parametrize("kt", ["u32", "i32", "f32", "u8", "i16", "u64", "f64"])
@pytest.mark.parametrize("vb", [0, 4])
def test_segmented_mixed_lengths(kt, vb):
    rng = np.random.default_rng(5)
    # log-uniform lengths 0 .. 60k: warp, CTA and multi-tile classes
    lengths = np.exp(rng.uniform(0, np.log(60_000), size=120)).astype(np.int64)
    lengths[:5] = [0, 1, 2, 0, 70_000]
    b, e, n = lengths_segments(lengths.tolist(), gap=3)
    keys = D.special_floats(kt, n, seed=2) if kt.startswith("f") else D.uniform_bits(kt, n, seed=2)
    vals = np.arange(n, dtype=np.uint32) if vb else None
    ko, vo, ek, ev = run_segmented(kt, keys, vals, b, e)
    assert same_bits(ko, ek)
    if vb:
        assert same_bits(vo, ev)


@pytest.mark.parametrize("max_len", [1, 33, 600, 5000])
@pytest.mark.parametrize("desc", [False, True])
def test_segmented_random_segmentations(max_len, desc):
    rng = np.random.default_rng(max_len)
    n = 300_000
    b, e = random_segments(n, rng, max_len)  # gaps, unordered
    keys = D.zipf_table("i32", n, seed=4, distinct=512)  # many ties: stability matters
    vals = np.arange(n, dtype=np.uint32)
    ko, vo, ek, ev = run_segmented("i32", keys, vals, b, e, 0, 32, desc)
    assert same_bits(ko, ek) and same_bits(vo, ev)


@pytest.mark.parametrize("kt,begin,end", [("u32", 0, 20), ("f32", 3, 29), ("i64", 8, 48), ("u16", 4, 12),
                                          ("u32", 9, 9)])
def test_segmented_bit_ranges(kt, begin, end):
    lengths = [0, 5, 300, 3000, 25_000, 1, 100_000, 17]
    b, e, n = lengths_segments(lengths, gap=1)
    keys = D.uniform_bits(kt, n, seed=begin + end)
    vals = np.arange(n, dtype=np.uint32)
    ko, vo, ek, ev = run_segmented(kt, keys, vals, b, e, begin, end, True)
    assert same_bits(ko, ek) and same_bits(vo, ev)


@pytest.mark.parametrize("vb", [1, 2, 8, 16])
def test_segmented_value_widths(vb):
    lengths = [7, 700, 7000, 70_000]
    b, e, n = lengths_segments(lengths)
    keys = D.uniform_bits("f64", n, seed=vb)
    vals = D.values_for(n, vb)
    ko, vo, ek, ev = run_segmented("f64", keys, vals, b, e)
    assert same_bits(ko, ek) and same_bits(vo, ev)


def test_segmented_one_segment_equals_plain_sort():
    n = (1 << 20) + 3
    keys = D.uniform_bits("u32", n, seed=8)
    vals = np.arange(n, dtype=np.uint32)
    ko, vo, ek, ev = run_segmented("u32", keys, vals, [0], [n])
    pk, pv = O.oracle_sort("u32", keys, vals)
    assert same_bits(ko, ek) and same_bits(vo, ev) and same_bits(ko, pk) and same_bits(vo, pv)


def test_segmented_many_tiny_segments():
    n = 200_000
    lengths = (np.arange(n // 4) % 9).tolist()
    b, e, _ = lengths_segments(lengths)
    m = int(e[-1])
    keys = D.uniform_bits("u16", m, seed=9)
    vals = np.arange(m, dtype=np.uint32)
    ko, vo, ek, ev = run_segmented("u16", keys, vals, b, e)
    assert same_bits(ko, ek) and same_bits(vo, ev)


@pytest.mark.parametrize("kt", ["f64", "i8", "u32"])
def test_segmented_class_boundaries(kt):
    # lengths at the edges of the tiny class's item slots (32, 64, 96, 128: its capacity) and of the
    # one-warp, two-warp, four-warp, CTA and large-CTA classes (their capacities are 32, 64, 128, 256
    # and 512 x the items per thread: 16 for items of up to 8 bytes, 8 up to 16; items of up to 8
    # bytes also have a one-warp kernel of 8 items per thread, up to 256), with many ties
    lengths = [31, 32, 33, 63, 64, 65, 96, 97, 127, 128, 129, 255, 256, 257, 511, 512, 513, 1023, 1024, 1025,
               2047, 2048, 2049, 4095, 4096, 4097, 8191, 8192, 8193, 2, 1, 0] * 3
    b, e, n = lengths_segments(lengths, gap=2)
    rng = np.random.default_rng(11)
    keys = D.uniform_bits(kt, 64, seed=12)[rng.integers(0, 64, size=n)]
    vals = np.arange(n, dtype=np.uint32)
    for desc in (False, True):
        ko, vo, ek, ev = run_segmented(kt, keys, vals, b, e, 0, 8 * keys.dtype.itemsize, desc)
        assert same_bits(ko, ek) and same_bits(vo, ev)
