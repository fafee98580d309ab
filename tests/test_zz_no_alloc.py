"""The no-allocation entry point (cusort_sort_db_noalloc).

It exists for callers that cannot allocate device memory when they sort (an
allocator hook sorting its own free lists, a plugin whose host process has
reserved all device memory, a latency-bound loop that must not let cudaMalloc
synchronise the device).  Its results must equal the CPU oracle's (a stable
sort, bit for bit) and the ordinary DoubleBuffer entry points' (which take
caller temp storage, selectors included), also on a second call that reuses
the library's scratch array; a call must leave the device's free memory
unchanged; and sizes that do not fit the array must be refused.  This file is
collected last on purpose.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from libcusort_b200 import _capi  # noqa: E402
from oracle import oracle as O  # noqa: E402
from tests import datagen as D  # noqa: E402
from tests.gpu_helpers import DevBuf, run_ours, same_bits  # noqa: E402

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("no CUDA device", allow_module_level=True)

SCRATCH_BYTES = 4 << 20  # CUSORT_NOALLOC_SCRATCH_BYTES in include/cusort_b200.h


def _stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def sort_noalloc(kt, keys, values=None, begin_bit=0, end_bit=None, descending=False):
    """One call through the C ABI; returns (rc, keys, values, key selector, value selector)."""
    lib = _capi.load()
    n = keys.shape[0]
    end_bit = 8 * keys.dtype.itemsize if end_bit is None else end_bit
    vb = 0 if values is None else values.dtype.itemsize * int(np.prod(values.shape[1:], dtype=np.int64))
    k0, k1 = DevBuf.from_array(keys), DevBuf(keys.nbytes)
    kdb = _capi.DoubleBufferC()
    kdb.d_buffers[0], kdb.d_buffers[1], kdb.selector = k0.ptr.value, k1.ptr.value, 0
    vdb = _capi.DoubleBufferC()
    vbufs = []
    if vb:
        vbufs = [DevBuf.from_array(values), DevBuf(values.nbytes)]
        vdb.d_buffers[0], vdb.d_buffers[1], vdb.selector = vbufs[0].ptr.value, vbufs[1].ptr.value, 0
    rc = lib.cusort_sort_db_noalloc(_capi.KEY_TYPES[kt], C.byref(kdb), vb, C.byref(vdb) if vb else None, n,
                                    begin_bit, end_bit, int(descending), _stream())
    torch.cuda.synchronize()
    if rc != 0:
        return rc, None, None, None, None
    ko = (k0, k1)[kdb.selector].to_array(keys)
    vo = vbufs[vdb.selector].to_array(values) if vb else None
    for b in [k0, k1] + vbufs:
        assert b.guards_ok()
    return rc, ko, vo, kdb.selector, vdb.selector


def test_no_alloc_matches_oracle_on_two_calls():
    # Two calls in a row: the second reuses (and must re-clear) the scratch.
    cases = [("i32", 1 << 20, 4, False, 0, 32, 11), ("f64", 300_001, 16, True, 3, 61, 12),
             ("i32", 1 << 20, 4, False, 0, 32, 14)]
    for kt, n, vb, desc, b, e, seed in cases:
        keys = D.special_floats(kt, n, seed=seed) if kt.startswith("f") else D.uniform_bits(kt, n, seed=seed)
        vals = D.values_for(n, vb)
        ek, ev = O.oracle_sort(kt, keys, vals, b, e, desc)
        rc, ko, vo, ks, vs = sort_noalloc(kt, keys, vals, b, e, desc)
        assert rc == 0
        assert same_bits(ko, ek) and same_bits(vo, ev), f"differs from the oracle ({kt}, n={n})"
        # same selector updates as the allocating DoubleBuffer entry point
        _, _, info = run_ours(kt, keys, vals, b, e, desc, api="db")
        assert (ks, vs) == (info["ksel"], info["vsel"])


def test_no_alloc_keys_only_matches_oracle():
    keys = D.uniform_bits("u32", 2_000_000, seed=13)
    ek, _ = O.oracle_sort("u32", keys, None, 0, 20)
    for _ in range(2):
        rc, ko, _, ks, _ = sort_noalloc("u32", keys, None, 0, 20)
        assert rc == 0
        assert same_bits(ko, ek)
        assert ks == 1  # 3 passes flip the selector once per pass


def test_no_alloc_call_leaves_free_memory_unchanged():
    lib = _capi.load()
    n = 1 << 20
    keys = D.uniform_bits("i32", n, seed=21)
    vals = D.values_for(n, 4)
    k0, k1 = DevBuf.from_array(keys), DevBuf(keys.nbytes)
    v0, v1 = DevBuf.from_array(vals), DevBuf(vals.nbytes)
    kdb, vdb = _capi.DoubleBufferC(), _capi.DoubleBufferC()

    def call():
        kdb.d_buffers[0], kdb.d_buffers[1], kdb.selector = k0.ptr.value, k1.ptr.value, 0
        vdb.d_buffers[0], vdb.d_buffers[1], vdb.selector = v0.ptr.value, v1.ptr.value, 0
        rc = lib.cusort_sort_db_noalloc(_capi.KEY_TYPES["i32"], C.byref(kdb), 4, C.byref(vdb), n, 0, 32, 0,
                                        _stream())
        torch.cuda.synchronize()
        return rc

    assert call() == 0  # warm-up: the first call may load the library's device code
    free0, _ = torch.cuda.mem_get_info()
    assert call() == 0
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, f"free device memory changed across a call: {free0} -> {free1}"


def test_no_alloc_rejects_sizes_beyond_the_scratch():
    n = 1 << 27  # needs ~7 MiB of temp storage, more than the fixed scratch
    lib = _capi.load()
    need = C.c_size_t(0)
    db = _capi.DoubleBufferC()
    assert lib.cusort_sort_keys_db(None, C.byref(need), _capi.KEY_TYPES["u32"], C.byref(db), n, 0, 32, None) == 0
    assert need.value > SCRATCH_BYTES
    keys = np.zeros(n, dtype=np.uint32)
    rc, *_ = sort_noalloc("u32", keys)
    assert rc == _capi.CUDA_ERROR_INVALID_VALUE
    # the library still works afterwards
    small = D.uniform_bits("u32", 5000, seed=1)
    rc, ko, _, _, _ = sort_noalloc("u32", small)
    assert rc == 0 and same_bits(ko, np.sort(small))
