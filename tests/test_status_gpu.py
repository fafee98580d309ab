"""Bounded device waits (failure detection without a GPU fault).

A test-only switch makes one tile never publish its lookback descriptors, so
every later tile's wait on it runs out; the kernels must then return (no
hang, no trap), raise the lookback-timeout bit in the device status word,
and leave the context usable for the next sort.
"""
from __future__ import annotations

import ctypes as C
import time

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


def test_lookback_timeout_sets_status_and_context_survives():
    lib = _capi.load()
    n = 1 << 20
    keys = D.uniform_bits("u32", n, seed=1)
    kin = DevBuf.from_array(keys)
    kout = DevBuf(keys.nbytes)
    nb = C.c_size_t(0)
    assert lib.cusort_sort_keys(None, C.byref(nb), 4, kin.ptr, kout.ptr, n, 0, 32, None) == 0
    temp = DevBuf(nb.value)
    prev_limit = lib.cusort_set_wait_limit_ns(50_000_000)  # 50 ms
    prev_skip = lib.cusort_debug_set_skip_tile(3)
    try:
        t0 = time.time()
        stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
        rc = lib.cusort_sort_keys(temp.ptr, C.byref(nb), 4, kin.ptr, kout.ptr, n, 0, 32, stream)
        assert rc == 0
        st = C.c_uint32(0)
        assert lib.cusort_read_device_status(temp.ptr, C.byref(st), stream) == 0
        elapsed = time.time() - t0
    finally:
        lib.cusort_debug_set_skip_tile(prev_skip)
        lib.cusort_set_wait_limit_ns(prev_limit)
    assert st.value & 1, f"expected the lookback-timeout bit, status={st.value}"
    assert elapsed < 20, f"timed-out sort took {elapsed:.1f}s"
    # the context is still usable and the next sort is correct
    ko, _, info = run_ours("u32", keys)
    ek, _ = O.oracle_sort("u32", keys)
    assert same_bits(ko, ek)
    assert info["status"] == 0
