"""cusort_sort_pairs_host: keys and values in (page-locked) HOST memory, the
copies overlapped with the sort inside the call.  Bit-exact against the CPU
oracle for several key and value widths, both orders, a partial bit range,
and an empty input; the outputs are read only after the stream is synchronised.
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
from tests.gpu_helpers import same_bits  # noqa: E402

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("no CUDA device", allow_module_level=True)

CORES = os.cpu_count() or 1


def _pinned(a: np.ndarray, pin: bool = True):
    t = torch.empty(max(a.nbytes, 1), dtype=torch.uint8, pin_memory=pin)
    if a.nbytes:
        t[: a.nbytes].copy_(torch.from_numpy(np.ascontiguousarray(a).view(np.uint8).reshape(-1)))
    return t


def run_host(kt, keys, vals, begin=0, end=None, desc=False, pin=True):
    lib = _capi.load()
    n = len(keys)
    end = 8 * keys.dtype.itemsize if end is None else end
    vb = vals.dtype.itemsize * int(np.prod(vals.shape[1:], dtype=np.int64))
    kin, vin = _pinned(keys, pin), _pinned(vals, pin)
    kout = torch.empty_like(kin)
    vout = torch.empty_like(vin)
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    P = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    nb = C.c_size_t(0)
    args = lambda t: (t, C.byref(nb), _capi.KEY_TYPES[kt], P(kin), P(kout), vb, P(vin), P(vout), n, begin, end,  # noqa
                      int(desc), stream)
    assert lib.cusort_sort_pairs_host(*args(None)) == 0
    temp = torch.empty(max(nb.value, 1), dtype=torch.uint8, device="cuda")
    assert lib.cusort_sort_pairs_host(*args(P(temp))) == 0
    torch.cuda.current_stream().synchronize()
    ko = kout[: keys.nbytes].numpy().view(keys.dtype).reshape(keys.shape)
    vo = vout[: vals.nbytes].numpy().view(vals.dtype).reshape(vals.shape)
    return ko, vo


@pytest.mark.parametrize("kt,vb", [("i32", 4), ("u32", 1), ("f32", 2), ("u64", 8), ("f64", 16), ("u16", 4),
                                   ("i8", 4)])
@pytest.mark.parametrize("desc", [False, True])
def test_host_pairs_match_oracle(kt, vb, desc):
    n = 3_000_017
    keys = D.special_floats(kt, n, seed=61) if kt.startswith("f") else D.uniform_bits(kt, n, seed=61)
    vals = D.values_for(n, vb)
    ko, vo = run_host(kt, keys, vals, desc=desc)
    ek, ev = O.oracle_sort(kt, keys, vals, 0, None, desc, threads=CORES)
    assert same_bits(ko, ek) and same_bits(vo, ev)


def test_host_pairs_pageable_memory():
    # pageable host buffers work too (the copies then do not overlap)
    n = 500_009
    keys = D.uniform_bits("i32", n, seed=64)
    vals = D.values_for(n, 8)
    ko, vo = run_host("i32", keys, vals, pin=False)
    ek, ev = O.oracle_sort("i32", keys, vals, 0, None, False, threads=CORES)
    assert same_bits(ko, ek) and same_bits(vo, ev)


def test_host_pairs_bit_range_and_empty():
    n = 1_000_003
    keys = D.uniform_bits("u32", n, seed=62)
    vals = D.values_for(n, 4)
    ko, vo = run_host("u32", keys, vals, 5, 21)
    ek, ev = O.oracle_sort("u32", keys, vals, 5, 21, False, threads=CORES)
    assert same_bits(ko, ek) and same_bits(vo, ev)
    e = np.empty(0, dtype=np.uint32)
    ko, vo = run_host("u32", e, e.copy())
    assert ko.size == 0 and vo.size == 0


def test_radix_sort_host_torch_wrapper():
    from libcusort_b200.torch_sort import radix_sort_host
    g = torch.Generator().manual_seed(63)
    n = 2_000_003
    keys = torch.randint(-(2 ** 31), 2 ** 31, (n,), dtype=torch.int64, generator=g).to(torch.int32).pin_memory()
    vals = torch.arange(n, dtype=torch.int32).pin_memory()
    ko, vo = radix_sort_host(keys, vals)
    ref = torch.sort(keys, stable=True)
    assert torch.equal(ko, ref.values) and torch.equal(vo.long(), ref.indices)
    ko, vo = radix_sort_host(keys, vals, descending=True)
    ref = torch.sort(keys, stable=True, descending=True)
    assert torch.equal(ko, ref.values) and torch.equal(vo.long(), ref.indices)
