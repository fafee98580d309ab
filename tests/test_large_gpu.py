"""Above 2^30 items the sort switches to 64-bit offsets and descriptors
(reference: libcusort.cuh:2955-2960).  At that size the CPU oracle is too slow,
so the checks are size-independent properties computed on the GPU: the output
keys are non-decreasing, the output values (original indices) are a
permutation that maps the input keys onto the output keys, and equal keys keep
increasing indices (stability).
"""
from __future__ import annotations

import ctypes as C

import pytest

torch = pytest.importorskip("torch")

from libcusort_b200 import _capi  # noqa: E402

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("no CUDA device", allow_module_level=True)


def _free_gb():
    free, _ = torch.cuda.mem_get_info()
    return free / 2**30


@pytest.mark.skipif(torch.cuda.is_available() and _free_gb() < 40, reason="needs ~30 GB of device memory")
@pytest.mark.parametrize("api", ["raw", "db"])
def test_64bit_offsets_above_2p30(api):
    lib = _capi.load()
    n = (1 << 30) + 12_345
    off = C.c_int(0)
    assert lib.cusort_query_plan(4, 4, n, 0, 32, None, None, None, None, C.byref(off)) == 0 and off.value == 8
    g = torch.Generator(device="cuda")
    g.manual_seed(30)
    # 24-bit keys so equal keys are frequent (stability is exercised)
    keys = torch.randint(0, 1 << 24, (n,), dtype=torch.int32, device="cuda", generator=g)
    vals = torch.arange(n, dtype=torch.int32, device="cuda")  # uint32 bit pattern = index
    kout = torch.empty_like(keys)
    vout = torch.empty_like(vals)
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    P = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    nb = C.c_size_t(0)
    if api == "raw":
        args = lambda t: (t, C.byref(nb), 4, P(keys), P(kout), 4, P(vals), P(vout), n, 0, 32, stream)  # noqa: E731
        assert lib.cusort_sort_pairs(*args(None)) == 0
        temp = torch.empty(nb.value, dtype=torch.uint8, device="cuda")
        assert lib.cusort_sort_pairs(*args(P(temp))) == 0
        ko, vo = kout, vout
        kin = keys
    else:
        kin = keys.clone()
        kdb, vdb = _capi.DoubleBufferC(), _capi.DoubleBufferC()
        kdb.d_buffers[0], kdb.d_buffers[1] = keys.data_ptr(), kout.data_ptr()
        vdb.d_buffers[0], vdb.d_buffers[1] = vals.data_ptr(), vout.data_ptr()
        args = lambda t: (t, C.byref(nb), 4, C.byref(kdb), 4, C.byref(vdb), n, 0, 32, stream)  # noqa: E731
        assert lib.cusort_sort_pairs_db(*args(None)) == 0
        temp = torch.empty(nb.value, dtype=torch.uint8, device="cuda")
        assert lib.cusort_sort_pairs_db(*args(P(temp))) == 0
        assert kdb.selector == 0 and vdb.selector == 0  # 4 passes
        ko, vo = keys, vals
    torch.cuda.synchronize()
    st = C.c_uint32(0)
    assert lib.cusort_read_device_status(P(temp), C.byref(st), stream) == 0 and st.value == 0
    del temp
    chunk = 1 << 27
    for s in range(0, n, chunk):
        e = min(n, s + chunk + 1)
        k = ko[s:e].to(torch.int64)
        v = vo[s:e].to(torch.int64)
        assert bool((k[1:] >= k[:-1]).all()), "keys not sorted"
        same = k[1:] == k[:-1]
        assert bool((v[1:][same] > v[:-1][same]).all()), "equal keys lost their input order"
        assert bool(torch.equal(kin[v], ko[s:e])), "values are not the permutation of the keys"
    # every index appears exactly once
    seen = torch.zeros(n, dtype=torch.bool, device="cuda")
    seen[vo.to(torch.int64)] = True
    assert bool(seen.all())


@pytest.mark.skipif(torch.cuda.is_available() and _free_gb() < 40, reason="needs ~25 GB of device memory")
@pytest.mark.parametrize("kt,np_dtype,bits", [("u16", torch.int16, 16), ("u8", torch.uint8, 8)])
def test_count_fill_paths_above_2p30(kt, np_dtype, bits):
    # 1- and 2-byte keys-only full-range sorts (count and fill, one digit) with 64-bit counts:
    # the output is sorted and holds every key value exactly as often as the input
    lib = _capi.load()
    n = (1 << 30) + 777
    g = torch.Generator(device="cuda")
    g.manual_seed(31)
    keys = torch.randint(0, 1 << bits, (n,), dtype=torch.int32, device="cuda", generator=g).to(np_dtype)
    keys[: n // 5] = 3  # a heavy value
    kout = torch.empty_like(keys)
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    P = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    nb = C.c_size_t(0)
    kid = _capi.KEY_TYPES[kt]
    assert lib.cusort_sort_keys(None, C.byref(nb), kid, P(keys), P(kout), n, 0, bits, stream) == 0
    temp = torch.empty(nb.value, dtype=torch.uint8, device="cuda")
    assert lib.cusort_sort_keys(P(temp), C.byref(nb), kid, P(keys), P(kout), n, 0, bits, stream) == 0
    torch.cuda.synchronize()
    mask = (1 << bits) - 1
    ki = keys.to(torch.int64) & mask  # unsigned key value
    ko = kout.to(torch.int64) & mask
    assert bool((ko[1:] >= ko[:-1]).all()), "keys not sorted"
    assert torch.equal(torch.bincount(ki, minlength=1 << bits), torch.bincount(ko, minlength=1 << bits))
