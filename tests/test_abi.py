"""CPU tests of the C ABI (no GPU): the library loads, exports every symbol
include/cusort_b200.h declares, and answers size queries and argument checks
without making any CUDA call (reference behaviour: libcusort.cuh:2908-2931,
2609-2613)."""
from __future__ import annotations

import ctypes as C
import re
from pathlib import Path

import pytest

from libcusort_b200 import _capi

ROOT = Path(__file__).resolve().parents[1]
INVALID = _capi.CUDA_ERROR_INVALID_VALUE


def declared_symbols():
    text = (ROOT / "include" / "cusort_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(cusort_[a-z0-9_]+)\s*\(", text)))


def test_every_declared_symbol_is_exported():
    lib = _capi.load()
    syms = declared_symbols()
    assert len(syms) >= 16
    for s in syms:
        assert hasattr(lib, s), s
    assert set(syms) == set(_capi.SIGNATURES), "python bindings out of sync with the header"


def test_version():
    assert _capi.load().cusort_version().decode().startswith("1.0.1")


def _query_keys(kt, n, b, e, raw=True):
    lib = _capi.load()
    nb = C.c_size_t(12345)
    if raw:
        rc = lib.cusort_sort_keys(None, C.byref(nb), kt, None, None, n, b, e, None)
    else:
        db = _capi.DoubleBufferC()
        rc = lib.cusort_sort_keys_db(None, C.byref(nb), kt, C.byref(db), n, b, e, None)
    return rc, nb.value


def _query_pairs(kt, vb, n, b, e, raw=True):
    lib = _capi.load()
    nb = C.c_size_t(12345)
    if raw:
        rc = lib.cusort_sort_pairs(None, C.byref(nb), kt, None, None, vb, None, None, n, b, e, None)
    else:
        db, vdb = _capi.DoubleBufferC(), _capi.DoubleBufferC()
        rc = lib.cusort_sort_pairs_db(None, C.byref(nb), kt, C.byref(db), vb, C.byref(vdb), n, b, e, None)
    return rc, nb.value


@pytest.mark.parametrize("b,e", [(-1, 8), (0, -1), (9, 8), (0, 33)])
def test_invalid_bit_range(b, e):
    assert _query_keys(4, 1000, b, e)[0] == INVALID


def test_invalid_types():
    assert _query_keys(10, 1000, 0, 8)[0] == INVALID
    assert _query_pairs(4, 3, 1000, 0, 32)[0] == INVALID
    assert _query_pairs(4, 32, 1000, 0, 32)[0] == INVALID
    lib = _capi.load()
    assert lib.cusort_sort_keys(None, None, 4, None, None, 1000, 0, 32, None) == INVALID


def test_misaligned_temp_is_rejected():
    # checked on the host before any CUDA call: a temp pointer that is not 16-byte aligned
    lib = _capi.load()
    rc, need = _query_keys(4, 100_000, 0, 32)
    assert rc == 0
    nb = C.c_size_t(need)
    assert lib.cusort_sort_keys(C.c_void_p(0x10008), C.byref(nb), 4, C.c_void_p(0x20000), C.c_void_p(0x30000),
                                100_000, 0, 32, None) == INVALID
    nb = C.c_size_t(need - 1)  # too small, aligned
    assert lib.cusort_sort_keys(C.c_void_p(0x10000), C.byref(nb), 4, C.c_void_p(0x20000), C.c_void_p(0x30000),
                                100_000, 0, 32, None) == INVALID


def test_trivial_sizes():
    # in/out form reports 1 byte when a copy is still needed, DoubleBuffer 0
    assert _query_keys(4, 0, 0, 32) == (0, 0)
    assert _query_keys(4, 1, 0, 32) == (0, 1)
    assert _query_keys(4, 1, 0, 32, raw=False) == (0, 0)
    assert _query_keys(4, 1000, 5, 5) == (0, 1)
    assert _query_keys(4, 1000, 5, 5, raw=False) == (0, 0)
    assert _query_keys(4, -7, 0, 32) == (0, 0)


def test_temp_size_layout():
    n = 1 << 26
    rc, db_bytes = _query_keys(4, n, 0, 32, raw=False)
    assert rc == 0
    rc, raw_bytes = _query_keys(4, n, 0, 32, raw=True)
    assert rc == 0
    # in/out form with >= 2 passes adds one staging copy of the keys
    assert raw_bytes - db_bytes == n * 4
    # a single pass needs no staging
    assert _query_keys(4, n, 0, 8)[1] == _query_keys(4, n, 0, 8, raw=False)[1]
    rc, pairs = _query_pairs(4, 4, n, 0, 32)
    assert rc == 0 and pairs - db_bytes >= 2 * n * 4
    # descriptors: 256 x 4 bytes per tile; histogram 256 x 4 per pass; well under the data size
    assert db_bytes < n * 4 // 16


def test_offset_width_switch():
    lib = _capi.load()
    off = C.c_int(0)
    assert lib.cusort_query_plan(4, 0, (1 << 30) - 1, 0, 32, None, None, None, None, C.byref(off)) == 0
    assert off.value == 4
    assert lib.cusort_query_plan(4, 0, 1 << 30, 0, 32, None, None, None, None, C.byref(off)) == 0
    assert off.value == 8
    p = C.c_int(0)
    assert lib.cusort_query_plan(4, 0, 1 << 20, 3, 29, C.byref(p), None, None, None, None) == 0
    assert p.value == 4


def test_wide_offsets_hook(monkeypatch):
    # CUSORT_WIDE_OFFSETS=1 (a test hook) selects the 64-bit offset kernels of 2^30+ items at any
    # size, without the small-sort tile tiers (those kernels exist with 32-bit offsets only)
    lib = _capi.load()
    off, tile = C.c_int(0), C.c_int(0)
    monkeypatch.setenv("CUSORT_WIDE_OFFSETS", "1")
    assert lib.cusort_query_plan(4, 4, 1000, 0, 32, None, C.byref(tile), None, None, C.byref(off)) == 0
    assert off.value == 8
    # uint32 + uint32 with 64-bit offsets: 19 items per thread, the largest tile at which the 32-bit
    # warp counters still fit two CTAs' share of shared memory
    assert tile.value == 512 * 19
    assert _tile_items(4, 0, 1000) == 512 * 36
    monkeypatch.delenv("CUSORT_WIDE_OFFSETS")
    assert lib.cusort_query_plan(4, 4, 1000, 0, 32, None, C.byref(tile), None, None, C.byref(off)) == 0
    assert off.value == 4 and tile.value == 512 * 8


def _tile_items(kt, vb, n):
    lib = _capi.load()
    t = C.c_int(0)
    assert lib.cusort_query_plan(kt, vb, n, 0, 8 * _capi.KEY_BYTES[[k for k, v in _capi.KEY_TYPES.items()
                                                                    if v == kt][0]],
                                 None, C.byref(t), None, None, None) == 0
    return t.value


@pytest.mark.parametrize("kt", [4, 5, 8])  # u32, i32, f32
@pytest.mark.parametrize("vb,big", [(0, 512 * 32), (4, 512 * 16)])
def test_tile_tiers(kt, vb, big):
    # 4-byte keys, keys-only or 4-byte values: 8 items per thread up to 2^20 items, 16 up to
    # 2^23, the large tile above (so a small sort's grid still covers the SMs)
    assert _tile_items(kt, vb, 2) == 512 * 8
    assert _tile_items(kt, vb, 1 << 20) == 512 * 8
    assert _tile_items(kt, vb, (1 << 20) + 1) == 512 * 16
    assert _tile_items(kt, vb, 1 << 23) == 512 * 16
    assert _tile_items(kt, vb, (1 << 23) + 1) == big
    assert _tile_items(kt, vb, 1 << 26) == big


def test_tile_tiers_other_widths_unchanged():
    for kt, vb in ((4, 8), (4, 2), (6, 0), (2, 4)):
        assert _tile_items(kt, vb, 1 << 16) == _tile_items(kt, vb, 1 << 26)


def test_settings_roundtrip():
    lib = _capi.load()
    assert lib.cusort_set_launch_mode(1) == 0
    assert lib.cusort_set_launch_mode(0) == 1
    assert lib.cusort_set_launch_mode(7) == 0  # unknown mode ignored
    prev = lib.cusort_set_wait_limit_ns(123)
    assert lib.cusort_set_wait_limit_ns(prev) == 123
    assert lib.cusort_debug_set_skip_tile(5) == -1
    assert lib.cusort_debug_set_skip_tile(-1) == 5


def test_short_keys_one_digit_temp():
    # 2-byte keys-only over all 16 bits use one 16-bit digit: counts[65536] + group totals[256]
    # after the 256-byte control block, no descriptors and no staging (either API form)
    n = 1 << 26
    for kt in (2, 3):  # u16, i16
        for raw in (True, False):
            rc, nb = _query_keys(kt, n, 0, 16, raw=raw)
            assert rc == 0 and nb == 256 + (65536 + 256) * 4
    # a partial range sorts by 8-bit onesweep passes again (in/out form: staging)
    rc, nb = _query_keys(2, n, 0, 15, raw=True)
    assert rc == 0 and nb > n * 2
    # with values, too
    rc, nb = _query_pairs(2, 2, n, 0, 16)
    assert rc == 0 and nb > n * 4


def test_host_pairs_rejects_bad_arguments():
    # cusort_sort_pairs_host: value widths other than 1/2/4/8/16 and 2^32 items or more are refused
    lib = _capi.load()
    nb = C.c_size_t(0)
    assert lib.cusort_sort_pairs_host(None, C.byref(nb), 4, None, None, 3, None, None, 10, 0, 32, 0, None) != 0
    assert lib.cusort_sort_pairs_host(None, C.byref(nb), 4, None, None, 4, None, None, 1 << 32, 0, 32, 0, None) != 0
    assert lib.cusort_sort_pairs_host(None, C.byref(nb), 4, None, None, 4, None, None, 1000, 0, 32, 0, None) == 0
    assert nb.value > 1000 * (4 + 4) * 2
