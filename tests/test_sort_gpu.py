"""GPU parity tests: libcusort_b200 (through its C ABI) against the CPU oracle,
bit-exact, over key types, value widths, directions, bit ranges, sizes around
tile boundaries, special floats, skewed inputs, unaligned pointers and both
API forms; and against the reference library itself when oracle/_ref is built.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from libcusort_b200 import _capi  # noqa: E402
from oracle import oracle as O  # noqa: E402
from tests import datagen as D  # noqa: E402
from tests.gpu_helpers import run_ours, run_ref, same_bits  # noqa: E402

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("no CUDA device", allow_module_level=True)


def tile_of(kt: str, vb: int, n: int = 1 << 20) -> int:
    lib = _capi.load()
    tile = C.c_int(0)
    rc = lib.cusort_query_plan(_capi.KEY_TYPES[kt], vb, n, 0, 8 * _capi.KEY_BYTES[kt], None, C.byref(tile), None,
                               None, None)
    assert rc == 0
    return tile.value


def check(kt, keys, values=None, begin=0, end=None, desc=False, api="raw", **kw):
    ko, vo, info = run_ours(kt, keys, values, begin, end, desc, api=api, **kw)
    ek, ev = O.oracle_sort(kt, keys, values, begin, end, desc)
    assert same_bits(ko, ek), f"keys differ ({kt}, n={len(keys)}, bits=[{begin},{end}), desc={desc}, api={api})"
    if values is not None:
        assert same_bits(vo, ev), f"values differ ({kt}, n={len(keys)})"
    return info


# --- every key type, both directions, keys-only and pairs --------------------
@pytest.mark.parametrize("kt", D.KEY_TYPES)
@pytest.mark.parametrize("desc", [False, True])
@pytest.mark.parametrize("vb", [0, 4])
def test_key_types(kt, desc, vb):
    n = 3 * tile_of(kt, vb) + 17
    keys = D.uniform_bits(kt, n, seed=11 + D.KEY_TYPES.index(kt))
    vals = D.values_for(n, vb) if vb else None
    check(kt, keys, vals, desc=desc)


# --- every value width ------------------------------------------------------
@pytest.mark.parametrize("kt", ["u8", "i16", "f32", "i64", "f64"])
@pytest.mark.parametrize("vb", [1, 2, 8, 16])
def test_value_widths(kt, vb):
    n = 2 * tile_of(kt, vb) + 1001
    keys = D.uniform_bits(kt, n, seed=3)
    check(kt, keys, D.values_for(n, vb), desc=(vb == 8))


# --- partial bit ranges -----------------------------------------------------
@pytest.mark.parametrize("kt,begin,end", [
    ("u32", 0, 20), ("u32", 3, 29), ("i32", 5, 6), ("f32", 8, 16), ("f32", 0, 31), ("f32", 20, 32),
    ("i64", 0, 64), ("i64", 17, 61), ("f64", 40, 64), ("u16", 4, 12), ("i8", 1, 8), ("u64", 63, 64),
])
@pytest.mark.parametrize("desc", [False, True])
def test_bit_ranges(kt, begin, end, desc):
    n = 50_000
    keys = D.uniform_bits(kt, n, seed=begin * 100 + end)
    check(kt, keys, D.values_for(n, 4), begin, end, desc)


def test_zero_width_range_is_copy():
    keys = D.uniform_bits("u32", 1000, seed=1)
    vals = D.values_for(1000, 4)
    ko, vo, _ = run_ours("u32", keys, vals, 7, 7)
    assert same_bits(ko, keys) and same_bits(vo, vals)


# --- sizes around tile boundaries -------------------------------------------
@pytest.mark.parametrize("vb", [0, 4])
def test_sizes(vb):
    t = tile_of("u32", vb)
    for n in [0, 1, 2, 31, 32, 33, 255, 256, 257, t - 1, t, t + 1, 2 * t, 3 * t + 17, 1 << 20]:
        keys = D.uniform_bits("u32", n, seed=n)
        vals = D.values_for(n, vb) if vb else None
        check("u32", keys, vals)


# --- the three tile sizes of 4-byte keys (8 / 16 / large items per thread by item count) --
@pytest.mark.parametrize("tier_n", [1 << 20, 1 << 23, 1 << 26])
@pytest.mark.parametrize("kt,vb,desc", [("u32", 0, False), ("i32", 4, False), ("f32", 4, True)])
def test_tile_tiers(tier_n, kt, vb, desc):
    # sizes at a multiple of the tier's tile -1 / 0 / +1, as close to the tier's upper end as
    # the tier allows (the large tile just above 2^23, where it takes over)
    t = tile_of(kt, vb, tier_n)
    if tier_n > (1 << 23):
        m = (1 << 23) // t + 1
        sizes = [m * t - 1, m * t, m * t + 1]
    else:
        m = tier_n // t
        sizes = [m * t - 1, m * t, (m - 1) * t + 1]
    for n in sizes:
        assert tile_of(kt, vb, n) == t
        keys = D.uniform_bits(kt, n, seed=n % 1000)
        check(kt, keys, D.values_for(n, vb) if vb else None, desc=desc)


# --- distributions ------------------------------------------------------------
@pytest.mark.parametrize("kt", ["f32", "f64"])
@pytest.mark.parametrize("desc", [False, True])
def test_special_floats(kt, desc):
    n = 100_000
    keys = D.special_floats(kt, n, seed=5, frac=0.01)
    # a few NaN payloads and negative NaNs, denormals
    u = keys.view(O.NP_UINT[keys.dtype.itemsize])
    if kt == "f32":
        u[:4] = [0x7FC00001, 0xFFC00000, 0x00000001, 0x80000001]
    else:
        u[:4] = [0x7FF8000000000001, 0xFFF8000000000000, 1, 0x8000000000000001]
    check(kt, keys, D.values_for(n, 4), desc=desc)


@pytest.mark.parametrize("kind", ["low_entropy", "all_equal", "sorted", "reversed", "zipf", "zipf_lowbits"])
def test_distributions(kind):
    n = 300_000
    if kind == "low_entropy":
        keys = D.low_entropy("i32", n, seed=3)
    elif kind == "all_equal":
        keys = np.full(n, 12345, dtype=np.int32)
    elif kind == "sorted":
        keys = np.sort(D.uniform_bits("i32", n, seed=4))
    elif kind == "reversed":
        keys = np.sort(D.uniform_bits("i32", n, seed=4))[::-1].copy()
    elif kind == "zipf":
        keys = D.zipf_table("i32", n, seed=6)
    else:
        keys = D.zipf_table("i32", n, seed=6, below=16)
    check("i32", keys, D.values_for(n, 4))
    check("i32", keys, D.values_for(n, 4), begin=0, end=20)


# --- API forms ----------------------------------------------------------------
@pytest.mark.parametrize("begin,end", [(0, 32), (0, 24), (0, 8), (4, 11)])
@pytest.mark.parametrize("ksel0,vsel0", [(0, 0), (1, 0), (0, 1)])
def test_double_buffer_selectors(begin, end, ksel0, vsel0):
    n = 40_000
    keys = D.uniform_bits("u32", n, seed=9)
    vals = D.values_for(n, 8)
    info = check("u32", keys, vals, begin, end, api="db", ksel0=ksel0, vsel0=vsel0)
    passes = (end - begin + 7) // 8
    assert info["ksel"] == ksel0 ^ (passes & 1)
    assert info["vsel"] == vsel0 ^ (passes & 1)


@pytest.mark.parametrize("kt", ["u8", "u16", "u32", "f64"])
@pytest.mark.parametrize("offset", [1, 3])
def test_unaligned_pointers(kt, offset):
    n = 70_001
    keys = D.uniform_bits(kt, n, seed=offset)
    check(kt, keys, D.values_for(n, 2), offset_items=offset)
    check(kt, keys, D.values_for(n, 2), offset_items=offset, api="db")


@pytest.mark.parametrize("kt,vb", [("f32", 4), ("u16", 0), ("u8", 0), ("i16", 2)])
def test_graph_mode_matches_direct(kt, vb):
    # graph replay of every launch sequence: onesweep passes, 16-bit count + fill, 8-bit count + fill
    n = 1 << 18
    for seed in range(3):
        keys = D.uniform_bits(kt, n, seed=seed)
        vals = D.values_for(n, vb) if vb else None
        a = run_ours(kt, keys, vals, launch_mode=1)
        b = run_ours(kt, keys, vals, launch_mode=0)
        assert same_bits(a[0], b[0]) and (vals is None or same_bits(a[1], b[1]))
        ek, ev = O.oracle_sort(kt, keys, vals)
        assert same_bits(a[0], ek) and (vals is None or same_bits(a[1], ev))


def test_torch_radix_sort():
    from libcusort_b200.torch_sort import argsort, radix_sort
    x = torch.randn(100_003, device="cuda")
    k, _ = radix_sort(x)
    assert torch.equal(k, torch.sort(x, stable=True).values)
    perm = argsort(x, descending=True)
    assert torch.equal(perm, torch.sort(x, descending=True, stable=True).indices)


# --- the reference library itself -------------------------------------------
needs_ref = pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref/libcusort_ref.so not built")


@needs_ref
@pytest.mark.parametrize("kt", D.KEY_TYPES)
@pytest.mark.parametrize("vb", [0, 4, 16])
def test_reference_parity(kt, vb):
    n = 200_000
    keys = D.special_floats(kt, n, seed=21) if kt.startswith("f") else D.uniform_bits(kt, n, seed=21)
    vals = D.values_for(n, vb) if vb else None
    for desc in (False, True):
        for api in ("raw", "db"):
            rk, rv, rinfo = run_ref(kt, keys, vals, descending=desc, api=api)
            ok, ov, oinfo = run_ours(kt, keys, vals, descending=desc, api=api)
            assert same_bits(rk, ok), f"keys differ from the reference ({kt}, vb={vb}, desc={desc}, {api})"
            if vb:
                assert same_bits(rv, ov)
            if api == "db":
                assert rinfo["ksel"] == oinfo["ksel"] and rinfo["vsel"] == oinfo["vsel"]


@needs_ref
@pytest.mark.parametrize("kt,begin,end", [("u32", 0, 20), ("f32", 3, 29), ("f64", 11, 50), ("i16", 2, 9)])
def test_reference_parity_bit_ranges(kt, begin, end):
    n = 123_457
    keys = D.uniform_bits(kt, n, seed=begin + end)
    vals = D.values_for(n, 4)
    rk, rv, _ = run_ref(kt, keys, vals, begin, end, True)
    ok, ov, _ = run_ours(kt, keys, vals, begin, end, True)
    assert same_bits(rk, ok) and same_bits(rv, ov)


# --- payloads wider than 16 bytes (index sort + gather) -------------------------
@pytest.mark.parametrize("vb", [3, 24, 32, 100])
@pytest.mark.parametrize("desc", [False, True])
def test_wide_payloads(vb, desc):
    from tests.gpu_helpers import DevBuf
    lib = _capi.load()
    n = 123_457
    keys = D.uniform_bits("f32", n, seed=vb)
    vals = np.random.default_rng(vb).integers(0, 256, size=(n, vb), dtype=np.uint8)
    kin, kout = DevBuf.from_array(keys), DevBuf(keys.nbytes)
    vin, vout = DevBuf.from_array(vals), DevBuf(vals.nbytes)
    nb = C.c_size_t(0)
    args = (8, kin.ptr, kout.ptr, vb, vin.ptr, vout.ptr, n, 0, 32, int(desc), None)
    assert lib.cusort_sort_pairs_wide(None, C.byref(nb), *args) == 0
    temp = DevBuf(nb.value)
    assert lib.cusort_sort_pairs_wide(temp.ptr, C.byref(nb), *args) == 0
    torch.cuda.synchronize()
    ek, ev = O.oracle_sort("f32", keys, vals, 0, 32, desc)
    assert same_bits(kout.to_array(keys), ek) and same_bits(vout.to_array(vals), ev)
    assert all(b.guards_ok() for b in (kin, kout, vin, vout, temp))


# --- 1-byte keys-only over all 8 bits: count-and-fill path ---------------------
@pytest.mark.parametrize("kt", ["u8", "i8"])
@pytest.mark.parametrize("desc", [False, True])
@pytest.mark.parametrize("n", [1, 17, 4095, 1_000_003])
def test_byte_keys_count_fill(kt, desc, n):
    keys = D.uniform_bits(kt, n, seed=n)
    if n > 100:
        keys[: n // 3] = keys[0]  # one heavy value
    check(kt, keys, None, desc=desc)
    check(kt, keys, None, desc=desc, api="db")
    check(kt, keys, None, desc=desc, offset_items=3)


# --- 2-byte keys-only over all 16 bits: one 16-bit digit (count, scan, fill) -----
@pytest.mark.parametrize("kt", ["u16", "i16"])
@pytest.mark.parametrize("desc", [False, True])
@pytest.mark.parametrize("n", [2, 9, 1000, 65_537, 1_000_003, (1 << 22) + 5])
def test_short_keys_one_pass(kt, desc, n):
    keys = D.uniform_bits(kt, n, seed=n + 1)
    if n > 100:
        keys[: n // 4] = keys[1]  # one heavy value
        keys[n // 4: n // 3] = keys[2]
    check(kt, keys, None, desc=desc)
    check(kt, keys, None, desc=desc, api="db")
    check(kt, keys, None, desc=desc, offset_items=3)


def test_short_keys_one_pass_few_values():
    n = 777_777
    keys = np.random.default_rng(1).choice(np.array([0, 1, 65535, 32768, 32767], dtype=np.uint16), size=n)
    check("u16", keys, None)
    check("i16", keys.view(np.int16), None, desc=True)


@pytest.mark.parametrize("kt", ["u16", "i16"])
def test_short_keys_one_pass_counter_overflow(kt):
    # the 16-bit-digit count keeps two bins per 32-bit shared word (16-bit halves) and moves
    # 0x8000 to the global count whenever a half reaches it: with 2^24 keys each of the ~148
    # counting CTAs sees tens of thousands of copies of the heavy values, whose bins (0x1234,
    # 0x1235) share one word, so both halves cross 0x8000 in every CTA without carrying into
    # each other
    n = (1 << 24) + 5
    keys = D.uniform_bits(kt, n, seed=77)
    heavy = np.array([0x1234, 0x1235], dtype=np.uint16).view(keys.dtype)
    keys[: n * 2 // 5] = heavy[0]
    keys[n * 2 // 5: n * 3 // 4] = heavy[1]
    np.random.default_rng(78).shuffle(keys)
    check(kt, keys, None)
    check(kt, keys, None, desc=True)
    same = np.full((1 << 23) + 1, heavy[0], dtype=keys.dtype)  # every key equal
    check(kt, same, None)


@pytest.mark.parametrize("kt,vb", [("u32", 0), ("i32", 4), ("f32", 0), ("u64", 8), ("f64", 0), ("u16", 2), ("u8", 4),
                                   ("i64", 16)])
@pytest.mark.parametrize("desc", [False, True])
def test_one_digit_tiles(kt, vb, desc):
    # runs of 2^15 equal keys: whole tiles whose keys share their digit in every pass skip the
    # ranking and go out in input order; the tiles that straddle two runs are ranked as usual
    n = (1 << 21) + 12_345
    table = D.uniform_bits(kt, (n >> 15) + 1, seed=91)
    keys = table[np.arange(n) >> 15]
    vals = D.values_for(n, vb) if vb else None
    check(kt, keys, vals, desc=desc)
    if vb:
        check(kt, keys, vals, desc=desc, api="db")


@pytest.mark.parametrize("kt,vb", [("u32", 0), ("i32", 4), ("u16", 2), ("u16", 1), ("u64", 8), ("u8", 4), ("f32", 0)])
@pytest.mark.parametrize("shift", [4, 10])
def test_sorted_tiles(kt, vb, shift):
    # ascending keys with runs of 2^shift equal values: whole tiles whose digits never decrease are
    # written out unranked; one pair of neighbours swapped per 2^16 keys makes some tiles fail the
    # check (they are ranked as usual)
    n = (1 << 21) + 4321
    bits = 8 * np.dtype(O.NP_UINT[{"u32": 4, "i32": 4, "u16": 2, "u64": 8, "u8": 1, "f32": 4}[kt]]).itemsize
    raw = (np.arange(n, dtype=np.uint64) >> shift) & np.uint64((1 << min(bits, 63)) - 1)
    if kt == "f32":
        keys = raw.astype(np.float32)
    else:
        keys = raw.astype(O.NP_UINT[bits // 8]).view({"u32": np.uint32, "i32": np.int32, "u16": np.uint16,
                                                       "u64": np.uint64, "u8": np.uint8}[kt])
    keys = keys.copy()
    swap = np.arange(1000, n - 1, 1 << 16)
    keys[swap], keys[swap + 1] = keys[swap + 1].copy(), keys[swap].copy()
    vals = D.values_for(n, vb) if vb else None
    check(kt, keys, vals)
    check(kt, keys, vals, desc=True)


@pytest.mark.parametrize("kt,vb", [("f64", 16), ("u64", 16), ("i64", 16), ("u32", 16), ("u64", 8)])
@pytest.mark.parametrize("desc", [False, True])
def test_index_path_for_wide_values(kt, vb, desc):
    # from 2^20 items the in/out form sorts 8-byte keys with 16-byte values over 6+ digit passes as
    # keys + 32-bit input positions, then gathers the values: the same stable result (the other
    # shapes and the narrow bit range below take the direct path)
    n = (1 << 20) + 4099
    keys = D.special_floats(kt, n, seed=71) if kt.startswith("f") else D.uniform_bits(kt, n, seed=71)
    keys[: n // 3] = keys[5]  # a run of equal keys keeps its input order
    vals = D.values_for(n, vb)
    check(kt, keys, vals, desc=desc)
    bits = 8 * keys.dtype.itemsize
    check(kt, keys, vals, 2, bits - 3, desc=desc)
    check(kt, keys, vals, 0, 24, desc=desc)
