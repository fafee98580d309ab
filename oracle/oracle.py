"""Python bindings of the test oracle and of the reference library.

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's cpu_baseline / reference legs -- never by the libcusort_b200 product.

* ``oracle_sort``: CPU restatement (cusort_oracle.cpp): std::stable_sort on the
  masked twiddled key; libcusort.cuh semantics cited there.
* ``numpy_sort``: an independent numpy restatement (np.argsort kind="stable"),
  used to cross-check the C++ oracle.
* ``oracle_segmented_sort`` / ``numpy_segmented_sort``: the segmented sort's
  semantics (each segment [begin, end) sorted independently and stably in
  place of the output, everything else untouched), over the C++ oracle per
  segment and over one numpy lexsort by (segment, digit key) respectively.
  The reference has no segmented sort (only the name, libcusort.cuh:4); the
  semantics follow CUB's DeviceSegmentedRadixSort.
* ``ref_sort``: the UNMODIFIED reference, compiled for sm_100a into
  oracle/_ref/libcusort_ref.so by oracle/Makefile (needs a GPU to run).
"""
from __future__ import annotations

import ctypes as C
import json
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "_build" / "libcusort_oracle.so"
REF_SO = HERE / "_ref" / "libcusort_ref.so"

KEY_TYPES = {"u8": 0, "i8": 1, "u16": 2, "i16": 3, "u32": 4, "i32": 5, "u64": 6, "i64": 7, "f32": 8, "f64": 9}
NP_DTYPE = {"u8": np.uint8, "i8": np.int8, "u16": np.uint16, "i16": np.int16, "u32": np.uint32, "i32": np.int32,
            "u64": np.uint64, "i64": np.int64, "f32": np.float32, "f64": np.float64}
NP_UINT = {1: np.uint8, 2: np.uint16, 4: np.uint32, 8: np.uint64}

_oracle = None
_ref = None


def reference_dir() -> Path | None:
    """Checkout of the reference library (the directory holding libcusort.cuh), needed only to
    BUILD oracle/_ref: the environment variable CUSORT_REFERENCE_DIR, else the "reference_path"
    field of BASELINE.json at the repository root.  None when neither names a directory that
    holds libcusort.cuh (the GPU box only uses the prebuilt library)."""
    cand = os.environ.get("CUSORT_REFERENCE_DIR")
    if not cand:
        meta = HERE.parent / "BASELINE.json"
        if meta.exists():
            try:
                cand = json.loads(meta.read_text()).get("reference_path")
            except (ValueError, OSError):
                cand = None
    if cand and (Path(cand) / "libcusort.cuh").exists():
        return Path(cand)
    return None


def build(ref: bool = True) -> None:
    """make the oracle (and, with ref=True and a reference checkout, oracle/_ref)."""
    targets = ["oracle"]
    extra = []
    if ref:
        rd = reference_dir()
        if rd is None:
            raise RuntimeError("building oracle/_ref needs the reference checkout: set CUSORT_REFERENCE_DIR")
        targets.append("ref")
        extra.append(f"REF_DIR={rd}")
    subprocess.run(["make", "-s", "-j8", *targets, *extra], cwd=HERE, check=True)


def _load_oracle():
    global _oracle
    if _oracle is None:
        if not ORACLE_SO.exists():
            build(ref=False)
        lib = C.CDLL(str(ORACLE_SO))
        lib.oracle_sort.restype = C.c_int
        lib.oracle_sort.argtypes = [C.c_int, C.c_void_p, C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p, C.c_int64,
                                    C.c_int, C.c_int, C.c_int, C.c_int]
        lib.oracle_sort_permutation.restype = C.c_int
        lib.oracle_sort_permutation.argtypes = [C.c_int, C.c_void_p, C.c_int64, C.c_int, C.c_int, C.c_int, C.c_int,
                                                C.c_void_p]
        lib.oracle_digit_key.restype = C.c_uint64
        lib.oracle_digit_key.argtypes = [C.c_int, C.c_uint64, C.c_int, C.c_int, C.c_int]
        lib.oracle_digit_histogram.restype = C.c_int
        lib.oracle_digit_histogram.argtypes = [C.c_int, C.c_void_p, C.c_int64, C.c_int, C.c_int, C.c_int,
                                               C.c_void_p]
        _oracle = lib
    return _oracle


def _ptr(a: np.ndarray | None):
    return None if a is None else C.c_void_p(a.ctypes.data)


def oracle_sort(kt: str, keys: np.ndarray, values: np.ndarray | None = None, begin_bit: int = 0,
                end_bit: int | None = None, descending: bool = False, threads: int = 1):
    """Stable sort on the CPU; values may be any contiguous array with len == n (bytes per item 1..16)."""
    lib = _load_oracle()
    keys = np.ascontiguousarray(keys)
    n = keys.shape[0]
    end_bit = 8 * keys.dtype.itemsize if end_bit is None else end_bit
    ko = np.empty_like(keys)
    vo = None
    vb = 0
    if values is not None:
        values = np.ascontiguousarray(values)
        vo = np.empty_like(values)
        vb = values.nbytes // max(n, 1)
    rc = lib.oracle_sort(KEY_TYPES[kt], _ptr(keys), _ptr(ko), vb, _ptr(values), _ptr(vo), n, begin_bit, end_bit,
                         int(descending), threads)
    if rc:
        raise ValueError("oracle_sort rejected the arguments")
    return ko, vo


def oracle_perm(kt: str, keys: np.ndarray, begin_bit: int = 0, end_bit: int | None = None,
                descending: bool = False, threads: int = 1) -> np.ndarray:
    lib = _load_oracle()
    keys = np.ascontiguousarray(keys)
    end_bit = 8 * keys.dtype.itemsize if end_bit is None else end_bit
    perm = np.empty(keys.shape[0], dtype=np.int64)
    rc = lib.oracle_sort_permutation(KEY_TYPES[kt], _ptr(keys), keys.shape[0], begin_bit, end_bit, int(descending),
                                     threads, _ptr(perm))
    if rc:
        raise ValueError("oracle_sort_permutation rejected the arguments")
    return perm


def oracle_digit_key(kt: str, bits: int, begin_bit: int, end_bit: int, descending: bool = False) -> int:
    return int(_load_oracle().oracle_digit_key(KEY_TYPES[kt], bits, int(descending), begin_bit, end_bit))


def oracle_histogram(kt: str, keys: np.ndarray, begin_bit: int, end_bit: int, descending: bool = False):
    lib = _load_oracle()
    keys = np.ascontiguousarray(keys)
    passes = (end_bit - begin_bit + 7) // 8
    out = np.zeros(passes * 256, dtype=np.uint64)
    lib.oracle_digit_histogram(KEY_TYPES[kt], _ptr(keys), keys.shape[0], begin_bit, end_bit, int(descending),
                               _ptr(out))
    return out.reshape(passes, 256)


def numpy_digit_keys(kt: str, keys: np.ndarray, begin_bit: int, end_bit: int, descending: bool) -> np.ndarray:
    """Independent numpy restatement of the twiddle + bit-range extraction."""
    kb = keys.dtype.itemsize
    nb = 8 * kb
    bits = keys.view(NP_UINT[kb]).astype(np.uint64)
    sign = np.uint64(1) << np.uint64(nb - 1)
    allm = np.uint64((1 << nb) - 1) if nb < 64 else np.uint64(0xFFFFFFFFFFFFFFFF)
    if kt in ("f32", "f64"):
        neg = (bits & sign) != 0
        t = np.where(neg, (~bits) & allm, bits | sign)
    elif kt.startswith("i"):
        t = bits ^ sign
    else:
        t = bits
    if descending:
        t = (~t) & allm
    w = end_bit - begin_bit
    t = t >> np.uint64(begin_bit)
    if w < 64:
        t = t & np.uint64((1 << w) - 1)
    return t


def numpy_sort(kt: str, keys: np.ndarray, values=None, begin_bit=0, end_bit=None, descending=False):
    end_bit = 8 * keys.dtype.itemsize if end_bit is None else end_bit
    dk = numpy_digit_keys(kt, keys, begin_bit, end_bit, descending)
    perm = np.argsort(dk, kind="stable")
    return keys[perm], (None if values is None else values[perm])


def oracle_segmented_sort(kt: str, keys: np.ndarray, values, begins, ends, begin_bit: int = 0,
                          end_bit: int | None = None, descending: bool = False, keys_out=None, values_out=None):
    """Segmented stable sort: out[b:e] = oracle_sort(keys[b:e]) per segment; other positions keep
    keys_out / values_out (copied) as given."""
    ko = np.array(keys_out if keys_out is not None else np.zeros_like(keys), copy=True)
    vo = None
    if values is not None:
        vo = np.array(values_out if values_out is not None else np.zeros_like(values), copy=True)
    for b, e in zip(np.asarray(begins).tolist(), np.asarray(ends).tolist()):
        if e <= b:
            continue
        k, v = oracle_sort(kt, keys[b:e], None if values is None else values[b:e], begin_bit, end_bit, descending)
        ko[b:e] = k
        if values is not None:
            vo[b:e] = v
    return ko, vo


def numpy_segmented_sort(kt: str, keys: np.ndarray, values, begins, ends, begin_bit: int = 0,
                         end_bit: int | None = None, descending: bool = False, keys_out=None, values_out=None):
    """Independent restatement: one stable lexsort of the in-segment items by (segment, digit key)."""
    end_bit = 8 * keys.dtype.itemsize if end_bit is None else end_bit
    ko = np.array(keys_out if keys_out is not None else np.zeros_like(keys), copy=True)
    vo = None if values is None else np.array(values_out if values_out is not None else np.zeros_like(values),
                                                copy=True)
    begins = np.asarray(begins, dtype=np.int64)
    ends = np.asarray(ends, dtype=np.int64)
    lens = np.maximum(ends - begins, 0)
    if lens.sum() == 0:
        return ko, vo
    seg = np.repeat(np.arange(len(begins)), lens)
    pos = np.concatenate([np.arange(b, b + m) for b, m in zip(begins.tolist(), lens.tolist()) if m > 0])
    dk = numpy_digit_keys(kt, keys[pos], begin_bit, end_bit, descending)
    order = np.lexsort((dk, seg))  # stable: ties keep the in-segment input order
    ko[pos] = keys[pos[order]]
    if values is not None:
        vo[pos] = values[pos[order]]
    return ko, vo


# ---------------------------------------------------------------------------
# reference library (GPU)
# ---------------------------------------------------------------------------
def ref_available() -> bool:
    return REF_SO.exists()


def _load_ref():
    global _ref
    if _ref is None:
        if not REF_SO.exists():
            raise RuntimeError(f"{REF_SO} not built (oracle/Makefile target `ref`, needs the reference checkout)")
        lib = C.CDLL(str(REF_SO))
        for k in range(10):
            fn = getattr(lib, f"ref_sort_k{k}")
            fn.restype = C.c_int
            fn.argtypes = [C.c_int, C.c_int, C.c_int, C.c_void_p, C.POINTER(C.c_size_t), C.c_void_p, C.c_void_p,
                           C.POINTER(C.c_int), C.c_void_p, C.c_void_p, C.POINTER(C.c_int), C.c_int64, C.c_int,
                           C.c_int, C.c_void_p]
        _ref = lib
    return _ref


def ref_call(kt: str, value_bytes: int, descending: bool, raw: bool, temp_ptr, temp_bytes: int, k0, k1, ksel: int,
             v0, v1, vsel: int, n: int, begin_bit: int, end_bit: int, stream=None):
    """One call of the reference's DeviceRadixSort; returns (rc, temp_bytes, ksel, vsel)."""
    lib = _load_ref()
    fn = getattr(lib, f"ref_sort_k{KEY_TYPES[kt]}")
    tb = C.c_size_t(temp_bytes)
    ks = C.c_int(ksel)
    vs = C.c_int(vsel)
    rc = fn(value_bytes, int(descending), int(raw), temp_ptr, C.byref(tb), k0, k1, C.byref(ks), v0, v1, C.byref(vs),
            n, begin_bit, end_bit, stream)
    return rc, tb.value, ks.value, vs.value
