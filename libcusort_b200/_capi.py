"""ctypes bindings of the C ABI declared in include/cusort_b200.h.

The shared library is built in-tree (libcusort_b200/_lib/libcusort_b200.so).
Loading fails loudly when it is missing: there is no fallback path.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libcusort_b200.so"

# cusort_key_type (include/cusort_b200.h)
KEY_TYPES = {
    "u8": 0, "i8": 1, "u16": 2, "i16": 3, "u32": 4,
    "i32": 5, "u64": 6, "i64": 7, "f32": 8, "f64": 9,
}
KEY_BYTES = {"u8": 1, "i8": 1, "u16": 2, "i16": 2, "u32": 4, "i32": 4, "u64": 8, "i64": 8, "f32": 4, "f64": 8}

CUDA_SUCCESS = 0
CUDA_ERROR_INVALID_VALUE = 1
CUDA_ERROR_TIMEOUT = 909  # cudaErrorTimeout

# Every sort/utility symbol the header declares, with (restype, argtypes).
_vp, _sz, _i64, _i, _u32, _u64 = C.c_void_p, C.c_size_t, C.c_int64, C.c_int, C.c_uint32, C.c_uint64


class DoubleBufferC(C.Structure):
    """Layout of cusort_double_buffer / cusort::DoubleBuffer<T>."""
    _fields_ = [("d_buffers", C.c_void_p * 2), ("selector", C.c_int)]


_P_SZ = C.POINTER(C.c_size_t)
_P_DB = C.POINTER(DoubleBufferC)

SIGNATURES = {
    "cusort_sort_keys_db": (_i, [_vp, _P_SZ, _i, _P_DB, _i64, _i, _i, _vp]),
    "cusort_sort_keys_descending_db": (_i, [_vp, _P_SZ, _i, _P_DB, _i64, _i, _i, _vp]),
    "cusort_sort_pairs_db": (_i, [_vp, _P_SZ, _i, _P_DB, _sz, _P_DB, _i64, _i, _i, _vp]),
    "cusort_sort_pairs_descending_db": (_i, [_vp, _P_SZ, _i, _P_DB, _sz, _P_DB, _i64, _i, _i, _vp]),
    "cusort_sort_keys": (_i, [_vp, _P_SZ, _i, _vp, _vp, _i64, _i, _i, _vp]),
    "cusort_sort_keys_descending": (_i, [_vp, _P_SZ, _i, _vp, _vp, _i64, _i, _i, _vp]),
    "cusort_sort_pairs": (_i, [_vp, _P_SZ, _i, _vp, _vp, _sz, _vp, _vp, _i64, _i, _i, _vp]),
    "cusort_sort_pairs_descending": (_i, [_vp, _P_SZ, _i, _vp, _vp, _sz, _vp, _vp, _i64, _i, _i, _vp]),
    "cusort_sort_pairs_wide": (_i, [_vp, _P_SZ, _i, _vp, _vp, _sz, _vp, _vp, _i64, _i, _i, _i, _vp]),
    "cusort_sort_pairs_host": (_i, [_vp, _P_SZ, _i, _vp, _vp, _sz, _vp, _vp, _i64, _i, _i, _i, _vp]),
    "cusort_segmented_sort_keys": (_i, [_vp, _P_SZ, _i, _vp, _vp, _i64, _i64, _vp, _vp, _i, _i, _i, _vp]),
    "cusort_segmented_sort_pairs": (_i, [_vp, _P_SZ, _i, _vp, _vp, _sz, _vp, _vp, _i64, _i64, _vp, _vp, _i, _i, _i,
                                         _vp]),
    "cusort_sort_db_noalloc": (_i, [_i, _P_DB, _sz, _P_DB, _i64, _i, _i, _i, _vp]),
    "cusort_mgpu_unique_id": (_i, [C.c_char_p]),
    "cusort_mgpu_comm_init": (_i, [C.POINTER(C.c_void_p), C.c_char_p, _i, _i]),
    "cusort_mgpu_comm_destroy": (_i, [_vp]),
    "cusort_mgpu_plan": (_i, [C.POINTER(C.c_uint64), _i, _i, C.POINTER(_i), C.POINTER(_i64), C.POINTER(_i64),
                              C.POINTER(_i64)]),
    "cusort_mgpu_sort": (_i, [_vp, _vp, _P_SZ, _i, _sz, _vp, _vp, _i64, _vp, _vp, _i64, C.POINTER(_i64), _i, _i,
                              _i, _vp]),
    "cusort_mgpu_set_timeout_ns": (_i, [_vp, _u64]),
    "cusort_mgpu_wait": (_i, [_vp, _vp]),
    "cusort_mgpu_set_timing": (_i, [_i]),
    "cusort_mgpu_get_phase_times": (_i, [C.POINTER(C.c_float), C.POINTER(C.c_char_p), _i]),
    "cusort_version": (C.c_char_p, []),
    "cusort_set_launch_mode": (_i, [_i]),
    "cusort_read_device_status": (_i, [_vp, C.POINTER(_u32), _vp]),
    "cusort_set_wait_limit_ns": (_u64, [_u64]),
    "cusort_debug_set_skip_tile": (_i64, [_i64]),
    "cusort_set_kernel_timing": (_i, [_i]),
    "cusort_get_kernel_times": (_i, [C.POINTER(C.c_float), C.POINTER(_i), _i]),
    "cusort_query_plan": (_i, [_i, _sz, _i64, _i, _i, C.POINTER(_i), C.POINTER(_i), C.POINTER(_i),
                               C.POINTER(_i), C.POINTER(_i)]),
}

_lib = None


class CusortError(RuntimeError):
    def __init__(self, code: int, what: str):
        super().__init__(f"{what} failed with cudaError_t {code}")
        self.code = code


def load() -> C.CDLL:
    """Load libcusort_b200.so (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise RuntimeError(
            f"{LIB_PATH} is missing: build it with `python -m libcusort_b200.build` "
            "(there is no CPU or library fallback for this path)")
    lib = C.CDLL(str(LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(code: int, what: str) -> None:
    if code != CUDA_SUCCESS:
        raise CusortError(code, what)


def key_type_id(kt) -> int:
    if isinstance(kt, int):
        return kt
    return KEY_TYPES[kt]
