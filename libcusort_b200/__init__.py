"""libcusort_b200 -- B200-native (sm_100a) LSD radix sort, a drop-in for
cusort::DeviceRadixSort of IlyaGrebnov/libcusort behind the C ABI in
include/cusort_b200.h (C++ callers: include/cusort_b200.cuh).

Python modules here are thin bindings for tests, the benchmark and PyTorch
callers; the sort itself is the CUDA library libcusort_b200/_lib/libcusort_b200.so.
"""
from ._capi import KEY_BYTES, KEY_TYPES, CusortError, DoubleBufferC, load  # noqa: F401

__version__ = "1.0.1-b200.1"
