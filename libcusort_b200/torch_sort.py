"""PyTorch-facing sort over the C ABI (zero-copy on CUDA tensors).

``radix_sort(keys, values=None, descending=False, begin_bit=0, end_bit=None)``
is a stable LSD radix sort of a 1-D CUDA tensor (plus an optional payload
tensor whose leading dimension is the item count) through
``cusort_sort_keys`` / ``cusort_sort_pairs`` of include/cusort_b200.h; payload
rows of other widths than 1, 2, 4, 8 or 16 bytes go through
``cusort_sort_pairs_wide``.  ``segmented_sort`` sorts every segment
[begin_offsets[s], end_offsets[s]) independently through
``cusort_segmented_sort_keys`` / ``cusort_segmented_sort_pairs``.
Temporary storage is a uint8 CUDA tensor from torch's caching allocator; the
work runs on torch's current stream.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _capi

_DTYPE_KEY = {
    torch.uint8: "u8", torch.int8: "i8", torch.int16: "i16", torch.int32: "i32", torch.int64: "i64",
    torch.float32: "f32", torch.float64: "f64",
}
for _name, _kt in (("uint16", "u16"), ("uint32", "u32"), ("uint64", "u64")):
    if hasattr(torch, _name):
        _DTYPE_KEY[getattr(torch, _name)] = _kt


def key_type_of(dtype: torch.dtype) -> str:
    try:
        return _DTYPE_KEY[dtype]
    except KeyError:
        raise TypeError(f"unsupported key dtype {dtype}") from None


_NATIVE_VB = (1, 2, 4, 8, 16)


def _value_bytes(values: torch.Tensor, n: int, any_width: bool = False) -> int:
    if values.dim() < 1 or values.shape[0] != n:
        raise ValueError("values must have the item count as leading dimension")
    if not values.is_contiguous():
        raise ValueError("values must be contiguous")
    vb = values.element_size()
    for d in values.shape[1:]:
        vb *= d
    if vb < 1 or (not any_width and vb not in _NATIVE_VB):
        raise ValueError(f"value payload of {vb} bytes per item is not supported (1, 2, 4, 8 or 16)")
    return vb


def _check_like(name: str, t: torch.Tensor, ref: torch.Tensor) -> None:
    """An output tensor must match its input in dtype, shape and device and be contiguous:
    the kernels write exactly the input's bytes into it."""
    if t.dtype != ref.dtype or t.shape != ref.shape or t.device != ref.device or not t.is_contiguous():
        raise ValueError(f"{name} must be a contiguous tensor of the input's dtype, shape and device "
                         f"(got {t.dtype}, {tuple(t.shape)}, {t.device})")


def _check_args(keys, values, out_keys, out_values, temp, any_width: bool = False) -> int:
    """Shape, type and device checks of radix_sort's tensors; returns the value bytes per item
    (0 for keys-only).  No CUDA call."""
    if keys.dim() != 1 or not keys.is_contiguous():
        raise ValueError("keys must be a contiguous 1-D tensor")
    key_type_of(keys.dtype)
    n = keys.numel()
    vb = 0
    if values is not None:
        if values.device != keys.device:
            raise ValueError(f"values are on {values.device}, keys on {keys.device}")
        vb = _value_bytes(values, n, any_width)
        if out_values is not None:
            _check_like("out_values", out_values, values)
    elif out_values is not None:
        raise ValueError("out_values given without values")
    if out_keys is not None:
        _check_like("out_keys", out_keys, keys)
    if temp is not None and (temp.device != keys.device or temp.dtype != torch.uint8 or not temp.is_contiguous()):
        raise ValueError("temp must be a contiguous uint8 tensor on the keys' device")
    return vb


def temp_storage_bytes(key_type: str, n: int, value_bytes: int = 0, begin_bit: int = 0, end_bit: int | None = None,
                       raw: bool = True) -> int:
    """Size query (no CUDA call), as DeviceRadixSort with d_temp_storage == nullptr."""
    lib = _capi.load()
    kb = _capi.KEY_BYTES[key_type]
    end_bit = 8 * kb if end_bit is None else end_bit
    nbytes = C.c_size_t(0)
    kt = _capi.key_type_id(key_type)
    if raw:
        if value_bytes:
            rc = lib.cusort_sort_pairs(None, C.byref(nbytes), kt, None, None, value_bytes, None, None, n,
                                       begin_bit, end_bit, None)
        else:
            rc = lib.cusort_sort_keys(None, C.byref(nbytes), kt, None, None, n, begin_bit, end_bit, None)
    else:
        db = _capi.DoubleBufferC()
        vdb = _capi.DoubleBufferC()
        if value_bytes:
            rc = lib.cusort_sort_pairs_db(None, C.byref(nbytes), kt, C.byref(db), value_bytes, C.byref(vdb), n,
                                          begin_bit, end_bit, None)
        else:
            rc = lib.cusort_sort_keys_db(None, C.byref(nbytes), kt, C.byref(db), n, begin_bit, end_bit, None)
    _capi.check(rc, "size query")
    return nbytes.value


def radix_sort(keys: torch.Tensor, values: torch.Tensor | None = None, *, descending: bool = False,
               begin_bit: int = 0, end_bit: int | None = None, out_keys: torch.Tensor | None = None,
               out_values: torch.Tensor | None = None, temp: torch.Tensor | None = None):
    """Stable radix sort; returns (sorted_keys, sorted_values_or_None). Inputs are not modified.
    Payload rows of any width are accepted (1, 2, 4, 8 and 16 bytes move with the keys; other
    widths are gathered by the sorted permutation)."""
    if not keys.is_cuda:
        raise ValueError("keys must be a CUDA tensor (this path has no CPU implementation)")
    vb = _check_args(keys, values, out_keys, out_values, temp, any_width=True)
    lib = _capi.load()
    kt = key_type_of(keys.dtype)
    n = keys.numel()
    end_bit = 8 * keys.element_size() if end_bit is None else end_bit
    out_keys = torch.empty_like(keys) if out_keys is None else out_keys
    if vb:
        out_values = torch.empty_like(values) if out_values is None else out_values
    kid = _capi.key_type_id(kt)
    wide = vb and vb not in _NATIVE_VB
    if wide:
        q = C.c_size_t(0)
        _capi.check(lib.cusort_sort_pairs_wide(None, C.byref(q), kid, None, None, vb, None, None, n, begin_bit,
                                               end_bit, int(descending), None), "size query")
        need = q.value
    else:
        need = temp_storage_bytes(kt, n, vb, begin_bit, end_bit, raw=True)
    if temp is None or temp.numel() < need:
        temp = torch.empty(max(need, 1), dtype=torch.uint8, device=keys.device)
    nbytes = C.c_size_t(temp.numel())
    stream = C.c_void_p(torch.cuda.current_stream(keys.device).cuda_stream)
    with torch.cuda.device(keys.device):
        if wide:
            rc = lib.cusort_sort_pairs_wide(C.c_void_p(temp.data_ptr()), C.byref(nbytes), kid,
                                            C.c_void_p(keys.data_ptr()), C.c_void_p(out_keys.data_ptr()), vb,
                                            C.c_void_p(values.data_ptr()), C.c_void_p(out_values.data_ptr()), n,
                                            begin_bit, end_bit, int(descending), stream)
        elif vb:
            fn = lib.cusort_sort_pairs_descending if descending else lib.cusort_sort_pairs
            rc = fn(C.c_void_p(temp.data_ptr()), C.byref(nbytes), kid, C.c_void_p(keys.data_ptr()),
                    C.c_void_p(out_keys.data_ptr()), vb, C.c_void_p(values.data_ptr()),
                    C.c_void_p(out_values.data_ptr()), n, begin_bit, end_bit, stream)
        else:
            fn = lib.cusort_sort_keys_descending if descending else lib.cusort_sort_keys
            rc = fn(C.c_void_p(temp.data_ptr()), C.byref(nbytes), kid, C.c_void_p(keys.data_ptr()),
                    C.c_void_p(out_keys.data_ptr()), n, begin_bit, end_bit, stream)
    _capi.check(rc, "cusort sort")
    return out_keys, (out_values if vb else None)


def radix_sort_host(keys: torch.Tensor, values: torch.Tensor, *, descending: bool = False, begin_bit: int = 0,
                    end_bit: int | None = None, device: torch.device | int | None = None):
    """Stable sort of (keys, values) held in HOST memory on a GPU (cusort_sort_pairs_host): the
    copies to and from the device overlap the sort and each other.  keys: contiguous 1-D CPU
    tensor; values: CPU tensor with one row of 1, 2, 4, 8 or 16 bytes per key (pinned memory is
    what lets the copies overlap).  Returns new pinned CPU tensors (sorted_keys, sorted_values),
    complete when the call returns.  No CPU fallback: it needs the library and a CUDA device."""
    if keys.device.type != "cpu" or values.device.type != "cpu":
        raise ValueError("radix_sort_host takes CPU tensors; use radix_sort for CUDA tensors")
    vb = _check_args(keys, values, None, None, None)
    lib = _capi.load()
    kt = key_type_of(keys.dtype)
    n = keys.numel()
    end_bit = 8 * keys.element_size() if end_bit is None else end_bit
    if device is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    else:
        dev = torch.device("cuda", device) if isinstance(device, int) else torch.device(device)
    kid = _capi.key_type_id(kt)
    out_keys = torch.empty(keys.shape, dtype=keys.dtype, pin_memory=True)
    out_values = torch.empty(values.shape, dtype=values.dtype, pin_memory=True)
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev)
        nbytes = C.c_size_t(0)

        def call(temp_ptr):
            return lib.cusort_sort_pairs_host(temp_ptr, C.byref(nbytes), kid, C.c_void_p(keys.data_ptr()),
                                              C.c_void_p(out_keys.data_ptr()), vb, C.c_void_p(values.data_ptr()),
                                              C.c_void_p(out_values.data_ptr()), n, begin_bit, end_bit,
                                              int(descending), C.c_void_p(stream.cuda_stream))

        _capi.check(call(None), "cusort_sort_pairs_host size query")
        temp = torch.empty(max(nbytes.value, 1), dtype=torch.uint8, device=dev)
        _capi.check(call(C.c_void_p(temp.data_ptr())), "cusort_sort_pairs_host")
        stream.synchronize()
    return out_keys, out_values


def _check_offsets(keys: torch.Tensor, begin_offsets: torch.Tensor, end_offsets: torch.Tensor) -> int:
    """Segment offsets: int64, 1-D, contiguous, equal lengths, on the keys' device.  Returns the
    segment count.  No CUDA call."""
    for name, t in (("begin_offsets", begin_offsets), ("end_offsets", end_offsets)):
        if t.dtype != torch.int64 or t.dim() != 1 or not t.is_contiguous() or t.device != keys.device:
            raise ValueError(f"{name} must be a contiguous 1-D int64 tensor on the keys' device "
                             f"(got {t.dtype}, {tuple(t.shape)}, {t.device})")
    if begin_offsets.numel() != end_offsets.numel():
        raise ValueError("begin_offsets and end_offsets must have the same length")
    return begin_offsets.numel()


def segmented_sort(keys: torch.Tensor, begin_offsets: torch.Tensor, end_offsets: torch.Tensor,
                   values: torch.Tensor | None = None, *, descending: bool = False, begin_bit: int = 0,
                   end_bit: int | None = None, out_keys: torch.Tensor | None = None,
                   out_values: torch.Tensor | None = None):
    """Sorts every segment [begin_offsets[s], end_offsets[s]) of keys (and values) stably and
    independently into the same positions (CUB DeviceSegmentedRadixSort semantics; the segments
    must not overlap).  Positions outside every segment are not written: fresh outputs start as
    copies of the inputs, so they keep the input there.  Returns (keys, values_or_None)."""
    if not keys.is_cuda:
        raise ValueError("keys must be a CUDA tensor (this path has no CPU implementation)")
    vb = _check_args(keys, values, out_keys, out_values, None)
    S = _check_offsets(keys, begin_offsets, end_offsets)
    lib = _capi.load()
    kt = key_type_of(keys.dtype)
    kid = _capi.key_type_id(kt)
    n = keys.numel()
    end_bit = 8 * keys.element_size() if end_bit is None else end_bit
    out_keys = keys.clone() if out_keys is None else out_keys
    if vb:
        out_values = values.clone() if out_values is None else out_values
    P = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    stream = C.c_void_p(torch.cuda.current_stream(keys.device).cuda_stream)
    nbytes = C.c_size_t(0)

    def call(tp):
        if vb:
            return lib.cusort_segmented_sort_pairs(tp, C.byref(nbytes), kid, P(keys), P(out_keys), vb, P(values),
                                                   P(out_values), n, S, P(begin_offsets), P(end_offsets),
                                                   begin_bit, end_bit, int(descending), stream)
        return lib.cusort_segmented_sort_keys(tp, C.byref(nbytes), kid, P(keys), P(out_keys), n, S,
                                              P(begin_offsets), P(end_offsets), begin_bit, end_bit,
                                              int(descending), stream)

    with torch.cuda.device(keys.device):
        _capi.check(call(None), "segmented size query")
        temp = torch.empty(max(nbytes.value, 1), dtype=torch.uint8, device=keys.device)
        _capi.check(call(C.c_void_p(temp.data_ptr())), "cusort segmented sort")
    return out_keys, (out_values if vb else None)


def argsort(keys: torch.Tensor, *, descending: bool = False) -> torch.Tensor:
    """Stable argsort (int64 indices) by sorting (key, index) pairs."""
    idx = torch.arange(keys.numel(), device=keys.device, dtype=torch.int64)
    _, perm = radix_sort(keys, idx, descending=descending)
    return perm
