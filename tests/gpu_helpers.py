"""GPU-side helpers for the parity tests: run one sort through the C ABI of
libcusort_b200 (or of the reference library) on numpy inputs, with guard
regions around every device buffer (checked after the call in place of a
memory sanitizer)."""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from libcusort_b200 import _capi
from oracle import oracle as O

GUARD = 512
PATTERN = 0xA5


class DevBuf:
    """uint8 device buffer with guard bytes on both sides; `ptr` is the payload."""

    def __init__(self, nbytes: int, offset: int = 0, fill: int = PATTERN):
        self.nbytes = nbytes
        self.offset = offset
        self.t = torch.full((GUARD + offset + nbytes + GUARD,), PATTERN, dtype=torch.uint8, device="cuda")
        if fill != PATTERN and nbytes:
            self.t[GUARD + offset:GUARD + offset + nbytes] = fill
        self.ptr = C.c_void_p(self.t.data_ptr() + GUARD + offset)

    @classmethod
    def from_array(cls, a: np.ndarray, offset: int = 0):
        b = cls(a.nbytes, offset)
        if a.nbytes:
            b.t[GUARD + offset:GUARD + offset + a.nbytes] = torch.from_numpy(
                np.ascontiguousarray(a).view(np.uint8).reshape(-1)).cuda()
        return b

    def to_array(self, like: np.ndarray) -> np.ndarray:
        raw = self.t[GUARD + self.offset:GUARD + self.offset + self.nbytes].cpu().numpy()
        return raw.view(like.dtype).reshape(like.shape)

    def guards_ok(self) -> bool:
        h = self.t[:GUARD + self.offset].cpu().numpy()
        tail = self.t[GUARD + self.offset + self.nbytes:].cpu().numpy()
        return bool((h == PATTERN).all() and (tail == PATTERN).all())


def _stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def run_ours(kt: str, keys: np.ndarray, values: np.ndarray | None = None, begin_bit: int = 0,
             end_bit: int | None = None, descending: bool = False, api: str = "raw", offset_items: int = 0,
             launch_mode: int = 0, ksel0: int = 0, vsel0: int = 0):
    """Sort with libcusort_b200; returns (keys, values, info) after checking guards and status."""
    lib = _capi.load()
    n = keys.shape[0]
    kb = keys.dtype.itemsize
    end_bit = 8 * kb if end_bit is None else end_bit
    vb = 0 if values is None else values.dtype.itemsize * int(np.prod(values.shape[1:], dtype=np.int64))
    kid = _capi.KEY_TYPES[kt]
    nb = C.c_size_t(0)
    info = {}
    prev_mode = lib.cusort_set_launch_mode(launch_mode)
    try:
        if api == "raw":
            kin = DevBuf.from_array(keys, offset_items * kb)
            kout = DevBuf(keys.nbytes, offset_items * kb)
            vin = DevBuf.from_array(values, offset_items * vb) if vb else None
            vout = DevBuf(values.nbytes, offset_items * vb) if vb else None
            args = lambda t, tb: (  # noqa: E731
                (t, tb, kid, kin.ptr, kout.ptr, vb, vin.ptr, vout.ptr, n, begin_bit, end_bit, _stream()) if vb else
                (t, tb, kid, kin.ptr, kout.ptr, n, begin_bit, end_bit, _stream()))
            if vb:
                fn = lib.cusort_sort_pairs_descending if descending else lib.cusort_sort_pairs
            else:
                fn = lib.cusort_sort_keys_descending if descending else lib.cusort_sort_keys
            rc = fn(*args(None, C.byref(nb)))
            assert rc == 0, f"size query rc={rc}"
            info["temp_bytes"] = nb.value
            temp = DevBuf(nb.value, fill=0x5A)
            tb = C.c_size_t(nb.value)
            rc = fn(*args(temp.ptr if nb.value else None, C.byref(tb)))
            torch.cuda.synchronize()
            assert rc == 0, f"sort rc={rc}"
            ko = kout.to_array(keys)
            vo = vout.to_array(values) if vb else None
            # the in/out form must leave its inputs untouched
            assert np.array_equal(kin.to_array(keys).view(np.uint8), np.ascontiguousarray(keys).view(np.uint8))
            if vb:
                assert np.array_equal(vin.to_array(values).view(np.uint8),
                                      np.ascontiguousarray(values).view(np.uint8))
            bufs = [kin, kout, temp] + ([vin, vout] if vb else [])
        else:
            k0 = DevBuf.from_array(keys, offset_items * kb)
            k1 = DevBuf(keys.nbytes, offset_items * kb)
            kbufs = [k0, k1] if ksel0 == 0 else [k1, k0]
            kdb = _capi.DoubleBufferC()
            kdb.d_buffers[0] = kbufs[0].ptr.value
            kdb.d_buffers[1] = kbufs[1].ptr.value
            kdb.selector = ksel0
            vdb = _capi.DoubleBufferC()
            vbufs = []
            if vb:
                v0 = DevBuf.from_array(values, offset_items * vb)
                v1 = DevBuf(values.nbytes, offset_items * vb)
                vbufs = [v0, v1] if vsel0 == 0 else [v1, v0]
                vdb.d_buffers[0] = vbufs[0].ptr.value
                vdb.d_buffers[1] = vbufs[1].ptr.value
                vdb.selector = vsel0
            if vb:
                fn = lib.cusort_sort_pairs_descending_db if descending else lib.cusort_sort_pairs_db
                call = lambda t, tb: fn(t, tb, kid, C.byref(kdb), vb, C.byref(vdb), n, begin_bit, end_bit,  # noqa
                                        _stream())
            else:
                fn = lib.cusort_sort_keys_descending_db if descending else lib.cusort_sort_keys_db
                call = lambda t, tb: fn(t, tb, kid, C.byref(kdb), n, begin_bit, end_bit, _stream())  # noqa
            rc = call(None, C.byref(nb))
            assert rc == 0, f"size query rc={rc}"
            info["temp_bytes"] = nb.value
            temp = DevBuf(nb.value, fill=0x5A)
            tb = C.c_size_t(nb.value)
            rc = call(temp.ptr if nb.value else None, C.byref(tb))
            torch.cuda.synchronize()
            assert rc == 0, f"sort rc={rc}"
            info["ksel"] = kdb.selector
            info["vsel"] = vdb.selector
            ko = kbufs[kdb.selector].to_array(keys)
            vo = vbufs[vdb.selector].to_array(values) if vb else None
            bufs = [k0, k1, temp] + vbufs
        if nb.value >= 4:
            st = C.c_uint32(0)
            assert lib.cusort_read_device_status(temp.ptr, C.byref(st), _stream()) == 0
            info["status"] = st.value
            assert st.value == 0, f"device status {st.value}"
        for b in bufs:
            assert b.guards_ok(), "guard region overwritten"
    finally:
        lib.cusort_set_launch_mode(prev_mode)
    return ko, vo, info


def run_ref(kt: str, keys: np.ndarray, values: np.ndarray | None = None, begin_bit: int = 0,
            end_bit: int | None = None, descending: bool = False, api: str = "raw"):
    """Sort with the reference library (oracle/_ref); returns (keys, values, info)."""
    n = keys.shape[0]
    kb = keys.dtype.itemsize
    end_bit = 8 * kb if end_bit is None else end_bit
    vb = 0 if values is None else values.dtype.itemsize * int(np.prod(values.shape[1:], dtype=np.int64))
    raw = api == "raw"
    k0 = DevBuf.from_array(keys)
    k1 = DevBuf(keys.nbytes)
    v0 = DevBuf.from_array(values) if vb else None
    v1 = DevBuf(values.nbytes) if vb else None
    vp0 = v0.ptr if vb else None
    vp1 = v1.ptr if vb else None
    rc, tb, _, _ = O.ref_call(kt, vb, descending, raw, None, 0, k0.ptr, k1.ptr, 0, vp0, vp1, 0, n, begin_bit,
                              end_bit, _stream())
    assert rc == 0, f"reference size query rc={rc}"
    temp = DevBuf(max(tb, 1))
    rc, _, ks, vs = O.ref_call(kt, vb, descending, raw, temp.ptr if tb else None, tb, k0.ptr, k1.ptr, 0, vp0, vp1,
                               0, n, begin_bit, end_bit, _stream())
    torch.cuda.synchronize()
    assert rc == 0, f"reference sort rc={rc}"
    if raw:
        ko = k1.to_array(keys)
        vo = v1.to_array(values) if vb else None
    else:
        ko = (k0, k1)[ks].to_array(keys)
        vo = (v0, v1)[vs].to_array(values) if vb else None
    return ko, vo, {"temp_bytes": tb, "ksel": ks, "vsel": vs}


def same_bits(a: np.ndarray, b: np.ndarray) -> bool:
    return a.shape == b.shape and np.array_equal(np.ascontiguousarray(a).view(np.uint8),
                                                 np.ascontiguousarray(b).view(np.uint8))
