"""Sharded multi-GPU sort (C ABI cusort_mgpu_*) for PyTorch callers.

One process per GPU.  The NCCL communicator is the library's own
(cusort_mgpu_comm_init); its 128-byte id is created on rank 0 and broadcast
through the default torch.distributed process group.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _capi
from .torch_sort import _check_args, key_type_of


def _check_output(name: str, t: torch.Tensor, ref: torch.Tensor, cap: int) -> None:
    """Other ranks write up to `cap` items into an output through IPC: it must hold them."""
    if (t.dtype != ref.dtype or t.device != ref.device or not t.is_contiguous() or t.dim() != ref.dim()
            or t.shape[1:] != ref.shape[1:] or t.shape[0] < cap):
        raise ValueError(f"{name} must be a contiguous tensor of the input's dtype, device and row shape with at "
                         f"least capacity={cap} rows (got {t.dtype}, {tuple(t.shape)}, {t.device})")


class ShardedSorter:
    def __init__(self, rank: int, world: int, uid: bytes):
        self.lib = _capi.load()
        self.rank, self.world = rank, world
        comm = C.c_void_p()
        buf = C.create_string_buffer(bytes(uid), 128)
        _capi.check(self.lib.cusort_mgpu_comm_init(C.byref(comm), buf, world, rank), "cusort_mgpu_comm_init")
        self.comm = comm
        self.temp = None

    @staticmethod
    def unique_id() -> bytes:
        lib = _capi.load()
        buf = C.create_string_buffer(128)
        _capi.check(lib.cusort_mgpu_unique_id(buf), "cusort_mgpu_unique_id")
        return buf.raw

    @classmethod
    def from_torch_distributed(cls):
        import torch.distributed as dist
        rank, world = dist.get_rank(), dist.get_world_size()
        obj = [cls.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        return cls(rank, world, obj[0])

    def close(self):
        if self.comm:
            self.lib.cusort_mgpu_comm_destroy(self.comm)
            self.comm = None

    def set_timeout(self, seconds: float) -> None:
        """Bound on every host wait of this communicator (default 30 s); on expiry the
        communicator is aborted and the call raises CusortError (cudaErrorTimeout)."""
        _capi.check(self.lib.cusort_mgpu_set_timeout_ns(self.comm, int(seconds * 1e9)), "cusort_mgpu_set_timeout_ns")

    def wait(self) -> None:
        """Bounded wait for everything queued on the current stream (the exchange fence and the
        local sort included); raises CusortError if a peer failed or the limit passed."""
        _capi.check(self.lib.cusort_mgpu_wait(self.comm, C.c_void_p(torch.cuda.current_stream().cuda_stream)),
                    "cusort_mgpu_wait")

    @staticmethod
    def set_timing(enable: bool) -> bool:
        """Per-phase CUDA-event timing of later sort() calls on this host thread."""
        return bool(_capi.load().cusort_mgpu_set_timing(int(enable)))

    @staticmethod
    def phase_times() -> dict:
        """{phase name: ms} of this thread's last sort() while timing was on."""
        lib = _capi.load()
        ms = (C.c_float * 8)()
        names = (C.c_char_p * 8)()
        m = lib.cusort_mgpu_get_phase_times(ms, names, 8)
        return {names[i].decode(): float(ms[i]) for i in range(m)}

    def _call(self, temp_ptr, nbytes, kt, vb, kin, vin, n, kout, vout, cap, n_out, b, e, desc):
        stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
        return self.lib.cusort_mgpu_sort(self.comm, temp_ptr, C.byref(nbytes), _capi.key_type_id(kt), vb, kin, vin,
                                         n, kout, vout, cap, C.byref(n_out), b, e, int(desc), stream)

    def sort(self, keys: torch.Tensor, values: torch.Tensor | None = None, *, capacity: int | None = None,
             begin_bit: int = 0, end_bit: int | None = None, descending: bool = False, out_keys=None,
             out_values=None):
        """Sorts this rank's slice as part of the global sort; returns this rank's (keys, values) part."""
        if not keys.is_cuda:
            raise ValueError("keys must be a CUDA tensor (this path has no CPU implementation)")
        vb = _check_args(keys, values, None, None, None)
        if out_values is not None and values is None:
            raise ValueError("out_values given without values")
        kt = key_type_of(keys.dtype)
        n = keys.numel()
        end_bit = 8 * keys.element_size() if end_bit is None else end_bit
        cap = capacity if capacity is not None else 2 * n + 4096
        if cap < 0:
            raise ValueError("capacity must be >= 0")
        if out_keys is None:
            out_keys = torch.empty(cap, dtype=keys.dtype, device=keys.device)
        else:
            _check_output("out_keys", out_keys, keys, cap)
        if vb and out_values is None:
            out_values = torch.empty((cap,) + tuple(values.shape[1:]), dtype=values.dtype, device=keys.device)
        elif vb:
            _check_output("out_values", out_values, values, cap)
        kin = C.c_void_p(keys.data_ptr())
        vin = C.c_void_p(values.data_ptr()) if vb else None
        kout = C.c_void_p(out_keys.data_ptr())
        vout = C.c_void_p(out_values.data_ptr()) if vb else None
        nbytes = C.c_size_t(0)
        n_out = C.c_int64(0)
        _capi.check(self._call(None, nbytes, kt, vb, kin, vin, n, kout, vout, cap, n_out, begin_bit, end_bit,
                               descending), "cusort_mgpu_sort size query")
        if self.temp is None or self.temp.numel() < nbytes.value:
            self.temp = torch.empty(max(nbytes.value, 1), dtype=torch.uint8, device=keys.device)
        nbytes = C.c_size_t(self.temp.numel())
        _capi.check(self._call(C.c_void_p(self.temp.data_ptr()), nbytes, kt, vb, kin, vin, n, kout, vout, cap, n_out,
                               begin_bit, end_bit, descending), "cusort_mgpu_sort")
        m = n_out.value
        return out_keys[:m], (out_values[:m] if vb else None)


def plan(all_counts, world: int, rank: int):
    """Host-only planning step (cusort_mgpu_plan): returns (owner[256], send[world], recv[world], totals[world])."""
    import numpy as np
    lib = _capi.load()
    ac = np.ascontiguousarray(all_counts, dtype=np.uint64).reshape(world, 256)
    owner = np.zeros(256, dtype=np.int32)
    send = np.zeros(world, dtype=np.int64)
    recv = np.zeros(world, dtype=np.int64)
    totals = np.zeros(world, dtype=np.int64)
    rc = lib.cusort_mgpu_plan(ac.ctypes.data_as(C.POINTER(C.c_uint64)), world, rank,
                              owner.ctypes.data_as(C.POINTER(C.c_int)), send.ctypes.data_as(C.POINTER(C.c_int64)),
                              recv.ctypes.data_as(C.POINTER(C.c_int64)), totals.ctypes.data_as(C.POINTER(C.c_int64)))
    if rc:
        raise ValueError("cusort_mgpu_plan rejected the arguments")
    return owner, send, recv, totals
