"""Sharded multi-GPU sort on real GPUs through cusort_mgpu_sort.

With one GPU: a 1-rank communicator must give the single-GPU result.  With
>= 2 GPUs (one process per GPU, NCCL): the ranks' concatenated outputs must
equal the CPU oracle's stable sort of the global input, bit-exact, for each
exchange mode -- the fused partition + exchange pass writing into peers'
buffers ("routed", the default), the same pass run in chunks with copy-engine
pushes overlapping it ("pipe"; forced to 3 chunks here), copy-engine pushes
after a local partition ("copy") and NCCL send/recv ("nccl") -- on two calls
in a row with different inputs.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("no CUDA device", allow_module_level=True)

from libcusort_b200 import mgpu  # noqa: E402
from oracle import oracle as O  # noqa: E402
from tests import datagen as D  # noqa: E402


def test_single_rank_communicator_matches_oracle():
    s = mgpu.ShardedSorter(0, 1, mgpu.ShardedSorter.unique_id())
    try:
        keys = D.uniform_bits("i32", 300_001, seed=3)
        vals = np.arange(keys.size, dtype=np.uint32)
        ko, vo = s.sort(torch.from_numpy(keys).cuda(), torch.from_numpy(vals.view(np.int32)).cuda())
        ek, ev = O.oracle_sort("i32", keys, vals)
        assert np.array_equal(ko.cpu().numpy(), ek)
        assert np.array_equal(vo.cpu().numpy().view(np.uint32), ev)
    finally:
        s.close()


@pytest.mark.parametrize("exchange", ["routed", "pipe", "copy", "nccl"])
@pytest.mark.parametrize("kt,vdtype", [("u32", np.uint16), ("i16", np.uint8), ("f32", None), ("f64", np.uint64),
                                       ("u8", np.uint16)])
def test_single_rank_full_exchange_pipeline(monkeypatch, exchange, kt, vdtype):
    # The exchange kernels (routed partition into the receive buffer, chunked routing, copy-engine
    # and NCCL exchanges) on one GPU: a 1-rank communicator forced through the whole pipeline.
    monkeypatch.setenv("CUSORT_MGPU_FORCE_EXCHANGE", "1")
    monkeypatch.setenv("CUSORT_MGPU_EXCHANGE", exchange)
    monkeypatch.setenv("CUSORT_MGPU_CHUNKS", "3")
    s = mgpu.ShardedSorter(0, 1, mgpu.ShardedSorter.unique_id())
    try:
        n = 400_003
        for seed in (5, 6):  # two calls into the same buffers
            keys = D.zipf_table(kt, n, seed=seed, distinct=4096)
            vals = None if vdtype is None else np.random.default_rng(seed).integers(
                0, np.iinfo(vdtype).max, size=n, dtype=vdtype)
            kd = torch.from_numpy(np.ascontiguousarray(keys)).cuda()
            vd = None if vals is None else torch.from_numpy(vals.view(
                {1: np.int8, 2: np.int16, 8: np.int64}[vals.dtype.itemsize])).cuda()
            ko, vo = s.sort(kd, vd, capacity=n)
            ek, ev = O.oracle_sort(kt, keys, vals)
            assert np.array_equal(ko.cpu().numpy().view(np.uint8), ek.view(np.uint8))
            if vals is not None:
                assert np.array_equal(vo.cpu().numpy().view(vals.dtype), ev)
    finally:
        s.close()


def _port():
    so = socket.socket()
    so.bind(("127.0.0.1", 0))
    p = so.getsockname()[1]
    so.close()
    return p


def _worker(rank, world, port, case, exchange, q):
    import ctypes as C

    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["CUSORT_MGPU_EXCHANGE"] = exchange
    if exchange == "pipe":
        os.environ["CUSORT_MGPU_CHUNKS"] = "3"
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    s = None
    try:
        s = mgpu.ShardedSorter.from_torch_distributed()
        kind, kt, n, begin, end, desc, with_values = case
        ok = True
        for call in range(2):  # second call: new data into the same (already mapped) buffers
            seed = 2 + call
            keys = (D.zipf_table(kt, n, seed=seed, distinct=1 << 14) if kind == "zipf"
                    else D.uniform_bits(kt, n, seed=seed))
            gidx = np.arange(n, dtype=np.uint32)
            sl = np.array_split(np.arange(n), world)[rank]
            kd = torch.from_numpy(np.ascontiguousarray(keys[sl])).cuda()  # the tensor dtype selects the key type
            vd = torch.from_numpy(gidx[sl].view(np.int32)).cuda() if with_values else None
            if call == 0:
                out_k = torch.empty(n, dtype=kd.dtype, device="cuda")
                out_v = torch.empty(n, dtype=torch.int32, device="cuda") if with_values else None
            ko, vo = s.sort(kd, vd, capacity=n, begin_bit=begin, end_bit=end, descending=desc, out_keys=out_k,
                            out_values=out_v)
            st = C.c_uint32(0)
            rc = s.lib.cusort_read_device_status(C.c_void_p(s.temp.data_ptr()), C.byref(st),
                                                 C.c_void_p(torch.cuda.current_stream().cuda_stream))
            parts = [None] * world
            dist.all_gather_object(parts, (ko.cpu().numpy().tobytes(),
                                           vo.cpu().numpy().tobytes() if with_values else b"", rc, st.value))
            if rank == 0:
                gk = np.frombuffer(b"".join(p[0] for p in parts), dtype=keys.dtype)
                ek, ev = O.oracle_sort(kt, keys, gidx if with_values else None, begin, end, desc)
                ok = ok and np.array_equal(gk.view(np.uint8), ek.view(np.uint8))
                if with_values:
                    gv = np.frombuffer(b"".join(p[1] for p in parts), dtype=np.uint32)
                    ok = ok and np.array_equal(gv, ev)
                ok = ok and all(p[2] == 0 and p[3] == 0 for p in parts)
        if rank == 0:
            q.put(bool(ok))
    finally:
        if s is not None:
            s.close()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs >= 2 GPUs")
@pytest.mark.parametrize("exchange", ["pipe", "routed", "copy", "nccl"])
@pytest.mark.parametrize("case", [
    ("uniform", "u32", 1 << 20, 0, 32, False, True),
    ("uniform", "f32", 777_777, 0, 32, True, True),
    ("zipf", "i32", 1 << 20, 0, 32, False, True),
    ("uniform", "u32", 500_000, 5, 27, False, True),
    ("uniform", "u64", 600_001, 0, 64, False, False),
    ("uniform", "i16", 300_007, 0, 16, True, True),
], ids=lambda c: "-".join(map(str, c)))
def test_sharded_sort_all_gpus(case, exchange):
    import torch.multiprocessing as mp
    world = torch.cuda.device_count()
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    mp.start_processes(_worker, args=(world, _port(), case, exchange, q), nprocs=world, join=True,
                       start_method="spawn")
    assert q.get() is True
