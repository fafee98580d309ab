"""Multi-GPU sharded sort, host logic on CPU (no GPU): two `gloo` ranks run the
library's real planning step (cusort_mgpu_plan over the all-gathered digit
counts) and the exchange; the GPU steps (digit counts, partition pass, local
sort) are stood in for by the oracle.  The concatenated rank outputs must equal
the oracle's stable sort of the global input -- which checks the plan, the
send/receive bookkeeping and the stability-by-global-index argument.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from libcusort_b200 import mgpu
from oracle import oracle as O
from tests import datagen as D


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _global_input(kind, kt, n, seed):
    if kind == "uniform":
        return D.uniform_bits(kt, n, seed)
    if kind == "equal":
        return np.full(n, 7, dtype=O.NP_DTYPE[kt])
    if kind == "zipf":
        return D.zipf_table(kt, n, seed, distinct=4096)
    if kind == "floats":
        return D.special_floats(kt, n, seed, frac=0.01)
    raise ValueError(kind)


def _worker(rank, world, port, case, out_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        kind, kt, n, begin, end, desc = case
        keys = _global_input(kind, kt, n, seed=5)
        gidx = np.arange(n, dtype=np.uint32)
        sl = np.array_split(np.arange(n), world)[rank]
        k, v = keys[sl], gidx[sl]
        msd_b = max(begin, end - 8)
        dk = O.numpy_digit_keys(kt, k, msd_b, end, desc).astype(np.int64)
        counts = torch.from_numpy(np.bincount(dk, minlength=256).astype(np.int64))
        gathered = [torch.zeros(256, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(gathered, counts)
        all_counts = torch.stack(gathered).numpy().astype(np.uint64)
        owner, send, recv, totals = mgpu.plan(all_counts, world, rank)
        assert int(totals.sum()) == n and int(send.sum()) == len(k) and int(recv.sum()) == int(totals[rank])
        # stable partition by the owner digit (the GPU's one-pass sort)
        perm = np.argsort(dk, kind="stable")
        pk, pv = k[perm], v[perm]
        assert np.all(np.diff(owner[dk[perm]]) >= 0)
        # all-to-all in source-rank order
        bounds = np.concatenate([[0], np.cumsum(send)])
        reqs, rbufs = [], {}
        for q in range(world):
            chunk_k = torch.from_numpy(np.ascontiguousarray(pk[bounds[q]:bounds[q + 1]]).view(np.uint8).copy())
            chunk_v = torch.from_numpy(pv[bounds[q]:bounds[q + 1]].astype(np.int64))
            if q == rank:
                rbufs[q] = (chunk_k, chunk_v)
                continue
            if send[q] > 0:
                reqs.append(dist.isend(chunk_k, q))
                reqs.append(dist.isend(chunk_v, q))
            if recv[q] > 0:
                bk = torch.empty(int(recv[q]) * keys.dtype.itemsize, dtype=torch.uint8)
                bv = torch.empty(int(recv[q]), dtype=torch.int64)
                reqs.append(dist.irecv(bk, q))
                reqs.append(dist.irecv(bv, q))
                rbufs[q] = (bk, bv)
        for r in reqs:
            r.wait()
        rk = np.concatenate([rbufs[q][0].numpy().view(keys.dtype) for q in range(world) if q in rbufs] or
                            [np.empty(0, dtype=keys.dtype)])
        rv = np.concatenate([rbufs[q][1].numpy().astype(np.uint32) for q in range(world) if q in rbufs] or
                            [np.empty(0, dtype=np.uint32)])
        assert len(rk) == int(totals[rank])
        # stable local sort of the received items (the GPU's full-key sort)
        ok, ov = O.oracle_sort(kt, rk, rv, begin, end, desc)
        parts = [None] * world
        dist.all_gather_object(parts, (ok.tobytes(), ov.tobytes()))
        if rank == 0:
            gk = np.frombuffer(b"".join(p[0] for p in parts), dtype=keys.dtype)
            gv = np.frombuffer(b"".join(p[1] for p in parts), dtype=np.uint32)
            ek, ev = O.oracle_sort(kt, keys, gidx, begin, end, desc)
            out_q.put(bool(np.array_equal(gk.view(np.uint8), ek.view(np.uint8)) and np.array_equal(gv, ev)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("case", [
    ("uniform", "u32", 20_000, 0, 32, False),
    ("uniform", "i64", 9_999, 0, 64, True),
    ("floats", "f32", 12_345, 0, 32, False),
    ("zipf", "u32", 20_000, 0, 32, False),
    ("equal", "i32", 5_000, 0, 32, False),
    ("uniform", "u32", 20_000, 3, 20, False),
], ids=lambda c: "-".join(map(str, c)))
def test_sharded_sort_host_logic_two_gloo_ranks(case):
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    mp.start_processes(_worker, args=(2, _port(), case, q), nprocs=2, join=True, start_method="spawn")
    assert q.get() is True


def test_plan_properties():
    rng = np.random.default_rng(0)
    for world in (1, 2, 3, 4, 8, 16):
        counts = rng.integers(0, 1000, size=(world, 256)).astype(np.uint64)
        counts[:, 17] += 50_000  # one heavy digit
        owner, send, recv, totals = mgpu.plan(counts, world, world - 1)
        assert np.all(np.diff(owner) >= 0) and owner.min() >= 0 and owner.max() < world
        assert int(totals.sum()) == int(counts.sum())
        assert int(send.sum()) == int(counts[world - 1].sum())
        # receive counts of this rank = sum over its digits of every rank's counts
        mine = owner == world - 1
        assert np.array_equal(recv, counts[:, mine].sum(axis=1).astype(np.int64))
    # balanced for uniform counts
    owner, _, _, totals = mgpu.plan(np.ones((8, 256), dtype=np.uint64), 8, 0)
    assert np.all(totals == 256)
