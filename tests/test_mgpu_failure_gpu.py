"""Failure handling of the sharded sort: a rank that never joins a call.

Two ranks on two GPUs (child processes, NVLS off in NCCL) sort once together.
Then rank 1 stays alive but never joins the second call -- it only waits on
the host -- so nothing of rank 1 is freed while rank 0 still might reach it.
Rank 0's second cusort_mgpu_sort must give up within its communicator's limit
(a few seconds) with an error instead of waiting forever in the all-gather;
the communicator is aborted, every later call on it fails at once, and the
device stays usable: a plain single-GPU sort right after is correct.  The
reference has no multi-GPU code; its own only wait is the unbounded lookback
spin (libcusort.cuh:1360-1374).
"""
from __future__ import annotations

import multiprocessing as mp
import os
import time

import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("no CUDA device", allow_module_level=True)

LIMIT_S = 3.0


def _rank_main(rank: int, uid: bytes, results, second_done, timeout_s: float):
    import numpy as np
    import torch

    from libcusort_b200 import _capi, mgpu
    from libcusort_b200.torch_sort import radix_sort
    out = {"rank": rank}
    try:
        torch.cuda.set_device(rank)
        s = mgpu.ShardedSorter(rank, 2, uid)
        s.set_timeout(timeout_s)
        g = torch.Generator(device="cuda")
        g.manual_seed(rank)
        n = 1 << 20
        keys = torch.randint(0, 2 ** 31, (n,), dtype=torch.int32, device="cuda", generator=g)
        vals = torch.arange(n, dtype=torch.int32, device="cuda") + rank * n
        ko, vo = s.sort(keys, vals)
        s.wait()
        k = ko.cpu().numpy()
        out["first_ok"] = bool(np.all(k[1:] >= k[:-1]))
        out["first_n"] = int(ko.numel())
        if rank == 1:
            # never joins the second call: waits on the host until rank 0 is done
            results.put(out)
            second_done.wait(120)
            s.close()
            return
        t0 = time.monotonic()
        try:
            s.sort(keys, vals)
            s.wait()
            out["second_err"] = None
        except _capi.CusortError as e:
            out["second_err"] = e.code
        out["second_s"] = time.monotonic() - t0
        try:  # the aborted communicator fails at once from now on
            s.sort(keys, vals)
            out["third_err"] = None
        except _capi.CusortError as e:
            out["third_err"] = e.code
        s.close()
        # the device is still usable
        ks, perm = radix_sort(keys, torch.arange(n, dtype=torch.int32, device="cuda"))
        ref = torch.sort(keys, stable=True)
        out["after_ok"] = bool(torch.equal(ks, ref.values)) and bool(torch.equal(perm.long(), ref.indices))
    except Exception as e:  # reported to the parent
        out["exception"] = f"{type(e).__name__}: {e}"
    results.put(out)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_rank_that_never_joins_ends_the_call_with_an_error():
    from libcusort_b200 import _capi, mgpu
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ.setdefault("NCCL_DEBUG", "WARN")
    uid = mgpu.ShardedSorter.unique_id()
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    second_done = ctx.Event()
    procs = [ctx.Process(target=_rank_main, args=(r, uid, results, second_done, LIMIT_S)) for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    try:
        deadline = time.monotonic() + 240
        while len(got) < 2 and time.monotonic() < deadline:
            try:
                r = results.get(timeout=5)
            except Exception:
                continue
            got[r["rank"]] = r
            if r["rank"] == 0:
                second_done.set()
        second_done.set()
        for p in procs:
            p.join(60)
    finally:
        for p in procs:
            if p.is_alive():
                p.kill()
                p.join(10)
    assert set(got) == {0, 1}, f"missing rank reports: {got}"
    r0, r1 = got[0], got[1]
    assert "exception" not in r0 and "exception" not in r1, (r0, r1)
    assert r0["first_ok"] and r1["first_ok"] and r0["first_n"] + r1["first_n"] == 2 << 20
    assert r0["second_err"] is not None, "a call whose peer never joined did not fail"
    assert r0["second_s"] < LIMIT_S + 10, f"the failure took {r0['second_s']:.1f} s"
    assert r0["third_err"] == _capi.CUDA_ERROR_TIMEOUT
    assert r0["after_ok"]
