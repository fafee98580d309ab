"""bench.py's N>1 path: the sharded multi-GPU sort, one rank per GPU.

Default: strong scaling of the global 2^32-item sort of uint32
keys (uniform, seeded per rank) with uint32 values = global index, split
evenly over the ranks (--total-log2n changes the global size).  --weak
instead gives every rank 2^log2n items.  value = all ranks' items / the
slowest rank's time.

Beside the timed figure the line carries:
  verified       the timed output checked globally: every rank sorted, ranks
                 in order, counts, values a permutation of 0..n-1 (exact sums
                 of v and v^2 against their closed forms), every value still
                 carrying its own key (a sum of a mix of (key, value) equal
                 before and after), stability inside and across ranks;
  strong_scaling the SAME global problem sorted on ONE GPU by rank 0 (the
                 single-GPU library, before the sharded run, its memory freed
                 after), so the speed-up is like for like;
  phases         per-phase device times of one sharded call (CUDA events);
  zipf           the configs[4] Zipf(1.1) variant over 2^24 distinct values,
                 timed and verified the same way;
  e2e            pinned host slice -> device -> sharded sort -> host, on a
                 bounded sample of at most 2^28 items per GPU.
"""
from __future__ import annotations

import ctypes as C
import datetime
import json
import os
from pathlib import Path


def _peaks(root: Path):
    p = root / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    return 6650.0, "fallback 6.65 TB/s"


_XCHG_DESC = {
    "pipe": "MSD-digit all-gather, chunked fused partition pass (own items straight into this GPU's receive buffer, "
            "each peer's into a contiguous staging run) with copy-engine pushes into the peers' IPC-mapped buffers "
            "overlapping the next chunk, NCCL one-word fence, local sort",
    "routed": "MSD-digit all-gather, ONE fused partition+exchange onesweep pass storing each item into its "
              "owner's buffer over NVLink (IPC-mapped peer pointers), NCCL one-word fence, local sort",
    "copy": "MSD-digit all-gather, partition pass, all-to-all as copy-engine pushes over NVLink into "
            "IPC-mapped peer buffers, local sort",
    "nccl": "MSD-digit all-gather, partition pass, all-to-all as grouped ncclSend/ncclRecv, local sort",
}
# Library kernels per step: digit count (1) + partition (routed: init + onesweep = 2; otherwise
# init + histogram + onesweep = 3) + local 4-pass sort (init + histogram + 4 onesweep = 6); the
# pipelined exchange runs C chunks: C digit counts + 1 sum + C x (init + onesweep) + 6.
_LAUNCHES = {"routed": 9, "copy": 10, "nccl": 10}
M32 = 0xFFFFFFFF
CHUNK = 1 << 26


def _chunks(n_local: int) -> int:
    return min(8, max(1, n_local >> 24))


def _mul32(torch, x, c: int):
    """(x * c) mod 2^32 for int64 tensors x in [0, 2^32) without int64 overflow."""
    return ((x & 0xFFFF) * c + (((x >> 16) * c) & 0xFFFF) * 65536) & M32


def _fmix32(torch, x):
    """MurmurHash3's 32-bit finalizer (public domain): a bijection on 32-bit words."""
    x = x & M32
    x = x ^ (x >> 16)
    x = _mul32(torch, x, 0x85EBCA6B)
    x = x ^ (x >> 13)
    x = _mul32(torch, x, 0xC2B2AE35)
    return x ^ (x >> 16)


def _slice(n_total: int, world: int, r: int):
    n = n_total // world + (1 if r < n_total % world else 0)
    first = r * (n_total // world) + min(r, n_total % world)
    return n, first


def _fill_rank(torch, dev, keys, vals, n_total, world, r, dist_kind, zipf_cdf=None, off=0):
    """Rank r's slice of the global input into keys/vals[off:off+n_r] (int32 bit patterns of uint32):
    uniform keys from generator seed 1000 + r, or Zipf(1.1) draws over 2^24 ranks mapped through a
    seeded bijective 32-bit mix; values = global index."""
    n, first = _slice(n_total, world, r)
    g = torch.Generator(device=dev)
    g.manual_seed((1000 if dist_kind == "uniform" else 5000) + r)
    for s0 in range(0, n, CHUNK):
        m = min(CHUNK, n - s0)
        if dist_kind == "uniform":
            k = torch.randint(-(2 ** 31), 2 ** 31, (m,), dtype=torch.int64, device=dev, generator=g)
        else:
            u = torch.rand(m, dtype=torch.float64, device=dev, generator=g)
            rk = torch.searchsorted(zipf_cdf, u).clamp_(max=zipf_cdf.numel() - 1)
            k = _fmix32(torch, rk ^ 0x5BD1E995)
        keys[off + s0:off + s0 + m] = _as_i32(torch, k & M32)
        vals[off + s0:off + s0 + m] = _as_i32(torch, torch.arange(first + s0, first + s0 + m, dtype=torch.int64,
                                                                  device=dev))
    return n, first


def _as_i32(torch, x):
    """int32 tensor with the bit patterns of x (int64 values in [0, 2^32))."""
    return (x - ((x >> 31) << 32)).to(torch.int32)


def _zipf_cdf(torch, dev, distinct=1 << 24, s=1.1):
    p = torch.arange(1, distinct + 1, dtype=torch.float64, device=dev).pow_(-s)
    c = torch.cumsum(p, 0)
    return c / c[-1]


def _u32(torch, t):
    return t.view(torch.int32).to(torch.int64) & M32


def _pair_mix_sum(torch, k32, v32) -> int:
    """Exact sum over items of fmix32(key ^ fmix32(value)): equal before and after the sort iff (up to
    hash collisions) the multiset of (key, value) pairs is unchanged."""
    tot = 0
    for s0 in range(0, k32.numel(), CHUNK):
        k = _u32(torch, k32[s0:s0 + CHUNK])
        v = _u32(torch, v32[s0:s0 + CHUNK])
        tot += int(_fmix32(torch, k ^ _fmix32(torch, v)).sum().item())
    return tot


def _local_checks(torch, ko, vo):
    """This rank's part: sorted (unsigned), stable (equal adjacent keys -> increasing values), exact
    sums of v and v^2 (split in 16-bit halves so no int64 overflows), first/last (key, value)."""
    n = ko.numel()
    sorted_ok, stable_ok = True, True
    s1 = s_hh = s_hl = s_ll = 0
    prev_k = prev_v = None
    for s0 in range(0, n, CHUNK):
        k = _u32(torch, ko[s0:s0 + CHUNK])
        v = _u32(torch, vo[s0:s0 + CHUNK])
        if prev_k is not None:
            k = torch.cat([prev_k, k])
            v = torch.cat([prev_v, v])
        sorted_ok &= bool((k[1:] >= k[:-1]).all().item())
        eq = k[1:] == k[:-1]
        stable_ok &= bool((v[1:][eq] > v[:-1][eq]).all().item())
        body = v[1:] if prev_k is not None else v
        hi, lo = body >> 16, body & 0xFFFF
        s1 += int(body.sum().item())
        s_hh += int((hi * hi).sum().item())
        s_hl += int((hi * lo).sum().item())
        s_ll += int((lo * lo).sum().item())
        prev_k, prev_v = k[-1:], v[-1:]
    s2 = (s_hh << 32) + (s_hl << 17) + s_ll
    ends = None
    if n:
        ends = (int(_u32(torch, ko[:1]).item()), int(_u32(torch, vo[:1]).item()),
                int(_u32(torch, ko[-1:]).item()), int(_u32(torch, vo[-1:]).item()))
    return {"n": n, "sorted": sorted_ok, "stable": stable_ok, "s1": s1, "s2": s2, "ends": ends}


def _global_verdict(stats, n_total, mix_in, mix_out):
    counts_ok = sum(s["n"] for s in stats) == n_total
    nonempty = [s for s in stats if s["n"]]
    order_ok, stable_across = True, True
    for a, b in zip(nonempty, nonempty[1:]):
        order_ok &= a["ends"][2] <= b["ends"][0]
        if a["ends"][2] == b["ends"][0]:
            stable_across &= a["ends"][3] < b["ends"][1]
    s1 = sum(s["s1"] for s in stats)
    s2 = sum(s["s2"] for s in stats)
    n = n_total
    perm_ok = s1 == n * (n - 1) // 2 and s2 == (n - 1) * n * (2 * n - 1) // 6
    return {"ranks_sorted": all(s["sorted"] for s in stats), "ranks_ordered": order_ok, "counts": counts_ok,
            "permutation": perm_ok, "values_carry_keys": mix_in == mix_out,
            "stable": all(s["stable"] for s in stats) and stable_across}


def _timed(torch, dist, dev, step, steps, warmup):
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        out = step()
    b.record()
    torch.cuda.synchronize()
    ms = torch.tensor([a.elapsed_time(b)], device=dev)
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    dist.barrier()
    return ms.item() / steps, out


def _one_gpu_same_problem(torch, dev, n_total, world, steps=3, warmup=1):
    """Rank 0 alone: the whole global uniform input (every rank's slice, same seeds) sorted on this
    GPU by the single-GPU library (in/out form), ms per sort; memory released afterwards."""
    from . import _capi
    lib = _capi.load()
    keys = torch.empty(n_total, dtype=torch.int32, device=dev)
    vals = torch.empty(n_total, dtype=torch.int32, device=dev)
    off = 0
    for r in range(world):
        n, _ = _fill_rank(torch, dev, keys, vals, n_total, world, r, "uniform", off=off)
        off += n
    ko, vo = torch.empty_like(keys), torch.empty_like(vals)
    s = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    P = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    nb = C.c_size_t(0)
    args = lambda t: (t, C.byref(nb), _capi.KEY_TYPES["u32"], P(keys), P(ko), 4, P(vals), P(vo), n_total, 0, 32, s)  # noqa
    _capi.check(lib.cusort_sort_pairs(*args(None)), "size query")
    temp = torch.empty(max(nb.value, 1), dtype=torch.uint8, device=dev)
    for _ in range(warmup):
        _capi.check(lib.cusort_sort_pairs(*args(P(temp))), "sort")
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        _capi.check(lib.cusort_sort_pairs(*args(P(temp))), "sort")
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / steps
    k = ko.view(torch.int32)[:: max(1, n_total >> 20)].to(torch.int64) & M32
    ok = bool((k[1:] >= k[:-1]).all().item())
    del keys, vals, ko, vo, temp
    torch.cuda.empty_cache()
    return {"t1_ms": ms, "gkeys_per_s": n_total / (ms * 1e-3) / 1e9, "sorted_sample": ok,
            "how": "rank 0 alone, before the sharded run: the same global input (every rank's slice, same seeds, "
                   "rank order) sorted by cusort_sort_pairs (in/out form, 64-bit offsets) on ONE GPU; "
                   f"{warmup} warm-up + {steps} timed sorts, CUDA events"}


def run(args, torch):
    import torch.distributed as dist

    from . import mgpu

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    os.environ.setdefault("NCCL_DEBUG", "WARN")  # keep stdout to the one JSON line
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    sorter = None
    try:
        if getattr(args, "weak", False):
            n_total = (1 << args.log2n) * world
            scaling = "weak"
        else:
            n_total = 1 << (args.total_log2n or 32)
            scaling = "strong"
        # the same global problem on one GPU first (rank 0 alone; the others wait)
        one_gpu = None
        if scaling == "strong" and rank == 0:
            one_gpu = _one_gpu_same_problem(torch, dev, n_total, world)
        dist.barrier()

        sorter = mgpu.ShardedSorter.from_torch_distributed()
        n_local, first = _slice(n_total, world, rank)
        keys = torch.empty(n_local, dtype=torch.int32, device=dev)
        vals = torch.empty(n_local, dtype=torch.int32, device=dev)
        _fill_rank(torch, dev, keys, vals, n_total, world, rank, "uniform")
        keys = keys.view(torch.uint32) if hasattr(torch, "uint32") else keys
        mix_in = _pair_mix_sum(torch, keys, vals)
        cap = int(n_local * 1.5) + 65536
        out_k = torch.empty(cap, dtype=keys.dtype, device=dev)
        out_v = torch.empty(cap, dtype=torch.int32, device=dev)

        def step():
            return sorter.sort(keys, vals, capacity=cap, out_keys=out_k, out_values=out_v)

        ms_step, (ko, vo) = _timed(torch, dist, dev, step, args.steps, args.warmup)

        def verify(ko, vo, mix_in):
            st = _local_checks(torch, ko, vo)
            st["mix"] = _pair_mix_sum(torch, ko, vo)
            stats = [None] * world
            dist.all_gather_object(stats, st)
            mixes = [None] * world
            dist.all_gather_object(mixes, mix_in)
            return _global_verdict(stats, n_total, sum(mixes), sum(s["mix"] for s in stats)), \
                [s["n"] for s in stats]

        verified, per_rank = verify(ko, vo, mix_in)

        # per-phase device times of two more calls (events on the stream; not the timed figure)
        mgpu.ShardedSorter.set_timing(True)
        phases = {}
        for _ in range(2):
            step()
            for k, v in mgpu.ShardedSorter.phase_times().items():
                phases[k] = phases.get(k, 0.0) + v / 2
        mgpu.ShardedSorter.set_timing(False)
        sorter.wait()  # bounded wait: a failed peer raises here instead of hanging
        allph = [None] * world
        dist.all_gather_object(allph, phases)

        # e2e: pinned host slice -> H2D -> sharded sort -> D2H of this rank's part,
        # on a sample of at most 2^28 items per GPU (the first items of each slice)
        e_local = min(n_local, 1 << 28)
        e_total = sum(min(_slice(n_total, world, r)[0], 1 << 28) for r in range(world))
        e_cap = int(e_local * 1.5) + 65536
        kh = keys[:e_local].cpu().pin_memory()
        vh = vals[:e_local].cpu().pin_memory()
        okh = torch.empty(e_cap, dtype=keys.dtype, pin_memory=True)
        ovh = torch.empty(e_cap, dtype=torch.int32, pin_memory=True)
        kd, vd = keys[:e_local].clone(), vals[:e_local].clone()
        del keys, vals, ko, vo

        def e2e_step():
            kd.copy_(kh, non_blocking=True)
            vd.copy_(vh, non_blocking=True)
            k2, v2 = sorter.sort(kd, vd, capacity=e_cap, out_keys=out_k[:e_cap], out_values=out_v[:e_cap])
            m = k2.numel()
            okh[:m].copy_(k2, non_blocking=True)
            ovh[:m].copy_(v2, non_blocking=True)

        e_steps = max(3, min(args.steps, 10))
        e_ms, _ = _timed(torch, dist, dev, e2e_step, e_steps, 2)
        del kd, vd, kh, vh, okh, ovh, out_k, out_v
        torch.cuda.empty_cache()

        # configs[4]'s Zipf(1.1) variant over 2^24 distinct values (strong scaling only)
        zipf = None
        if scaling == "strong":
            cdf = _zipf_cdf(torch, dev)
            keys = torch.empty(n_local, dtype=torch.int32, device=dev)
            vals = torch.empty(n_local, dtype=torch.int32, device=dev)
            _fill_rank(torch, dev, keys, vals, n_total, world, rank, "zipf", zipf_cdf=cdf)
            del cdf
            keys = keys.view(torch.uint32) if hasattr(torch, "uint32") else keys
            zmix_in = _pair_mix_sum(torch, keys, vals)
            zcap = 2 * n_local + 65536  # the hottest key alone holds ~11.5% of all items
            out_k = torch.empty(zcap, dtype=keys.dtype, device=dev)
            out_v = torch.empty(zcap, dtype=torch.int32, device=dev)

            def zstep():
                return sorter.sort(keys, vals, capacity=zcap, out_keys=out_k, out_values=out_v)

            z_steps = max(3, min(args.steps, 5))
            zms, (zko, zvo) = _timed(torch, dist, dev, zstep, z_steps, 1)
            zver, zper = verify(zko, zvo, zmix_in)
            zipf = {"ms_per_step": zms, "gkeys_per_s": n_total / (zms * 1e-3) / 1e9, "steps": z_steps,
                    "verified": zver, "items_per_rank": zper,
                    "data": "keys = fmix32(rank ^ 0x5BD1E995) of Zipf(1.1) draws over 2^24 ranks (inverse CDF, "
                            "seeded per rank), values = global index"}
            del keys, vals, out_k, out_v, zko, zvo

        if rank != 0:
            return None
        mode = os.environ.get("CUSORT_MGPU_EXCHANGE", "routed")
        mode = mode if mode in _XCHG_DESC else "routed"
        if mode == "pipe" and _chunks(n_local) == 1:
            mode = "routed"
        launches = (3 * _chunks(n_local) + 7) if mode == "pipe" else _LAUNCHES[mode]
        root = Path(__file__).resolve().parents[1]
        peak, peak_src = _peaks(root)
        kb = vb = 4
        # per-GPU algorithmic bytes: partition pass + 4 local passes (2*(K+V) each) + one histogram read
        local_bytes = (1 + 4) * 2 * n_local * (kb + vb) + 2 * n_local * kb
        xchg = n_local * (kb + vb) * (world - 1) / world  # expected bytes each GPU sends over NVLink
        t_ideal = local_bytes / (peak * 1e9) + xchg / 770e9
        value = n_total / (ms_step * 1e-3) / 1e9
        out = {
            "metric": "Gkeys/s (sharded uint32/uint32 SortPairs across GPUs)", "value": value,
            "unit": "Gkeys/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": scaling, "vs_baseline": None,
            "dtype": "uint32 keys / uint32 values (integer radix)",
            "data": "synthetic (seeded uniform uint32 keys per rank, values = global index)",
            "config": {"workload": "configs[4]-style sharded global sort: " + _XCHG_DESC[mode],
                       "exchange": mode,
                       "n_total": n_total, "n_per_gpu": n_local, "parallelism": f"shard{world}",
                       "l2": f"inputs per GPU {n_local * 8 / 2**20:.0f} MiB > L2"},
            "verified": verified, "items_per_rank": per_rank,
            "gpu_launches": args.steps * launches,
            "phases_ms": {"rank0": allph[0], "max_over_ranks": {k: max(p.get(k, 0.0) for p in allph)
                                                                for k in allph[0]}},
            "roofline": {"bound": "hbm+nvlink", "achieved_frac_of_pipeline": t_ideal / (ms_step * 1e-3),
                         "t_ideal_ms": t_ideal * 1e3, "local_hbm_bytes_per_gpu": local_bytes,
                         "nvlink_bytes_per_gpu": xchg, "peak_hbm_gbs": peak, "peak_source": peak_src,
                         "nvlink_gbs": 770.0, "nvlink_source": "measured peer copy per direction on this pool"},
            "e2e": {"value": e_total / (e_ms * 1e-3) / 1e9, "unit": "Gkeys/s", "ms_per_step": e_ms,
                    "sample": f"{e_total} items ({e_total // world} per GPU) of the same workload",
                    "h2d_bytes_per_step": e_total * (kb + vb), "d2h_bytes_per_step": e_total * (kb + vb)},
        }
        if one_gpu is not None:
            one_gpu["speedup"] = one_gpu["t1_ms"] / ms_step
            one_gpu["efficiency_vs_same_problem_on_1_gpu"] = one_gpu["t1_ms"] / (world * ms_step)
            out["strong_scaling"] = one_gpu
        if zipf is not None:
            out["zipf"] = zipf
        return out
    finally:
        if sorter is not None:
            sorter.close()
        dist.destroy_process_group()
