"""bench.py's N>1 path: the sharded multi-GPU sort, one rank per GPU.

Default: strong scaling of the global 2^32-item sort of uint32
keys (uniform, seeded per rank) with uint32 values = global index, split
evenly over the ranks (--total-log2n changes the global size).  --weak
instead gives every rank 2^log2n items.  value = all ranks' items / the
slowest rank's time.  The end-to-end figure (pinned host slice -> device ->
sharded sort -> host) runs the same call on a bounded sample of at most
2^28 items per GPU, stated in the JSON line.
"""
from __future__ import annotations

import ctypes as C
import datetime
import json
import os
import statistics
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


def _chunks(n_local: int) -> int:
    return min(8, max(1, n_local >> 24))


def run(args, torch):
    import torch.distributed as dist

    from . import mgpu

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        # The reference has no multi-GPU mode: rank 0 runs its single-GPU bench, the others exit.
        if rank != 0:
            return None
        import bench
        torch.cuda.set_device(local)
        from oracle import oracle as O
        if not O.ref_available():
            return {"impl": "reference", "unavailable": "oracle/_ref/libcusort_ref.so was not built"}
        out = bench.run_single(args, torch)
        out["note"] = "reference is single-GPU only: rank 0 ran the N=1 workload, other ranks idle"
        return out

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    os.environ.setdefault("NCCL_DEBUG", "WARN")  # keep stdout to the one JSON line
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    sorter = None
    try:
        sorter = mgpu.ShardedSorter.from_torch_distributed()
        if getattr(args, "weak", False):
            n_total = (1 << args.log2n) * world
            scaling = "weak"
        else:
            n_total = 1 << (args.total_log2n or 32)
            scaling = "strong"
        n_local = n_total // world + (1 if rank < n_total % world else 0)
        first = rank * (n_total // world) + min(rank, n_total % world)
        g = torch.Generator(device=dev)
        g.manual_seed(1000 + rank)
        # uint32 keys (the int32 bit pattern, sorted as unsigned) and uint32 global-index values
        keys = torch.empty(n_local, dtype=torch.int32, device=dev)
        vals = torch.empty(n_local, dtype=torch.int32, device=dev)
        chunk = 1 << 27
        for s0 in range(0, n_local, chunk):
            m = min(chunk, n_local - s0)
            keys[s0:s0 + m] = torch.randint(-(2 ** 31), 2 ** 31, (m,), dtype=torch.int64, device=dev,
                                            generator=g).to(torch.int32)
            vals[s0:s0 + m] = torch.arange(first + s0, first + s0 + m, dtype=torch.int64, device=dev).to(torch.int32)
        keys = keys.view(torch.uint32) if hasattr(torch, "uint32") else keys
        cap = int(n_local * 1.5) + 65536
        out_k = torch.empty(cap, dtype=keys.dtype, device=dev)
        out_v = torch.empty(cap, dtype=torch.int32, device=dev)

        def step():
            return sorter.sort(keys, vals, capacity=cap, out_keys=out_k, out_values=out_v)

        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize()
        dist.barrier()
        torch.cuda.synchronize()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(args.steps):
            ko, vo = step()
        b.record()
        torch.cuda.synchronize()
        ms = torch.tensor([a.elapsed_time(b)], device=dev)
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        dist.barrier()
        ms_step = ms.item() / args.steps

        # verification: each rank sorted, ranks ordered, counts add up (unsigned
        # order checked as signed order of the bit pattern with the top bit flipped)
        n_mine = ko.numel()
        ks = ko.view(torch.int32) ^ (-(2 ** 31))
        ok_local = bool((ks[1:] >= ks[:-1]).all().item()) if n_mine > 1 else True
        lo = ks[0].item() if n_mine else 2 ** 31 - 1
        hi = ks[-1].item() if n_mine else -(2 ** 31)
        del ks
        stats = [None] * world
        dist.all_gather_object(stats, (n_mine, lo, hi, ok_local, int(n_local)))
        counts_ok = sum(s[0] for s in stats) == n_total
        order_ok = all(stats[i][2] <= stats[j][1] for i in range(world) for j in range(i + 1, world)
                       if stats[i][0] and stats[j][0])
        sorted_ok = all(s[3] for s in stats)

        # e2e: pinned host slice -> H2D -> sharded sort -> D2H of this rank's part,
        # on a sample of at most 2^28 items per GPU (the first items of each slice)
        e_local = min(n_local, 1 << 28)
        e_total = sum(min(n_total // world + (1 if r < n_total % world else 0), 1 << 28) for r in range(world))
        e_cap = int(e_local * 1.5) + 65536
        kh = keys[:e_local].cpu().pin_memory()
        vh = vals[:e_local].cpu().pin_memory()
        okh = torch.empty(e_cap, dtype=keys.dtype, pin_memory=True)
        ovh = torch.empty(e_cap, dtype=torch.int32, pin_memory=True)
        kd, vd = keys[:e_local].clone(), vals[:e_local].clone()
        del keys, vals

        def e2e_step():
            kd.copy_(kh, non_blocking=True)
            vd.copy_(vh, non_blocking=True)
            k2, v2 = sorter.sort(kd, vd, capacity=e_cap, out_keys=out_k[:e_cap], out_values=out_v[:e_cap])
            m = k2.numel()
            okh[:m].copy_(k2, non_blocking=True)
            ovh[:m].copy_(v2, non_blocking=True)

        e_steps = max(3, min(args.steps, 10))
        for _ in range(2):
            e2e_step()
        torch.cuda.synchronize()
        dist.barrier()
        a.record()
        for _ in range(e_steps):
            e2e_step()
        b.record()
        torch.cuda.synchronize()
        ems = torch.tensor([a.elapsed_time(b)], device=dev)
        dist.all_reduce(ems, op=dist.ReduceOp.MAX)
        e_ms = ems.item() / e_steps

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
        return {
            "metric": "Gkeys/s (sharded uint32/uint32 SortPairs across GPUs)", "value": n_total / (ms_step * 1e-3) / 1e9,
            "unit": "Gkeys/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": scaling, "vs_baseline": None,
            "dtype": "uint32 keys / uint32 values (integer radix)",
            "data": "synthetic (seeded uniform uint32 keys per rank, values = global index)",
            "config": {"workload": "configs[4]-style sharded global sort: " + _XCHG_DESC[mode],
                       "exchange": mode,
                       "n_total": n_total, "n_per_gpu": n_local, "parallelism": f"shard{world}",
                       "l2": f"inputs per GPU {n_local * 8 / 2**20:.0f} MiB > L2"},
            "verified": {"ranks_sorted": sorted_ok, "ranks_ordered": order_ok, "counts": counts_ok},
            "gpu_launches": args.steps * launches,
            "roofline": {"bound": "hbm+nvlink", "achieved_frac_of_pipeline": t_ideal / (ms_step * 1e-3),
                         "t_ideal_ms": t_ideal * 1e3, "local_hbm_bytes_per_gpu": local_bytes,
                         "nvlink_bytes_per_gpu": xchg, "peak_hbm_gbs": peak, "peak_source": peak_src,
                         "nvlink_gbs": 770.0, "nvlink_source": "measured peer copy per direction on this pool"},
            "e2e": {"value": e_total / (e_ms * 1e-3) / 1e9, "unit": "Gkeys/s", "ms_per_step": e_ms,
                    "sample": f"{e_total} items ({e_total // world} per GPU) of the same workload",
                    "h2d_bytes_per_step": e_total * (kb + vb), "d2h_bytes_per_step": e_total * (kb + vb)},
        }
    finally:
        if sorter is not None:
            sorter.close()
        dist.destroy_process_group()
