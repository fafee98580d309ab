#!/usr/bin/env python
"""Benchmark of the B200 radix sort (one JSON line on rank 0).

Default workload (N=1): BASELINE config 2 -- SortPairs ascending of 2^26
int32 keys uniform over all 32 bits with uint32 values = original index,
through the library's in/out-pointer C ABI (cusort_sort_pairs).  A "step" is
one complete sort call (init + histogram + 4 onesweep passes).

  value     Gkeys/s with inputs resident in HBM (inputs are 512 MiB > L2,
            so no L2 flush is needed between steps)
  e2e       same metric through the same C ABI with HOST buffers: pinned
            H2D copy of keys+values, sort, D2H copy of sorted keys+values
  roofline  onesweep kernel: algorithmic bytes 2*n*(K+V) per launch over its
            CUDA-event launch duration (measured live in a second pass with
            per-kernel events), against MEASURED_PEAKS.json hbm_gbs
  cpu_baseline  the oracle's parallel std::stable_sort on the host cores,
            bounded sample

--impl reference times the UNMODIFIED reference library compiled for sm_100a
(oracle/_ref) on the same workload through its own public API.

secondary  u32 keys-only 2^26; the other BASELINE.json single-GPU configs at
            2^26; configs[0] (2^20 u32 keys-only, 4 MiB: L2-resident, so a
            hot-L2, launch-latency-bound figure), direct and graph launches;
            input orders (sorted, reverse sorted, all equal, 16 distinct
            values; keys-only and pairs); ours only: segmented sort of 2^26
            pairs, one entry per length class

N>1 (torchrun): sharded multi-GPU sort of 2^32 int32/uint32 pairs split over
the GPUs (strong scaling, configs[4]); --weak for 2^26 pairs per GPU.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "Gkeys/s (2^26 int32 keys + uint32 values, SortPairs, 1 GPU)"
UNIT = "Gkeys/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--log2n", type=int, default=26)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-secondary", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--total-log2n", type=int, default=None,
                    help="N>1: global item count 2^this, split over the GPUs (strong scaling; default 32, configs[4])")
    ap.add_argument("--weak", action="store_true",
                    help="N>1: 2^log2n items per GPU (weak scaling) instead of the fixed global size")
    ap.add_argument("--profile-case", choices=["u32_keys", "i32_u32_pairs", "i32_u32_pairs_lowent", "u16_keys",
                                               "seg_i32_u32_pairs_1000"], default=None,
                    help="only run --warmup + --steps sorts of this case (for ncu captures)")
    ap.add_argument("--lookback-stall", action="store_true",
                    help="report the lookback timer of a library built with CUSORT_LOOKBACK_TIMER=1 (see build.py)")
    return ap.parse_args()


# ---------------------------------------------------------------------------
# clocks sampling (nvidia-smi) around the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []
        self.t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.t = threading.Thread(target=self._read, daemon=True)
        self.t.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.time(), line.strip()))

    def stop(self, t0: float, t1: float):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for ts, line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            rows.append((ts, parts))
        inside = [r for r in rows if t0 <= r[0] <= t1] or rows
        sm = [float(p[1]) for _, p in inside if p[1].replace(".", "").isdigit()]
        mx = [float(p[2]) for _, p in inside if p[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for _, p in inside:
            for nm, v in zip(names, p[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(inside),
                "window": "timed region" if any(t0 <= r[0] <= t1 for r in rows) else "whole run"}


# ---------------------------------------------------------------------------
# workload
# ---------------------------------------------------------------------------
def make_inputs(torch, n: int, seed: int, device):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    keys = torch.randint(-(2 ** 31), 2 ** 31, (n,), dtype=torch.int64, device=device, generator=g).to(torch.int32)
    vals = torch.arange(n, dtype=torch.int32, device=device)  # uint32 bit pattern = index
    return keys, vals


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    return 6650.0, "fallback 6.65 TB/s"


def traffic_from_profiles(workload: str):
    p = ROOT / "profiles" / "onesweep_traffic.json"
    if not p.exists():
        return None
    d = json.loads(p.read_text())
    return d.get(workload)


class Sorter:
    """One SortPairs/SortKeys call through a C ABI (ours or the reference's).

    api="raw": the in/out-pointer form (inputs never written).  api="db": the
    DoubleBuffer form over (keys_in, keys_out) and (vals_in, vals_out); every
    call starts from selector 0, so the caller restores keys_in / vals_in
    before each call (the form clobbers both buffers)."""

    def __init__(self, impl, torch, kt_name, kid, kb, vb, n, keys_in, keys_out, vals_in, vals_out, stream,
                 descending=False, begin_bit=0, end_bit=None, api="raw"):
        self.torch = torch
        self.impl = impl
        self.n = n
        self.api = api
        s = C.c_void_p(stream)
        kin, kout = C.c_void_p(keys_in.data_ptr()), C.c_void_p(keys_out.data_ptr())
        vin = C.c_void_p(vals_in.data_ptr()) if vb else None
        vout = C.c_void_p(vals_out.data_ptr()) if vb else None
        bb, eb = begin_bit, (8 * kb if end_bit is None else end_bit)
        self.sel = (0, 0)  # DoubleBuffer selectors after the last call
        if impl == "ours":
            from libcusort_b200 import _capi
            lib = _capi.load()
            if api == "db":
                kdb, vdb = _capi.DoubleBufferC(), _capi.DoubleBufferC()
                kdb.d_buffers[0], kdb.d_buffers[1] = kin.value, kout.value
                if vb:
                    vdb.d_buffers[0], vdb.d_buffers[1] = vin.value, vout.value

                def call(t, tb):
                    kdb.selector, vdb.selector = 0, 0
                    if vb:
                        fn = lib.cusort_sort_pairs_descending_db if descending else lib.cusort_sort_pairs_db
                        rc = fn(t, C.byref(tb), kid, C.byref(kdb), vb, C.byref(vdb), n, bb, eb, s)
                    else:
                        fn = lib.cusort_sort_keys_descending_db if descending else lib.cusort_sort_keys_db
                        rc = fn(t, C.byref(tb), kid, C.byref(kdb), n, bb, eb, s)
                    self.sel = (kdb.selector, vdb.selector)
                    return rc
                self.call = call
            elif vb:
                fn = lib.cusort_sort_pairs_descending if descending else lib.cusort_sort_pairs
                self.call = lambda t, tb: fn(t, C.byref(tb), kid, kin, kout, vb, vin, vout, n, bb, eb, s)
            else:
                fn = lib.cusort_sort_keys_descending if descending else lib.cusort_sort_keys
                self.call = lambda t, tb: fn(t, C.byref(tb), kid, kin, kout, n, bb, eb, s)
            self.lib = lib
        else:
            from oracle import oracle as O
            rl = O._load_ref()
            fn = getattr(rl, f"ref_sort_k{kid}")
            ks, vs = C.c_int(0), C.c_int(0)
            dflag = int(bool(descending))
            raw = 1 if api == "raw" else 0

            def call(t, tb):
                ks.value, vs.value = 0, 0
                rc = fn(vb, dflag, raw, t, C.byref(tb), kin, kout, C.byref(ks), vin, vout, C.byref(vs), n, bb, eb, s)
                self.sel = (ks.value, vs.value)
                return rc
            self.call = call
        tb = C.c_size_t(0)
        rc = self.call(None, tb)
        if rc != 0:
            raise RuntimeError(f"size query failed rc={rc}")
        self.temp = torch.empty(max(tb.value, 1), dtype=torch.uint8, device=keys_in.device)
        self.tp = C.c_void_p(self.temp.data_ptr())
        self.tb = C.c_size_t(tb.value)

    def __call__(self):
        rc = self.call(self.tp, self.tb)
        if rc != 0:
            raise RuntimeError(f"sort failed rc={rc}")


def time_steps(torch, fn, steps: int, warmup: int, dist=None):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        fn()
    b.record()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    return a.elapsed_time(b)


def time_restored(torch, restore, fn, steps: int, warmup: int):
    """Mean ms per call of fn() when every call needs its inputs restored first
    (the DoubleBuffer form clobbers both buffers): restore() runs outside the
    timed interval, and CUDA events on the launching stream bracket each call."""
    for _ in range(warmup):
        restore()
        fn()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for a, b in ev:
        restore()
        a.record()
        fn()
        b.record()
    torch.cuda.synchronize()
    return sum(a.elapsed_time(b) for a, b in ev) / steps


def verify_index_pairs(torch, keys_in, ko, vo, unsigned=False):
    """Checks a SortPairs output whose input values were the original indices:
    keys ascending, values a permutation of 0..n-1, every value carrying its
    own key (keys_in[value] == key) and stability (inside each run of equal
    keys the values strictly increase)."""
    k = ko.view(torch.int32)
    n = k.numel()
    if unsigned:
        k = k ^ torch.tensor(-(2 ** 31), dtype=torch.int32, device=k.device)
    idx = vo.view(torch.int32).to(torch.int64) & 0xFFFFFFFF
    out = {"sorted": bool((k[1:] >= k[:-1]).all().item())}
    out["permutation"] = bool(torch.equal(torch.sort(idx).values, torch.arange(n, device=idx.device)))
    out["values_carry_keys"] = bool(torch.equal(keys_in.view(torch.int32)[idx], ko.view(torch.int32)))
    eq = k[1:] == k[:-1]
    out["stable"] = bool((idx[1:][eq] > idx[:-1][eq]).all().item())
    out["equal_key_pairs_checked"] = int(eq.sum().item())
    return out


def e2e_measure(torch, sorter_factory, n, kb, vb, keys_host, vals_host, steps, warmup, device):
    """Host buffers: per step H2D (keys, values), sort, D2H (sorted keys, values)."""
    kin = torch.empty(n * kb, dtype=torch.uint8, device=device)
    kout = torch.empty_like(kin)
    vin = torch.empty(max(n * vb, 1), dtype=torch.uint8, device=device)
    vout = torch.empty_like(vin)
    ko_h = torch.empty(n * kb, dtype=torch.uint8, pin_memory=True)
    vo_h = torch.empty(max(n * vb, 1), dtype=torch.uint8, pin_memory=True)
    sorter = sorter_factory(kin, kout, vin, vout)

    def step():
        kin.copy_(keys_host, non_blocking=True)
        if vb:
            vin.copy_(vals_host, non_blocking=True)
        sorter()
        ko_h.copy_(kout, non_blocking=True)
        if vb:
            vo_h.copy_(vout, non_blocking=True)

    ms = time_steps(torch, step, steps, warmup)
    return ms / steps, ko_h, vo_h


def e2e_host_call(torch, lib, kid, kb, vb, n, keys_host, vals_host, steps, warmup, device):
    """Host buffers through cusort_sort_pairs_host: one call per step moves the keys and values
    up, sorts and moves them down (all on the current stream)."""
    ko_h = torch.empty(n * kb, dtype=torch.uint8, pin_memory=True)
    vo_h = torch.empty(n * vb, dtype=torch.uint8, pin_memory=True)
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    P = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    nb = C.c_size_t(0)
    args = lambda t: (t, C.byref(nb), kid, P(keys_host), P(ko_h), vb, P(vals_host), P(vo_h), n, 0, 8 * kb, 0,  # noqa
                      stream)
    if lib.cusort_sort_pairs_host(*args(None)) != 0:
        raise RuntimeError("cusort_sort_pairs_host size query failed")
    temp = torch.empty(nb.value, dtype=torch.uint8, device=device)

    def step():
        rc = lib.cusort_sort_pairs_host(*args(C.c_void_p(temp.data_ptr())))
        if rc != 0:
            raise RuntimeError(f"cusort_sort_pairs_host failed: {rc}")

    ms = time_steps(torch, step, steps, warmup)
    del temp
    return ms / steps, ko_h, vo_h


def cpu_baseline(seconds: float, n_full: int):
    """Oracle parallel stable sort of int32/uint32 pairs on all host cores, on the FULL workload
    size (whole sorts repeated until about `seconds` have passed); a one-thread row on a 2^24
    sample beside it."""
    from oracle import oracle as O
    cores = os.cpu_count() or 1
    rng = np.random.default_rng(2)
    m = n_full
    keys = rng.integers(-(2 ** 31), 2 ** 31, size=m, dtype=np.int64).astype(np.int32)
    vals = np.arange(m, dtype=np.uint32)
    reps, t_total = 0, 0.0
    while (t_total < seconds or reps < 2) and reps < 1000:
        t0 = time.perf_counter()
        O.oracle_sort("i32", keys, vals, 0, 32, False, threads=cores)
        t_total += time.perf_counter() - t0
        reps += 1
    rate = reps * m / t_total / 1e9
    # one-thread std::stable_sort on a 2^24 sample, bounded to about a fifth of the time
    m1 = min(m, 1 << 24)
    reps1, t1 = 0, 0.0
    while (t1 < seconds / 5 or reps1 < 1) and reps1 < 100:
        t0 = time.perf_counter()
        O.oracle_sort("i32", keys[:m1], vals[:m1], 0, 32, False, threads=1)
        t1 += time.perf_counter() - t0
        reps1 += 1
    return {"value": rate, "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"{reps} x {m} int32/uint32 pairs (2^{m.bit_length() - 1}, the full workload), "
                      f"__gnu_parallel::stable_sort over {cores} OpenMP threads, {t_total:.1f} s",
            "cpu_model": cpu_model(),
            "single_thread": {"value": reps1 * m1 / t1 / 1e9, "unit": UNIT, "cores": 1,
                              "sample": f"{reps1} x {m1} pairs (2^{m1.bit_length() - 1} sample), "
                                        f"std::stable_sort, {t1:.1f} s"}}


def cpu_model():
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return None


def run_single(args, torch, dist=None, rank=0, world=1):
    device = torch.device("cuda", torch.cuda.current_device())
    n = 1 << args.log2n
    kt, kid, kb, vb = "i32", 5, 4, 4
    keys, vals = make_inputs(torch, n, seed=2, device=device)
    kin = keys.view(torch.uint8)
    vin = vals.view(torch.uint8)
    kout = torch.empty_like(kin)
    vout = torch.empty_like(vin)
    stream = torch.cuda.current_stream().cuda_stream
    sorter = Sorter(args.impl, torch, kt, kid, kb, vb, n, kin, kout, vin, vout, stream)
    smi = ClockSampler(device.index if device.index is not None else 0)
    smi.start()
    # extra untimed spin-up so clocks are settled and sampled
    t_spin = time.time()
    while time.time() - t_spin < 1.0:
        sorter()
        torch.cuda.synchronize()
    t0 = time.time()
    ms = time_steps(torch, sorter, args.steps, args.warmup, dist)
    t1 = time.time()
    clocks = smi.stop(t0 - 0.2, t1 + 0.2)
    ms_step = ms / args.steps
    value = n / (ms_step * 1e-3) / 1e9

    # check of the timed output: sorted, permutation, values carry their keys, stable
    verified = verify_index_pairs(torch, keys, kout, vout)

    out = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int32 keys / uint32 values (integer radix)", "data": "synthetic (seeded uniform int32 keys, "
        "values = index)",
        "config": {"workload": "configs[1]: SortPairs 2^26 int32 keys uniform + uint32 index values", "n": n,
                   "key": "int32", "value_bytes": 4, "api": "in/out pointers (cusort_sort_pairs)",
                   "l2": "inputs 512 MiB > 126 MB L2 (no flush needed)"},
        "verified": verified,
        "clocks": clocks,
    }
    if args.impl == "ours":
        P = 4
        out["gpu_launches"] = args.steps * (2 + P)
        # live per-kernel timing pass (events around each kernel, on the launch stream)
        lib = sorter.lib
        lib.cusort_set_kernel_timing(1)
        acc = {0: [], 1: [], 2: []}
        for _ in range(max(3, min(args.steps, 20))):
            sorter()
            buf = (C.c_float * 16)()
            kinds = (C.c_int * 16)()
            m = lib.cusort_get_kernel_times(buf, kinds, 16)
            for i in range(m):
                acc[kinds[i]].append(buf[i])
        lib.cusort_set_kernel_timing(0)
        os_ms = statistics.mean(acc[2])
        h_ms = statistics.mean(acc[1])
        peak, peak_src = peaks()
        alg = 2 * n * (kb + vb)
        achieved = alg / (os_ms * 1e-3) / 1e9
        traffic = traffic_from_profiles("i32_u32_pairs_2^26")
        out["roofline"] = {"bound": "hbm", "kernel": "onesweep_kernel", "achieved": achieved, "peak": peak,
                           "unit": "GB/s", "frac": achieved / peak, "peak_source": peak_src,
                           "traffic": traffic,
                           "traffic_source": "dram__bytes_read.sum + dram__bytes_write.sum of one onesweep launch "
                                             "from the committed ncu capture (profiles/onesweep_traffic.json), not "
                                             "measured in this run",
                           "algorithmic_bytes_per_launch": alg,
                           "launch_ms": os_ms, "histogram_launch_ms": h_ms,
                           "histogram_gbs": n * kb / (h_ms * 1e-3) / 1e9,
                           "whole_sort_frac": (4 * alg / (ms_step * 1e-3) / 1e9) / peak}
    # e2e through the same C ABI with host buffers
    keys_h = kin.cpu().pin_memory()
    vals_h = vin.cpu().pin_memory()

    def factory(a, b, c, d):
        return Sorter(args.impl, torch, kt, kid, kb, vb, n, a, b, c, d, torch.cuda.current_stream().cuda_stream)

    e2e_steps = max(3, min(args.steps, 10))
    if args.impl == "ours":
        # the library's own host-buffer entry point: copies and sort overlapped inside one call
        e_ms, ko_h, vo_h = e2e_host_call(torch, sorter.lib, kid, kb, vb, n, keys_h, vals_h, e2e_steps, 2, device)
        path = ("cusort_sort_pairs_host (C ABI): pinned host keys + values in, sorted keys + values out; the keys go "
                "up and are sorted with their positions while the values go up, the sorted keys come down while "
                "the values are gathered, then the values come down")
    else:
        e_ms, ko_h, vo_h = e2e_measure(torch, factory, n, kb, vb, keys_h, vals_h, e2e_steps, 2, device)
        path = "pinned host -> H2D -> sort (C ABI) -> D2H -> pinned host"
    same = bool(torch.equal(ko_h[: n * kb], kout.cpu()) and torch.equal(vo_h[: n * vb], vout.cpu()))
    out["e2e"] = {"value": n / (e_ms * 1e-3) / 1e9, "unit": UNIT, "h2d_bytes_per_step": n * (kb + vb),
                  "d2h_bytes_per_step": n * (kb + vb), "ms_per_step": e_ms, "steps": e2e_steps,
                  "path": path, "output_equals_device_sort": same}
    if not args.no_secondary:
        out["secondary"] = secondary(args, torch, device)
        out["secondary"]["double_buffer_api_2^26"] = double_buffer_forms(args, torch, device)
        out["secondary"]["other_configs_2^26"] = other_configs(args, torch, device)
        out["secondary"]["configs[0]_u32_keys_2^20_hot_l2"] = small_hot_l2(args, torch, device)
        out["secondary"]["input_patterns_2^26"] = input_patterns(args, torch, device)
        if args.impl == "ours":
            out["secondary"]["segmented_2^26"] = segmented(args, torch, device)
    if args.impl == "ours" and not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_baseline(args.cpu_seconds, n)
    if args.impl == "reference":
        out["impl"] = "reference"
        out["cpu_baseline"] = {"value": value, "unit": UNIT, "cores": 0, "kind": "reference",
                               "sample": "the reference library has no CPU path: this arm runs the UNMODIFIED "
                                         "libcusort.cuh 1.0.1 built for sm_100a (nvcc 12.9, default build) on the "
                                         "same B200, full workload"}
    return out


def double_buffer_forms(args, torch, device):
    """The DoubleBuffer API form (each library's fastest: no staging buffers) of the two headline
    workloads: 2^26 int32 keys + uint32 index values, and 2^26 uint32 keys-only.  The inputs are
    restored from a pristine copy before every call (outside the timed interval); CUDA events
    bracket each call; 3 warm-up + 10 timed calls.  The pairs output of the last call is checked
    (sorted, permutation, values carry their keys, stable)."""
    n = 1 << args.log2n
    stream = torch.cuda.current_stream().cuda_stream
    res = {}
    keys, vals = make_inputs(torch, n, seed=2, device=device)
    kbuf, vbuf = keys.clone(), vals.clone()
    k_alt, v_alt = torch.empty_like(keys), torch.empty_like(vals)
    s = Sorter(args.impl, torch, "i32", 5, 4, 4, n, kbuf, k_alt, vbuf, v_alt, stream, api="db")

    def restore():
        kbuf.copy_(keys)
        vbuf.copy_(vals)
    ms = time_restored(torch, restore, s, 10, 3)
    ks, vs = s.sel
    res["i32_u32_pairs_2^26"] = {"ms_per_step": round(ms, 4), "gkeys_per_s": round(n / (ms * 1e-3) / 1e9, 2),
                                 "verified": verify_index_pairs(torch, keys, (kbuf, k_alt)[ks], (vbuf, v_alt)[vs])}
    del s, kbuf, vbuf, k_alt, v_alt, vals
    g = torch.Generator(device=device)
    g.manual_seed(1)
    ukeys = torch.randint(0, 256, (n * 4,), dtype=torch.uint8, device=device, generator=g)
    kbuf, k_alt = ukeys.clone(), torch.empty_like(ukeys)
    dummy = torch.empty(1, dtype=torch.uint8, device=device)
    s = Sorter(args.impl, torch, "u32", 4, 4, 0, n, kbuf, k_alt, dummy, dummy, stream, api="db")
    ms = time_restored(torch, lambda: kbuf.copy_(ukeys), s, 10, 3)
    ko = (kbuf, k_alt)[s.sel[0]].view(torch.int32) ^ torch.tensor(-(2 ** 31), dtype=torch.int32, device=device)
    res["u32_keys_only_2^26"] = {"ms_per_step": round(ms, 4), "gkeys_per_s": round(n / (ms * 1e-3) / 1e9, 2),
                                 "sorted": bool((ko[1:] >= ko[:-1]).all().item())}
    return res


def secondary(args, torch, device):
    """u32 keys-only 2^26 (the other single-GPU headline config), same impl."""
    n = 1 << args.log2n
    res = {}
    g = torch.Generator(device=device)
    g.manual_seed(1)
    kin = torch.randint(0, 256, (n * 4,), dtype=torch.uint8, device=device, generator=g)
    kout = torch.empty_like(kin)
    dummy = torch.empty(1, dtype=torch.uint8, device=device)
    s = Sorter(args.impl, torch, "u32", 4, 4, 0, n, kin, kout, dummy, dummy, torch.cuda.current_stream().cuda_stream)
    ms = time_steps(torch, s, max(10, args.steps), 3) / max(10, args.steps)
    res["u32_keys_only_2^26"] = {"ms_per_step": ms, "gkeys_per_s": n / (ms * 1e-3) / 1e9,
                                 "whole_sort_eff_gbs": 4 * 2 * n * 4 / (ms * 1e-3) / 1e9}
    if args.impl == "ours":
        lib = s.lib
        lib.cusort_set_kernel_timing(1)
        v = []
        for _ in range(5):
            s()
            buf = (C.c_float * 16)()
            kinds = (C.c_int * 16)()
            m = lib.cusort_get_kernel_times(buf, kinds, 16)
            v += [buf[i] for i in range(m) if kinds[i] == 2]
        lib.cusort_set_kernel_timing(0)
        res["u32_keys_only_2^26"]["onesweep_launch_ms"] = statistics.mean(v)
        res["u32_keys_only_2^26"]["onesweep_gbs"] = 2 * n * 4 / (statistics.mean(v) * 1e-3) / 1e9
    return res


def small_hot_l2(args, torch, device):
    """2^20 u32 keys-only (seeded uniform), ascending, 4 passes.  The 4 MiB input
    and output stay in the 126 MB L2 between steps, so this is a hot-L2, launch-latency-bound
    figure (not an HBM one): back-to-back sorts, CUDA events around 200 of them.  Ours is timed
    with direct launches and with the cached CUDA graph; the reference's default build (CUDA
    12.9) has direct launches only."""
    n = 1 << 20
    steps = 200
    try:
        g = torch.Generator(device=device)
        g.manual_seed(1)
        kin = torch.randint(0, 256, (n * 4,), dtype=torch.uint8, device=device, generator=g)
        kout = torch.empty_like(kin)
        dummy = torch.empty(1, dtype=torch.uint8, device=device)
        s = Sorter(args.impl, torch, "u32", 4, 4, 0, n, kin, kout, dummy, dummy,
                   torch.cuda.current_stream().cuda_stream)
        res = {"n": n, "l2": "hot (4 MiB input, no flush)", "bound": "launch latency"}
        modes = [("direct", 0), ("graph", 1)] if args.impl == "ours" else [("direct", None)]
        for name, mode in modes:
            if mode is not None:
                s.lib.cusort_set_launch_mode(mode)
            ms = time_steps(torch, s, steps, 10) / steps
            res[name] = {"us_per_sort": round(ms * 1e3, 2), "gkeys_per_s": round(n / (ms * 1e-3) / 1e9, 2)}
        if args.impl == "ours":
            s.lib.cusort_set_launch_mode(0)
        ko = kout.view(torch.int32).to(torch.int64) & 0xFFFFFFFF
        res["sorted"] = bool((ko[1:] >= ko[:-1]).all().item())
        return res
    except Exception as e:  # the headline line must not depend on this informational leg
        if args.impl == "ours":
            from libcusort_b200 import _capi
            _capi.load().cusort_set_launch_mode(0)
        return {"error": f"{type(e).__name__}: {e}"}


def seg_call(torch, keys, vals, kout, vout, seglen, stream):
    """Segmented SortPairs (int32 keys, uint32 values) over equal-length segments of `seglen`
    items (the last one shorter) through cusort_segmented_sort_pairs; returns the sort callable."""
    from libcusort_b200 import _capi
    lib = _capi.load()
    n = keys.numel()
    S = (n + seglen - 1) // seglen
    b = torch.arange(S, dtype=torch.int64, device=keys.device) * seglen
    e = torch.clamp(b + seglen, max=n)
    P = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    nb = C.c_size_t(0)
    s = C.c_void_p(stream)
    args = lambda t: (t, C.byref(nb), 5, P(keys), P(kout), 4, P(vals), P(vout), n, S, P(b), P(e), 0, 32, 0, s)  # noqa: E731
    if lib.cusort_segmented_sort_pairs(*args(None)) != 0:
        raise RuntimeError("segmented size query failed")
    temp = torch.empty(max(nb.value, 1), dtype=torch.uint8, device=keys.device)

    def call():
        if lib.cusort_segmented_sort_pairs(*args(P(temp))) != 0:
            raise RuntimeError("segmented sort failed")
    call.keep = (b, e, temp)
    call.segments = S
    return call


def composite_baselines(torch, keys, vals, kout_seg, vout_seg, seglen, stream):
    """ms per sort of the segmented problem as ONE stable sort of (segment << 32 | twiddled key):
    torch.sort(stable=True), and this library's uint64 SortPairs over bits [0, 32 + segment
    bits); both checked equal to the segmented sort's output (kout_seg / vout_seg)."""
    n = keys.numel()
    segbits = max(1, int((n - 1) // seglen).bit_length())
    seg = torch.arange(n, dtype=torch.int64, device=keys.device) // seglen
    out = {}

    def composite():
        return (seg << 32) | ((keys.to(torch.int64) + 2 ** 31) & 0xFFFFFFFF)

    def torch_way():
        c = composite()
        r = torch.sort(c, stable=True)
        return r.values, vals[r.indices]
    ms = time_steps(torch, torch_way, 5, 2) / 5
    _, tv = torch_way()
    out["torch_sort_stable"] = {"ms": round(ms, 4), "same_values": bool(torch.equal(tv, vout_seg))}
    ck = composite()
    ck_out = torch.empty_like(ck)
    vin, v_out = vals.clone(), torch.empty_like(vals)
    s = Sorter("ours", torch, "u64", 6, 8, 4, n, ck, ck_out, vin, v_out, stream, begin_bit=0, end_bit=32 + segbits)

    def ours_way():
        ck.copy_(composite())
        s()
    ms = time_steps(torch, ours_way, 5, 2) / 5
    out["cusort_u64_pairs"] = {"ms": round(ms, 4), "bits": 32 + segbits, "same_values": bool(torch.equal(v_out, vout_seg))}
    del seg, ck, ck_out, vin, v_out, s
    return out


def segmented(args, torch, device):
    """Segmented sort (CUB DeviceSegmentedRadixSort semantics; the reference has none) of 2^26
    int32 keys + uint32 index values in equal-length segments, one entry per length class: the
    warp all-pairs class (16), the warp and CTA shared-memory classes (1000, 4000) and the
    segmented onesweep (2^20).  3 warm-up + 10 timed sorts each; inputs > L2.  The first and
    last segment of each timed output are checked against torch's stable sort.

    Beside each, the same result through one stable sort of a composite 64-bit key (segment
    index in the bits above the 32 key bits; what a caller without a segmented sort would do),
    timed including the kernel that builds the composite key: with torch.sort(stable=True)
    (torch's own GPU sort) and with this library's 64-bit SortPairs over only the bits in use."""
    n = 1 << args.log2n
    res = {}
    try:
        g = torch.Generator(device=device)
        g.manual_seed(1)
        keys = torch.randint(-(2 ** 31), 2 ** 31, (n,), dtype=torch.int64, device=device, generator=g).to(torch.int32)
        vals = torch.arange(n, dtype=torch.int32, device=device)
        kout, vout = torch.empty_like(keys), torch.empty_like(vals)
        stream = torch.cuda.current_stream().cuda_stream
        for seglen in (16, 1000, 4000, 1 << 20):
            call = seg_call(torch, keys, vals, kout, vout, seglen, stream)
            ms = time_steps(torch, call, 10, 3) / 10
            ok = True
            for i in (0, call.segments - 1):
                a0, a1 = i * seglen, min(n, (i + 1) * seglen)
                ref = torch.sort(keys[a0:a1], stable=True)
                ok &= bool(torch.equal(ref.values, kout[a0:a1])) and bool(torch.equal(vals[a0:a1][ref.indices],
                                                                                       vout[a0:a1]))
            res[f"seglen_{seglen}"] = {"segments": call.segments, "ms_per_step": round(ms, 4),
                                       "gkeys_per_s": round(n / (ms * 1e-3) / 1e9, 2), "checked": ok}
            res[f"seglen_{seglen}"]["composite_key_baselines_ms"] = composite_baselines(
                torch, keys, vals, kout, vout, seglen, stream)
        return res
    except Exception as e:  # informational leg: keep the headline line
        res["error"] = f"{type(e).__name__}: {e}"
        return res


def other_configs(args, torch, device):
    """The other BASELINE.json single-GPU configs at 2^26, same impl and API (in/out pointers),
    seeded synthetic data with the configs' shapes and distributions: configs[1]'s low-entropy
    variant, configs[2]'s keys-only dtype sweep (ascending and descending), configs[3]'s double
    keys + 16-byte values and 20-bit Zipf keys.  Time per sort (CUDA events, 3 warm-up + 10)."""
    n = 1 << args.log2n
    g = torch.Generator(device=device)
    g.manual_seed(7)
    stream = torch.cuda.current_stream().cuda_stream
    dummy = torch.empty(1, dtype=torch.uint8, device=device)
    res = {}

    def words(bits):
        lo, hi = (-(2 ** (bits - 1)), 2 ** (bits - 1)) if bits < 64 else (-(2 ** 63), 2 ** 63 - 1)
        return torch.randint(lo, hi, (n,), dtype=torch.int64, device=device, generator=g)

    def normal_specials(dtype, sigma):
        x = torch.randn(n, dtype=dtype, device=device, generator=g) * sigma
        idx = torch.randperm(n, device=device, generator=g)[: 5 * (n // 1000)].view(5, -1)
        for row, v in zip(idx, (-0.0, 0.0, float("inf"), float("-inf"), float("nan"))):
            x[row] = v
        return x

    def run(name, kt, kid, kb, keys, vals=None, vb=0, desc=False, begin=0, end=None):
        kin = keys.contiguous().view(torch.uint8)
        kout = torch.empty_like(kin)
        vin = vals.contiguous().view(torch.uint8) if vb else dummy
        vout = torch.empty_like(vin) if vb else dummy
        srt = Sorter(args.impl, torch, kt, kid, kb, vb, n, kin, kout, vin, vout, stream, desc, begin, end)
        ms = time_steps(torch, srt, 10, 3) / 10
        res[name] = {"ms_per_step": round(ms, 4), "gkeys_per_s": round(n / (ms * 1e-3) / 1e9, 2)}
        del srt, kin, kout

    a, b, c = words(32), words(32), words(32)
    run("configs[1]_low_entropy_i32_u32_pairs", "i32", 5, 4, (a & b & c).to(torch.int32),
        torch.arange(n, dtype=torch.int32, device=device), 4)
    del a, b, c
    for kt, kid, kb in (("i8", 1, 1), ("i16", 3, 2), ("i32", 5, 4), ("i64", 7, 8)):
        w = words(8 * kb)
        keys = w.to({1: torch.int8, 2: torch.int16, 4: torch.int32, 8: torch.int64}[kb])
        for desc in (False, True):
            run(f"configs[2]_{kt}_keys_{'desc' if desc else 'asc'}", kt, kid, kb, keys, desc=desc)
    for kt, kid, kb, dt in (("f32", 8, 4, torch.float32), ("f64", 9, 8, torch.float64)):
        keys = normal_specials(dt, 1e3)
        for desc in (False, True):
            run(f"configs[2]_{kt}_keys_{'desc' if desc else 'asc'}", kt, kid, kb, keys, desc=desc)
    keys = torch.randn(n, dtype=torch.float64, device=device, generator=g)
    idx = torch.arange(n, dtype=torch.int64, device=device)
    vals = torch.stack([idx, ~idx], dim=1)  # ulonglong2 (index, ~index)
    run("configs[3]_f64_keys_16B_values", "f64", 9, 8, keys, vals, 16)
    del vals, idx
    table = words(32).to(torch.int32)[:65536]
    ranks = torch.arange(1, 65537, dtype=torch.float64, device=device)
    draws = torch.multinomial((ranks ** -1.1).float(), n, replacement=True, generator=g)
    run("configs[3]_u32_keys_bits_0_20_zipf_u32_values", "u32", 4, 4, table[draws],
        torch.arange(n, dtype=torch.int32, device=device), 4, begin=0, end=20)
    return res


def input_patterns(args, torch, device):
    """int32 keys-only and int32 + uint32 index pairs at 2^26 in orders and cardinalities a
    uniform bench does not show, same impl and API (in/out pointers): already sorted (keys =
    63 i), sorted with runs of 1024 equal keys (i >> 10), reverse sorted, all keys equal, 16
    distinct values in random order.  Time per sort
    (CUDA events, 3 warm-up + 10)."""
    n = 1 << args.log2n
    g = torch.Generator(device=device)
    g.manual_seed(12)
    stream = torch.cuda.current_stream().cuda_stream
    i = torch.arange(n, dtype=torch.int64, device=device)
    vals = i.to(torch.int32).view(torch.uint8)
    dummy = torch.empty(1, dtype=torch.uint8, device=device)
    pats = {
        "sorted": lambda: (i * 63).to(torch.int32),
        "sorted_runs_of_1024_equal": lambda: (i >> 10).to(torch.int32),
        "reverse_sorted": lambda: ((n - i) * 63).to(torch.int32),
        "all_equal": lambda: torch.full((n,), 123456789, dtype=torch.int32, device=device),
        "16_distinct_values": lambda: (torch.randint(0, 16, (n,), device=device, generator=g) * 0x10204081).to(
            torch.int32),
    }
    res = {}
    for name, make in pats.items():
        kin = make().contiguous().view(torch.uint8)
        kout = torch.empty_like(kin)
        for vb in (0, 4):
            vout = torch.empty_like(vals) if vb else dummy
            srt = Sorter(args.impl, torch, "i32", 5, 4, vb, n, kin, kout, vals if vb else dummy, vout, stream)
            ms = time_steps(torch, srt, 10, 3) / 10
            res[f"{name}_{'i32_u32_pairs' if vb else 'i32_keys'}"] = {"ms_per_step": round(ms, 4),
                                                                     "gkeys_per_s": round(n / (ms * 1e-3) / 1e9, 2)}
            del srt, vout
        del kin, kout
    return res


def profile_case(args, torch):
    """Plain sorts of one case, nothing else (the command that ncu captures)."""
    device = torch.device("cuda", 0)
    n = 1 << args.log2n
    if args.profile_case == "u16_keys":  # one 16-bit digit: hist16 + fill16
        g = torch.Generator(device=device)
        g.manual_seed(1)
        kin = torch.randint(0, 256, (n * 2,), dtype=torch.uint8, device=device, generator=g)
        kout = torch.empty_like(kin)
        dummy = torch.empty(1, dtype=torch.uint8, device=device)
        s = Sorter(args.impl, torch, "u16", 2, 2, 0, n, kin, kout, dummy, dummy,
                   torch.cuda.current_stream().cuda_stream)
    elif args.profile_case == "seg_i32_u32_pairs_1000":  # segmented, 1000-item segments (CTA class)
        keys, vals = make_inputs(torch, n, seed=1, device=device)
        kout, vout = torch.empty_like(keys), torch.empty_like(vals)
        s = seg_call(torch, keys, vals, kout, vout, 1000, torch.cuda.current_stream().cuda_stream)
    if args.profile_case in ("u16_keys", "seg_i32_u32_pairs_1000"):
        for _ in range(args.warmup + args.steps):
            s()
        torch.cuda.synchronize()
        print(json.dumps({"profile_case": args.profile_case, "n": n, "impl": args.impl,
                          "sorts": args.warmup + args.steps}))
        return
    if args.profile_case == "u32_keys":
        kt, kid, kb, vb = "u32", 4, 4, 0
    else:
        kt, kid, kb, vb = "i32", 5, 4, 4
    keys, vals = make_inputs(torch, n, seed=2, device=device)
    if args.profile_case == "i32_u32_pairs_lowent":  # configs[1]'s low-entropy keys: a & b & c
        b, c = make_inputs(torch, n, seed=3, device=device)[0], make_inputs(torch, n, seed=4, device=device)[0]
        keys = keys & b & c
        del b, c
    kin, vin = keys.view(torch.uint8), vals.view(torch.uint8)
    kout, vout = torch.empty_like(kin), torch.empty_like(vin)
    s = Sorter(args.impl, torch, kt, kid, kb, vb, n, kin, kout, vin, vout, torch.cuda.current_stream().cuda_stream)
    for _ in range(args.warmup + args.steps):
        s()
    torch.cuda.synchronize()
    print(json.dumps({"profile_case": args.profile_case, "n": n, "impl": args.impl, "sorts": args.warmup + args.steps}))


def lookback_stall(args, torch):
    """Share of the onesweep time spent in the decoupled lookback, from a library built with
    CUSORT_NVCC_DEFINES=-DCUSORT_LOOKBACK_TIMER=1: after one sort the control block holds, summed
    over every tile of every pass, the longest time any digit-owning thread of the tile spent in
    the lookback (ns), the descriptor-window rounds of all digit threads, the tile count and the
    rounds that re-polled a predecessor with nothing published.  frac = that time / (onesweep
    CTAs x the passes' summed launch time): the share of each CTA's time its digit-owning warps
    were held by the lookback (the other warps reorder meanwhile)."""
    device = torch.device("cuda", 0)
    n = 1 << args.log2n
    out = {"lookback_stall": True, "n": n}
    from libcusort_b200 import _capi
    lib = _capi.load()
    for name, kt, kid, vb in (("i32_u32_pairs", "i32", 5, 4), ("u32_keys", "u32", 4, 0)):
        keys, vals = make_inputs(torch, n, seed=2, device=device)
        kin, vin = keys.view(torch.uint8), vals.view(torch.uint8)
        kout, vout = torch.empty_like(kin), torch.empty_like(vin)
        s = Sorter("ours", torch, kt, kid, 4, vb, n, kin, kout, vin, vout, torch.cuda.current_stream().cuda_stream)
        for _ in range(3):
            s()
        lib.cusort_set_kernel_timing(1)
        s()
        buf, kinds = (C.c_float * 16)(), (C.c_int * 16)()
        m = lib.cusort_get_kernel_times(buf, kinds, 16)
        lib.cusort_set_kernel_timing(0)
        os_ms = sum(buf[i] for i in range(m) if kinds[i] == 2)
        torch.cuda.synchronize()
        w = s.temp[128:160].view(torch.int64).tolist()
        if w[2] == 0:
            out[name] = {"error": "no timer words: the library was not built with CUSORT_LOOKBACK_TIMER=1"}
            continue
        grid = C.c_int(0)
        lib.cusort_query_plan(kid, vb, n, 0, 32, None, None, C.byref(grid), None, None)
        out[name] = {"onesweep_ms_4_passes": os_ms, "ctas": grid.value, "tiles": w[2],
                     "lookback_ns_per_tile": w[0] / w[2], "frac": w[0] / grid.value / (os_ms * 1e6),
                     "rounds_per_digit_tile": w[1] / w[2] / 256, "empty_round_share": w[3] / max(w[1], 1)}
    print(json.dumps(out))


def main():
    args = parse()
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if world > 1 or args.gpus > 1:
        if args.impl == "reference":
            # The reference has no multi-GPU mode: rank 0 runs its single-GPU bench, the others exit.
            if rank != 0:
                return
            torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
            from oracle import oracle as O
            if not O.ref_available():
                print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libcusort_ref.so was not built"}))
                return
            out = run_single(args, torch)
            out["note"] = "reference is single-GPU only: rank 0 ran the N=1 workload, other ranks idle"
            print(json.dumps(out))
            return
        from libcusort_b200 import mgpu_bench
        out = mgpu_bench.run(args, torch)
        if out is not None and rank == 0:
            print(json.dumps(out))
        return
    if not torch.cuda.is_available():
        print(json.dumps({"error": "no CUDA device"}))
        sys.exit(1)
    if args.impl == "reference":
        from oracle import oracle as O
        if not O.ref_available():
            print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libcusort_ref.so was not built "
                                                                  "(needs the reference checkout at build time)"}))
            return
    torch.cuda.set_device(0)
    if args.lookback_stall:
        lookback_stall(args, torch)
        return
    if args.profile_case:
        profile_case(args, torch)
        return
    out = run_single(args, torch)
    print(json.dumps(out))


if __name__ == "__main__":
    main()
