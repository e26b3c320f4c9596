"""Benchmark of the B200 onesweep radix sort (the headline of the metric
"Onesweep sort Gkeys/s; scan/reduce HBM GB/s"), with scan, reduce and
segment-reduce lines attached.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (one "step"): DeviceRadixSort::SortPairs of n = 2^28 uint32 keys
uniform over 2^32 with uint32 values = iota, per GPU.
Inputs (2 GiB per step) are larger than L2 (126 MB), so no L2 flush is needed
between sort steps; the reduce line (64 MiB input) flushes L2 between
iterations.  Data: seeded PCG32 synthetic inputs.

Under torchrun (N > 1) every rank sorts its own 2^28-pair shard (weak
scaling); timings are the max over ranks.

--impl reference times the reference algorithm's CPU path: the reference
(LuisaCompute DSL kernels) cannot be built or run here, so this is the CPU
restatement in oracle/ (multi-threaded LSD radix sort) on the host cores.
"""
from __future__ import annotations

import argparse
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

N_SORT = 1 << 28
METRIC = "Onesweep sort Gkeys/s; scan/reduce HBM GB/s (% of ~8 TB/s) at 1/2/4/8 B200"
UNIT = "Gkeys/s"
# DRAM bytes per pair per onesweep launch from the committed ncu capture
# (profiles/), or None before one exists.
TRAFFIC_PER_PAIR_PASS = 4.27e9 / 2**28  # DRAM bytes per pair per pass, 2^28 capture in profiles/sort_pairs_u32_2p28_launches.md


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# ---------------------------------------------------------------------------
class ClockSampler:
    """Samples nvidia-smi SM clocks and throttle reasons while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self.thread = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", str(self.gpu)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        time.sleep(0.25)
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            time.sleep(0.15)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        return False

    def summary(self):
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = max(mx, float(parts[2]))
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


def physical_gpu(local_rank: int) -> int:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [v.strip() for v in vis.split(",") if v.strip()]
        if local_rank < len(ids) and ids[local_rank].isdigit():
            return int(ids[local_rank])
    return local_rank


# ---------------------------------------------------------------------------
def run_reference_arm(args, rank, world):
    """CPU path of the reference algorithm on the host cores (rank 0 only)."""
    if rank != 0:
        return 0
    import oracle  # the reference algorithm's CPU restatement; nothing of the package is loaded here

    cores = os.cpu_count() or 1
    sample = 1 << 24  # bounded sample of the 2^28-pair workload per step
    rng = np.random.Generator(np.random.PCG64(1))
    keys = rng.integers(0, 1 << 32, size=sample, dtype=np.uint64).astype(np.uint32)  # uniform over 2^32
    vals = np.arange(sample, dtype=np.uint32)
    for _ in range(max(args.warmup, 1)):
        oracle.radix_sort(keys, vals, threads=cores)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        oracle.radix_sort(keys, vals, threads=cores)
        times.append(time.perf_counter() - t0)
    sec = sum(times) / len(times)
    value = sample / sec / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "u32", "data": "synthetic (numpy PCG64 seeded)",
        "config": {"workload": "SortPairs u32 keys (uniform 2^32) + u32 iota values, BASELINE config 3",
                   "n_per_step": sample, "note": "reference CPU path = oracle/ LSD radix sort restatement "
                   "(LuisaCompute, the reference's runtime, is absent: reference not buildable); the rate is "
                   "per pair over a 2^24-pair sample of the 2^28-pair step (numpy PCG64 inputs, same distribution)"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": f"{sample} pairs per step (bounded sample of 2^28)"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-extras", action="store_true", help="skip the scan/reduce/segment lines")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer end-to-end timing")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline")
    ap.add_argument("--n-log2", type=int, default=28, help="pairs per GPU = 2^n (profiling runs use less)")
    ap.add_argument("--no-mg", action="store_true", help="skip the config-5 multi-GPU lines")
    ap.add_argument("--mg-scale", type=int, default=0, help="shrink the config-5 inputs by 2^k (tests)")
    ap.add_argument("--extras-scale", type=int, default=0,
                    help="shrink the scan/reduce/segment inputs by 2^k (profiling runs)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        return run_reference_arm(args, rank, world)

    import torch

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", device_id=dev)

    import oracle  # checker and CPU baseline only
    from lc_parallel_primitive_b200 import _lib as L
    from lc_parallel_primitive_b200 import datagen as G
    from lc_parallel_primitive_b200.primitives import CommandList, DeviceRadixSort, Stream, synchronize

    lib = L.lib()
    peak, peak_kind = load_peaks()
    stream = torch.cuda.current_stream()
    sh = stream.cuda_stream

    # ---- inputs (host, pinned) ------------------------------------------------
    n = 1 << args.n_log2
    keys_np = G.u32(n, seed=1 + rank, stream=7)
    h_keys = torch.from_numpy(keys_np.view(np.int32)).pin_memory()
    # values = global input index (shard r holds elements r*n .. r*n+n-1)
    h_vals = torch.from_numpy(G.iota_u32(n, start=(rank * n) & 0xFFFFFFFF).view(np.int32)).pin_memory()
    h_keys_out = torch.empty_like(h_keys).pin_memory()
    h_vals_out = torch.empty_like(h_vals).pin_memory()
    d_keys = h_keys.to(dev)
    d_vals = h_vals.to(dev)
    d_keys_out = torch.empty_like(d_keys)
    d_vals_out = torch.empty_like(d_vals)
    tb = lib.lcpp_radix_sort_temp_bytes(L.U32, L.U32, n)
    d_temp = torch.empty(tb, dtype=torch.uint8, device=dev)

    mg_state = {}
    if world > 1:  # global sort through the multi-GPU C ABI, buffers allocated once
        from lc_parallel_primitive_b200 import multi_gpu as M

        comm = M.comm_for()
        mg_nranks = comm.nranks  # ranks of the library's NCCL communicator (ncclCommCount)
        cap = M.default_capacity(n)
        mg_ko = torch.empty(cap, dtype=torch.uint32, device=dev)
        mg_vo = torch.empty(cap, dtype=torch.uint32, device=dev)
        del d_temp
        d_temp = torch.empty(M.mg_sort_temp_bytes(d_keys.view(torch.uint32), d_vals.view(torch.uint32), cap, world),
                             dtype=torch.uint8, device=dev)

    def sort_once():
        if world == 1:
            L.check(lib.lcpp_radix_sort(L.U32, L.U32, 0, d_keys.data_ptr(), d_keys_out.data_ptr(),
                                        d_vals.data_ptr(), d_vals_out.data_ptr(), n, 0, 0, d_temp.data_ptr(), tb,
                                        sh), "sort")
        else:  # sampled splitters, partition pass, NCCL exchange, local sort
            mg_state["res"] = M.mg_sort_pairs(d_keys.view(torch.uint32), d_vals.view(torch.uint32), comm=comm,
                                              capacity=cap, temp=d_temp, keys_out=mg_ko, vals_out=mg_vo)

    for _ in range(args.warmup):
        sort_once()
    torch.cuda.synchronize()
    L.check(lib.lcpp_last_device_error(sh), "device error")

    # correctness of what is timed (size-independent properties on the device)
    if world == 1:
        k = d_keys_out.view(torch.int32) ^ torch.tensor(-(1 << 31), dtype=torch.int32, device=dev)
        assert bool((k[1:] >= k[:-1]).all()), "sort output not ordered"
        perm_keys = d_keys.view(torch.int32)[d_vals_out.view(torch.int32).long()]
        assert bool((perm_keys == d_keys_out.view(torch.int32)).all()), "values do not follow keys"
        del k, perm_keys
    else:
        r = mg_state["res"]
        k = r.keys.view(torch.int32).to(torch.int64) & 0xFFFFFFFF
        assert bool((k[1:] >= k[:-1]).all()), "rank slice not ordered"
        ends = torch.tensor([k[0].item() if k.numel() else -1, k[-1].item() if k.numel() else -1],
                            dtype=torch.int64, device=dev)
        allends = [torch.empty_like(ends) for _ in range(world)]
        torch.distributed.all_gather(allends, ends)
        e = torch.stack(allends).cpu().tolist()
        assert all(e[i][1] <= e[i + 1][0] for i in range(world - 1) if e[i][1] >= 0 and e[i + 1][0] >= 0)
        cnt = torch.tensor([r.n], dtype=torch.int64, device=dev)
        torch.distributed.all_reduce(cnt)
        assert int(cnt.item()) == world * n
        del k
        mg_state.clear()
    torch.cuda.empty_cache()
    sort_once()  # re-populate the allocator cache after the checks (untimed)
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return float(t.item())

    # ---- timed region: device-resident sort ---------------------------------
    launches0 = lib.lcpp_kernel_launch_count()
    lib.lcpp_profile_enable(1)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(physical_gpu(local_rank)) as clocks:
        barrier()
        torch.cuda.synchronize()
        start.record(stream)
        for _ in range(args.steps):
            sort_once()
        stop.record(stream)
        torch.cuda.synchronize()
        barrier()
    ms = start.elapsed_time(stop) / args.steps
    launches = lib.lcpp_kernel_launch_count() - launches0
    prof = {}
    for kname in ("rs_memset", "rs_histogram", "rs_bins_scan", "rs_onesweep"):
        c, t = L.C.c_uint64(0), L.C.c_double(0)
        lib.lcpp_profile_read(kname.encode(), L.C.byref(c), L.C.byref(t))
        prof[kname] = (int(c.value), float(t.value))
    lib.lcpp_profile_enable(0)
    ms = max_over_ranks(ms)
    value = world * n / (ms * 1e-3) / 1e9

    os_launches, os_ms = prof["rs_onesweep"]
    os_avg_ms = os_ms / max(os_launches, 1)
    os_bytes = 16 * n  # per pass: read key+value, write key+value (4 B each)
    os_achieved = os_bytes / (os_avg_ms * 1e-3) / 1e9
    hist_avg_ms = prof["rs_histogram"][1] / max(prof["rs_histogram"][0], 1)

    # ---- e2e through the public API with host buffers ---------------------------
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(torch, stream, n, world, h_keys, h_vals, h_keys_out, h_vals_out, d_keys, d_vals,
                      d_keys_out, d_vals_out, d_temp, args, barrier, max_over_ranks,
                      mg_sort=(lambda: (sort_once(), mg_state["res"])[1]) if world > 1 else None)

    # ---- CPU baseline (rank 0, N = 1 only) ------------------------------------
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cores = os.cpu_count() or 1
        sample = min(1 << 24, n)
        ks, vs = keys_np[:sample].copy(), np.arange(sample, dtype=np.uint32)
        oracle.radix_sort(ks, vs, threads=cores)
        reps, t0 = 3, time.perf_counter()
        for _ in range(reps):
            oracle.radix_sort(ks, vs, threads=cores)
        sec = (time.perf_counter() - t0) / reps
        cpu = {"value": sample / sec / 1e9, "unit": UNIT, "cores": cores, "kind": "port",
               "sample": f"{sample} of the 2^28 pairs, LSD radix sort (oracle/), {reps} reps"}

    extras = {}
    if not args.no_extras:
        del h_keys_out, h_vals_out
        extras = run_extras(torch, dev, lib, L, G, peak, rank, world, max_over_ranks, barrier, args.extras_scale)
    if not args.no_mg:
        del d_keys, d_vals, d_keys_out, d_vals_out, d_temp, mg_state
        torch.cuda.empty_cache()
        extras.update(run_mg_extras(torch, dev, lib, L, peak, rank, world, max_over_ranks, barrier, args.mg_scale))

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "u32", "data": "synthetic (PCG32 seeded, uniform u32 keys, iota values)",
            "config": {"workload": f"DeviceRadixSort::SortPairs, n=2^{args.n_log2} u32 keys + u32 values per GPU (BASELINE config 3)"
                       + ("" if world == 1 else "; global sort over all GPUs (lcpp_mg_sort: sampled extended-key splitters, one onesweep partition pass, NCCL send/recv exchange, local onesweep sort)"),
                       "n_per_gpu": n, "parallelism": f"global sort x{world} (NCCL point-to-point exchange in lcpp_mg_sort)" if world > 1 else "single GPU",
                       "l2": "inputs 2 GiB per step > 126 MB L2 (no flush needed)",
                       "algorithmic_bytes_per_pair": 68},
            "roofline": {"bound": "hbm", "kernel": "rs_onesweep_kernel (one 8-bit pass)",
                         "achieved": os_achieved, "peak": peak, "unit": "GB/s", "frac": os_achieved / peak,
                         "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else "fallback",
                         "traffic": TRAFFIC_PER_PAIR_PASS * n if TRAFFIC_PER_PAIR_PASS else None,
                         "traffic_source": "ncu dram__bytes_read+write of one onesweep launch at 2^28 pairs "
                                           "(profiles/sort_pairs_u32_2p28_launches.md), 15.9 B per pair; scaled "
                                           "by the pair count when n differs",
                         "avg_launch_ms": os_avg_ms, "bytes_per_launch": os_bytes,
                         "whole_sort_frac": (68 * n / (ms * 1e-3) / 1e9) / peak},
            "kernels": {k: {"launches": c, "total_ms": t} for k, (c, t) in prof.items()},
            "histogram_avg_ms": hist_avg_ms,
            "e2e": e2e,
            "gpu_launches": int(launches),
            "comm_nranks": (mg_nranks if world > 1 else 1),
            "clocks": clocks.summary(),
            "cpu_baseline": cpu,
            "extras": extras,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()
    return 0


def run_e2e(torch, stream, n, world, h_keys, h_vals, h_keys_out, h_vals_out, d_keys, d_vals, d_keys_out,
            d_vals_out, d_temp, args, barrier, max_over_ranks, mg_sort=None):
    """Same metric through the public API (DeviceRadixSort.SortPairs recorded
    into a CommandList and committed to a Stream), with every step's inputs
    copied from pinned host memory and its sorted pairs copied back.  The
    copies run on their own streams and overlap neighbouring steps (inputs of
    step k+1 and results of step k-1 move while step k sorts), as a streaming
    caller would run it; the time is first upload start to last download end."""
    from lc_parallel_primitive_b200.primitives import CommandList, DeviceRadixSort, Stream, synchronize

    sorter = DeviceRadixSort()
    sorter.create(None)
    # a streaming caller runs many steps: 16 keep the pipeline's fill and drain
    # (first upload, last sort and download) small against the steady state
    e2e_steps = max(3, min(16, args.steps))
    if world > 1:  # the multi-GPU entry point; this rank's slice of the result comes back
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        torch.cuda.synchronize()
        e0.record(stream)
        d2h = 0
        for _ in range(e2e_steps):
            d_keys.copy_(h_keys, non_blocking=True)
            d_vals.copy_(h_vals, non_blocking=True)
            r = mg_sort()
            m = min(r.keys.numel(), h_keys_out.numel())
            h_keys_out[:m].copy_(r.keys.view(torch.int32)[:m], non_blocking=True)
            h_vals_out[:m].copy_(r.values.view(torch.int32)[:m], non_blocking=True)
            d2h = 8 * r.keys.numel()
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
        e2e_ms = max_over_ranks(e0.elapsed_time(e1) / e2e_steps)
        return {"value": world * n / (e2e_ms * 1e-3) / 1e9, "unit": UNIT, "h2d_bytes_per_step": 8 * n,
                "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms, "api": "multi_gpu.mg_sort_pairs (lcpp_mg_sort)",
                "steps": e2e_steps}

    dev = d_keys.device
    up, down, comp = torch.cuda.Stream(dev), torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    api_stream = Stream(comp)
    kin = [d_keys, torch.empty_like(d_keys)]
    vin = [d_vals, torch.empty_like(d_vals)]
    kout = [d_keys_out, torch.empty_like(d_keys_out)]
    vout = [d_vals_out, torch.empty_like(d_vals_out)]
    ev = lambda: torch.cuda.Event(enable_timing=False)
    loaded, sorted_, fetched = [ev(), ev()], [ev(), ev()], [ev(), ev()]
    cmd = CommandList()
    sorter.SortPairs(cmd, d_temp, kin[0], kout[0], vin[0], vout[0], n)  # warm the path
    api_stream << cmd.commit() << synchronize()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(up)
    comp.wait_event(e0)
    down.wait_event(e0)
    for k in range(e2e_steps):
        b = k & 1
        if k >= 2:
            up.wait_event(sorted_[b])      # step k-2 has finished reading this input buffer
        with torch.cuda.stream(up):
            kin[b].copy_(h_keys, non_blocking=True)
            vin[b].copy_(h_vals, non_blocking=True)
        loaded[b].record(up)
        comp.wait_event(loaded[b])
        if k >= 2:
            comp.wait_event(fetched[b])    # step k-2's results have left this output buffer
        cmd = CommandList()
        sorter.SortPairs(cmd, d_temp, kin[b], kout[b], vin[b], vout[b], n)
        api_stream << cmd.commit()
        sorted_[b].record(comp)
        down.wait_event(sorted_[b])
        with torch.cuda.stream(down):
            h_keys_out.copy_(kout[b], non_blocking=True)
            h_vals_out.copy_(vout[b], non_blocking=True)
        fetched[b].record(down)
    e1.record(down)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / e2e_steps
    assert np.array_equal(h_vals_out[:1000].numpy(), vout[(e2e_steps - 1) & 1][:1000].cpu().numpy())
    del kin[1], vin[1], kout[1], vout[1]
    return {"value": n / (e2e_ms * 1e-3) / 1e9, "unit": UNIT, "h2d_bytes_per_step": 8 * n,
            "d2h_bytes_per_step": 8 * n, "ms_per_step": e2e_ms,
            "api": "DeviceRadixSort.SortPairs via CommandList/Stream; uploads, sorts and downloads on three "
                   "streams overlapping neighbouring steps",
            "steps": e2e_steps}


def run_extras(torch, dev, lib, L, G, peak, rank, world, max_over_ranks, barrier, shrink=0):
    """Scan (config 2), reduce (config 1), segment reduce (config 4), scan-by-key
    and reduce-by-key, each timed with CUDA events; GB/s from algorithmic bytes."""
    stream = torch.cuda.current_stream()
    sh = stream.cuda_stream
    out = {}
    # L2 flush between timed iterations: write a 256 MiB buffer (> 126 MB L2), then read
    # another one so the dirty lines are written back before the timed region starts.
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    flush_rd = torch.ones(64 << 20, dtype=torch.float32, device=dev)

    def timeit(fn, iters, flush_l2=False):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        tot = 0.0
        for _ in range(iters):
            if flush_l2:
                flush.zero_()
                flush_rd.sum()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            fn()
            b.record(stream)
            torch.cuda.synchronize()
            tot += a.elapsed_time(b)
        return max_over_ranks(tot / iters)

    # scan: 2^28 u32 exclusive, 2^28 f32 inclusive
    n = 1 << (28 - shrink)
    x = torch.from_numpy(G.u32_below(n, 16, seed=1, stream=5).view(np.int32)).to(dev)
    y = torch.empty_like(x)
    tb = lib.lcpp_scan_temp_bytes(L.U32, n)
    t = torch.empty(tb, dtype=torch.uint8, device=dev)
    ms = timeit(lambda: L.check(lib.lcpp_scan(0, L.U32, x.data_ptr(), y.data_ptr(), n, t.data_ptr(), tb, sh)), 20)
    out[f"scan_exclusive_u32_2p{28 - shrink}"] = {"ms": ms, "GB/s": 8 * n / ms / 1e6, "frac": 8 * n / ms / 1e6 / peak}
    xf = torch.from_numpy(G.f32_normal(n, seed=1, stream=5)).to(dev)
    ms = timeit(lambda: L.check(lib.lcpp_scan(1, L.F32, xf.data_ptr(), y.data_ptr(), n, t.data_ptr(), tb, sh)), 20)
    out[f"scan_inclusive_f32_2p{28 - shrink}"] = {"ms": ms, "GB/s": 8 * n / ms / 1e6, "frac": 8 * n / ms / 1e6 / peak}
    del xf, y, t

    # reduce: 2^24 int32 (L2 flushed between iterations) and 2^28 int32
    for logn in (24 - shrink, 28 - shrink):
        n = 1 << logn
        xr = x[:n] if logn == 28 - shrink else torch.from_numpy(G.i32_range(n, -1000, 1000, seed=1, stream=3)).to(dev)
        o = torch.empty(1, dtype=torch.int32, device=dev)
        tb = lib.lcpp_reduce_temp_bytes(L.I32, n)
        t = torch.empty(tb, dtype=torch.uint8, device=dev)
        red = lambda: L.check(lib.lcpp_reduce(0, L.I32, xr.data_ptr(), o.data_ptr(), n, t.data_ptr(), tb, sh))
        ms = timeit(red, 30, flush_l2=True)
        # per-kernel times from the library's own events, in a separate untimed pass
        lib.lcpp_profile_enable(1)
        timeit(red, 10, flush_l2=True)
        c, tt = L.C.c_uint64(0), L.C.c_double(0)
        lib.lcpp_profile_read(b"reduce", L.C.byref(c), L.C.byref(tt))
        lib.lcpp_profile_enable(0)
        out[f"reduce_sum_i32_2p{logn}"] = {"ms": ms, "GB/s": 4 * n / ms / 1e6, "frac": 4 * n / ms / 1e6 / peak,
                                           "kernels_avg_ms": float(tt.value) / max(int(c.value), 1)}
    del x

    # segment reduce: 2^27 f32, 2^20 lognormal segments
    N, S = 1 << (27 - shrink), 1 << (20 - shrink)
    off = G.lognormal_offsets(S, N, seed=1, stream=9)
    xs = torch.from_numpy(G.f32_unit(N, seed=1, stream=10)).to(dev)
    b = torch.from_numpy(off[:-1].view(np.int32).copy()).to(dev)
    e = torch.from_numpy(off[1:].view(np.int32).copy()).to(dev)
    o = torch.empty(S, dtype=torch.float32, device=dev)
    tb = lib.lcpp_segment_reduce_temp_bytes(L.F32, N, S)
    t = torch.empty(tb, dtype=torch.uint8, device=dev)
    seg = lambda: L.check(lib.lcpp_segment_reduce(0, L.F32, xs.data_ptr(), o.data_ptr(), S, b.data_ptr(),
                                                  e.data_ptr(), t.data_ptr(), tb, sh))
    ms = timeit(seg, 20)
    lib.lcpp_profile_enable(1)  # per-kernel times in a separate untimed pass
    timeit(seg, 10)
    kern = {}
    for kname in ("seg_partition", "seg_flat", "seg_fixup"):
        c, tt = L.C.c_uint64(0), L.C.c_double(0)
        lib.lcpp_profile_read(kname.encode(), L.C.byref(c), L.C.byref(tt))
        kern[kname + "_avg_ms"] = float(tt.value) / max(int(c.value), 1)
    lib.lcpp_profile_enable(0)
    byts = 4 * N + 4 * (S + 1) + 4 * S  # values + CSR offsets + outputs
    out[f"segment_sum_f32_2p{27 - shrink}_2p{20 - shrink}"] = {"ms": ms, "GB/s": byts / ms / 1e6,
                                                              "frac": byts / ms / 1e6 / peak, **kern}
    # segment Max over int32 (full range), same segmentation (config 4b)
    xi = torch.from_numpy(G.u32(N, seed=1, stream=13).view(np.int32)).to(dev)
    oi = torch.empty(S, dtype=torch.int32, device=dev)
    ms = timeit(lambda: L.check(lib.lcpp_segment_reduce(2, L.I32, xi.data_ptr(), oi.data_ptr(), S, b.data_ptr(),
                                                        e.data_ptr(), t.data_ptr(), tb, sh)), 20)
    out[f"segment_max_i32_2p{27 - shrink}_2p{20 - shrink}"] = {"ms": ms, "GB/s": byts / ms / 1e6,
                                                              "frac": byts / ms / 1e6 / peak}
    del xi, oi, xs

    # SortKeys (config 3a, 36 B/key) and the skewed SortPairs (config 3c, keys & 0xFF, 68 B/pair schedule)
    n = 1 << (28 - shrink)
    k = torch.from_numpy(G.u32(n, seed=2, stream=7).view(np.int32)).to(dev)
    ko = torch.empty_like(k)
    tbk = lib.lcpp_radix_sort_temp_bytes(L.U32, L.NONE, n)
    tk = torch.empty(tbk, dtype=torch.uint8, device=dev)
    ms = timeit(lambda: L.check(lib.lcpp_radix_sort(L.U32, L.NONE, 0, k.data_ptr(), ko.data_ptr(), None, None, n,
                                                    0, 0, tk.data_ptr(), tbk, sh)), 10)
    out[f"sort_keys_u32_2p{28 - shrink}"] = {"ms": ms, "Gkeys/s": n / ms / 1e6, "GB/s": 36 * n / ms / 1e6,
                                              "frac": 36 * n / ms / 1e6 / peak}
    del tk
    ks = torch.from_numpy(G.u32_masked(n, 0xFF, seed=3).view(np.int32)).to(dev)
    v = torch.arange(n, dtype=torch.int32, device=dev)
    vo = torch.empty_like(v)
    tbp = lib.lcpp_radix_sort_temp_bytes(L.U32, L.U32, n)
    tp = torch.empty(tbp, dtype=torch.uint8, device=dev)
    ms = timeit(lambda: L.check(lib.lcpp_radix_sort(L.U32, L.U32, 0, ks.data_ptr(), ko.data_ptr(), v.data_ptr(),
                                                    vo.data_ptr(), n, 0, 0, tp.data_ptr(), tbp, sh)), 10)
    out[f"sort_pairs_skewed8_u32_2p{28 - shrink}"] = {"ms": ms, "Gpairs/s": n / ms / 1e6, "GB/s": 68 * n / ms / 1e6,
                                                      "frac": 68 * n / ms / 1e6 / peak}
    del k, ko, ks, v, vo, tp

    # scan-by-key / reduce-by-key: 2^28 int32 keys in runs of mean length 100, int32 values
    n = 1 << (28 - shrink)
    gen = torch.Generator(device=dev)
    gen.manual_seed(11)
    keys = torch.cumsum((torch.rand(n, device=dev, generator=gen) < 0.01).to(torch.int32), 0, dtype=torch.int32)
    vals = torch.from_numpy(G.i32_range(n, -1000, 1000, seed=1, stream=12)).to(dev)
    outv = torch.empty_like(vals)
    uk = torch.empty_like(keys)
    nr = torch.empty(1, dtype=torch.int32, device=dev)
    tb = lib.lcpp_scan_by_key_temp_bytes(L.I32, L.I32, n)
    t = torch.empty(tb, dtype=torch.uint8, device=dev)
    ms = timeit(lambda: L.check(lib.lcpp_scan_by_key(0, 0, L.I32, L.I32, keys.data_ptr(), vals.data_ptr(),
                                                     outv.data_ptr(), n, None, t.data_ptr(), tb, sh)), 20)
    out[f"exclusive_sum_by_key_i32_2p{28 - shrink}"] = {"ms": ms, "GB/s": 12 * n / ms / 1e6,
                                                         "frac": 12 * n / ms / 1e6 / peak}
    ms = timeit(lambda: L.check(lib.lcpp_reduce_by_key(0, L.I32, L.I32, keys.data_ptr(), vals.data_ptr(),
                                                       uk.data_ptr(), outv.data_ptr(), nr.data_ptr(), n,
                                                       t.data_ptr(), tb, sh)), 20)
    runs = int(nr.item())
    byts = 8 * n + 8 * runs
    out[f"reduce_by_key_sum_i32_2p{28 - shrink}"] = {"ms": ms, "GB/s": byts / ms / 1e6, "frac": byts / ms / 1e6 / peak,
                                                     "runs": runs}
    return out


def _fill_u64_uniform(torch, out, gen):
    """Uniform 64-bit keys written into out (int64 view) in chunks."""
    chunk = 1 << 26
    for i in range(0, out.numel(), chunk):
        m = min(chunk, out.numel() - i)
        hi = torch.randint(0, 1 << 32, (m,), dtype=torch.int64, device=out.device, generator=gen)
        lo = torch.randint(0, 1 << 32, (m,), dtype=torch.int64, device=out.device, generator=gen)
        out[i:i + m] = (hi << 32) | lo


def _mix(torch, k64, v64):
    """Order-independent fingerprint term of (key, value) pairs: int64 sums wrap."""
    return ((k64 * -7046029254386353131) ^ (v64 * -4417276706812531889) ^ (k64 >> 29)).sum()


def run_mg_extras(torch, dev, lib, L, peak, rank, world, max_over_ranks, barrier, shrink=0, steps=3):
    """BASELINE config 5 at this N (strong scaling, total work fixed):
    5a global SortPairs of 2^31 uniform u64 keys + u32 values (= global index),
    5b ExclusiveSum of 2^32 u32 values uniform in [0,16), both sharded evenly
    in rank order and run through the multi-GPU C ABI (lcpp_mg_sort,
    lcpp_mg_scan).  Per-phase device times come from the library's events;
    the untimed checks verify the global result on the device."""
    from lc_parallel_primitive_b200 import multi_gpu as M

    comm = M.comm_for() if world > 1 else None
    stream = torch.cuda.current_stream()
    out = {}
    gen = torch.Generator(device=dev)

    def phases(names):
        res = {}
        for nm in names:
            c, t = L.C.c_uint64(0), L.C.c_double(0)
            lib.lcpp_profile_read(nm.encode(), L.C.byref(c), L.C.byref(t))
            v = max_over_ranks(float(t.value) / max(int(c.value), 1))
            if c.value or world > 1:
                res[nm + "_ms"] = v
        return res

    def timed(fn, k):
        for _ in range(2):
            fn()
        torch.cuda.synchronize()
        barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(k):
            fn()
        b.record(stream)
        torch.cuda.synchronize()
        barrier()
        return max_over_ranks(a.elapsed_time(b) / k)

    if comm is None:  # one rank: a 1-rank communicator through the same C ABI
        import ctypes as C

        uid = C.create_string_buffer(int(lib.lcpp_mg_unique_id_bytes()))
        L.check(lib.lcpp_mg_get_unique_id(uid))
        h = C.c_void_p()
        L.check(lib.lcpp_mg_comm_init_rank(C.byref(h), 1, uid, 0))

        class _One:
            handle, world, nranks, rank = h, 1, 1, 0
        comm = _One()
    nr = L.C.c_int(0)
    L.check(lib.lcpp_mg_comm_shape(comm.handle, L.C.byref(L.C.c_int(0)), L.C.byref(nr)))

    # ---- 5a ------------------------------------------------------------------
    N = 1 << (31 - shrink)
    n = N // world
    gen.manual_seed(1000 + rank)
    keys = torch.empty(n, dtype=torch.int64, device=dev)
    _fill_u64_uniform(torch, keys, gen)
    vals = torch.arange(rank * n, rank * n + n, dtype=torch.int64, device=dev).to(torch.int32)
    cap = M.default_capacity(n) if world > 1 else n
    ko = torch.empty(cap, dtype=torch.int64, device=dev)
    vo = torch.empty(cap, dtype=torch.int32, device=dev)
    tb = M.mg_sort_temp_bytes(keys.view(torch.uint64), vals.view(torch.uint32), cap, world)
    temp = torch.empty(tb, dtype=torch.uint8, device=dev)
    res = {}

    def sort5a():
        res["r"] = M.mg_sort_pairs(keys.view(torch.uint64), vals.view(torch.uint32), comm=comm, capacity=cap,
                                   temp=temp, keys_out=ko.view(torch.uint64), vals_out=vo.view(torch.uint32))

    sort5a()
    torch.cuda.synchronize()
    L.check(lib.lcpp_last_device_error(stream.cuda_stream), "device error (5a)")
    # untimed global check: order, continuity across ranks, count, stability,
    # pairs kept together (fingerprint of (key, value) before and after); in
    # chunks, so that the check needs little memory beside the buffers
    m = res["r"].n
    ok = True
    fp_in = torch.zeros((), dtype=torch.int64, device=dev)
    fp_out = torch.zeros((), dtype=torch.int64, device=dev)
    chunk = 1 << 26
    for i in range(0, n, chunk):
        j = min(i + chunk, n)
        fp_in += _mix(torch, keys[i:j], vals[i:j].to(torch.int64) & 0xFFFFFFFF)
    for i in range(0, m, chunk):
        j = min(i + chunk + 1, m)  # one item of overlap with the next chunk
        sk = ko[i:j] ^ (-(1 << 63))  # unsigned order as signed
        sv = vo[i:j].to(torch.int64) & 0xFFFFFFFF
        if j - i > 1:
            ok &= bool((sk[1:] >= sk[:-1]).all())
            eq = sk[1:] == sk[:-1]
            ok &= bool((sv[1:][eq] > sv[:-1][eq]).all())
        k_ = min(i + chunk, m)
        fp_out += _mix(torch, ko[i:k_], vo[i:k_].to(torch.int64) & 0xFFFFFFFF)
        del sk, sv
    stats = torch.stack([torch.tensor(m, dtype=torch.int64, device=dev), fp_in, fp_out])
    first = (ko[0] ^ (-(1 << 63))).item() if m else 0
    last = (ko[m - 1] ^ (-(1 << 63))).item() if m else 0
    ends = torch.tensor([first, last, int(vo[0].item()) & 0xFFFFFFFF if m else 0,
                         int(vo[m - 1].item()) & 0xFFFFFFFF if m else 0, m], dtype=torch.int64, device=dev)
    if world > 1:
        torch.distributed.all_reduce(stats)
        allends = [torch.empty_like(ends) for _ in range(world)]
        torch.distributed.all_gather(allends, ends)
        e = [t.cpu().tolist() for t in allends]
        e = [x for x in e if x[4] > 0]
        for a_, b_ in zip(e, e[1:]):
            ok &= a_[1] < b_[0] or (a_[1] == b_[0] and a_[3] < b_[2])
    st = stats.cpu().tolist()
    ok &= st[0] == N and st[1] == st[2]
    lib.lcpp_profile_enable(1)
    ms = timed(sort5a, steps)
    ph = phases(["mg_splitters", "mg_partition", "mg_plan", "mg_exchange", "mg_local_sort", "rs_onesweep"])
    lib.lcpp_profile_enable(0)
    per_pair = 200 if world == 1 else 268  # modelled HBM bytes per local pair (DESIGN: 5a)
    out[f"mg_sort_pairs_u64_2p{31 - shrink}"] = {
        "ms": ms, "Gpairs/s": N / (ms * 1e-3) / 1e9, "n_gpus": world, "n_per_gpu": n, "scaling": "strong",
        "check_ok": bool(ok), "max_slice": int(max_over_ranks(float(m))), "comm_nranks": nr.value,
        "hbm_bytes_per_pair_model": per_pair,
        "hbm_frac_model": per_pair * n / (ms * 1e-3) / 1e9 / peak,
        "nvlink_bytes_per_gpu": 12 * n * (world - 1) // world, **ph}
    del keys, vals, ko, vo, temp, res
    torch.cuda.empty_cache()

    # ---- 5b ------------------------------------------------------------------
    N = 1 << (32 - shrink)
    n = N // world
    gen.manual_seed(2000 + rank)
    x = torch.empty(n, dtype=torch.int32, device=dev)
    chunk = 1 << 27
    for i in range(0, n, chunk):
        x[i:i + chunk] = torch.randint(0, 16, (min(chunk, n - i),), dtype=torch.int32, device=dev, generator=gen)
    y = torch.empty_like(x)
    tb = M.mg_scan_temp_bytes(x.view(torch.uint32), world)
    temp = torch.empty(tb, dtype=torch.uint8, device=dev)

    def scan5b():
        M.mg_scan(False, x.view(torch.uint32), y.view(torch.uint32), comm=comm, temp=temp)

    scan5b()
    torch.cuda.synchronize()
    L.check(lib.lcpp_last_device_error(stream.cuda_stream), "device error (5b)")
    ok = True
    for i in range(0, n - 1, chunk):  # out[i+1] - out[i] == x[i] (mod 2^32), in chunks
        j = min(i + chunk, n - 1)
        ok &= bool(((y[i + 1:j + 1] - y[i:j]) == x[i:j]).all())
    first = int(y[0].item())
    tail = torch.tensor([int(y[-1].item()) + int(x[-1].item()), first], dtype=torch.int64, device=dev)
    if world > 1:
        allt = [torch.empty_like(tail) for _ in range(world)]
        torch.distributed.all_gather(allt, tail)
        t = [a_.cpu().tolist() for a_ in allt]
        ok &= t[0][1] == 0 and all((t[r][0] & 0xFFFFFFFF) == (t[r + 1][1] & 0xFFFFFFFF) for r in range(world - 1))
    else:
        ok &= first == 0
    lib.lcpp_profile_enable(1)
    ms = timed(scan5b, max(steps, 5))
    ph = phases(["mg_local_reduce", "mg_allgather", "mg_carry_scan"])
    lib.lcpp_profile_enable(0)
    out[f"mg_exclusive_sum_u32_2p{32 - shrink}"] = {
        "ms": ms, "GB/s_per_gpu_8B": 8 * n / (ms * 1e-3) / 1e9, "frac_8B": 8 * n / (ms * 1e-3) / 1e9 / peak,
        "frac_12B_structural": 12 * n / (ms * 1e-3) / 1e9 / peak, "n_gpus": world, "n_per_gpu": n,
        "scaling": "strong", "check_ok": bool(ok), "comm_nranks": nr.value, **ph}
    del x, y, temp
    torch.cuda.empty_cache()
    if world == 1:
        L.check(lib.lcpp_mg_comm_destroy(comm.handle))
    return out


if __name__ == "__main__":
    sys.exit(main())
