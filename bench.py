"""Benchmark: Soft-DTW DP cells/s, forward + backward, on the headline workload (a global batch of B=256
pairs, N=M=512, d=64, fp32, gamma=0.1, no band): ``SoftDTW(gamma=0.1)(X, Y).sum().backward()`` with X
requiring grad.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]

One process per GPU (torchrun for N > 1). The seeded global batch is cut into contiguous slices, one per
rank (strong scaling: B/N pairs per GPU, no collective on the data path). Prints ONE JSON line on rank 0.

* value       cells of the global batch / max over ranks of the summed per-step device time
              (CUDA events around each step; L2 flushed between steps, outside the timed events)
* fwd         the same for the forward alone (cost matrix, forward wavefront, costs)
* step_roofline  value against the whole step's bound: min(HBM bandwidth / algorithmic bytes per cell,
              MUFU rate / transcendentals per cell), for fwd+bwd and for fwd
* weak        (N > 1) every rank runs a full batch of B pairs of its own: weak scaling, secondary
* e2e         the same metric through the public API with inputs in pinned host memory: H2D copy of
              X and Y, the step, D2H read of the loss, all inside the timed region; with the box's
              measured pinned H2D bandwidth and the copy-bound rate it implies
* roofline    the dominant kernel (by device time per step), timed alone through the C ABI with CUDA
              events on its stream; algorithmic bytes per DP cell / duration vs measured HBM bandwidth
* cpu_baseline  the reference's own CPU operator (compiled from its source, oracle/_ref) driven by the
              reference's module glue (restated in oracle/oracle.py), on a bounded sample of the same
              workload, all host threads
* --impl reference: that same CPU path as the reference arm (rank 0 only). That arm never imports
              torchsoftdtw_b200: the inputs come from workloads.py loaded as a file, the cells are
              counted by the oracle.
"""

from __future__ import annotations

import argparse
import importlib.util
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

# NCCL prints its version banner on stdout when NCCL_DEBUG=VERSION (the default of some images), and it reads
# the variable when torch loads it; the bench prints one JSON line on stdout.
if os.environ.get("NCCL_DEBUG", "").upper() == "VERSION":
    os.environ["NCCL_DEBUG"] = "WARN"

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def _load_workloads():
    """torchsoftdtw_b200/workloads.py loaded as a plain file: the seeded inputs are pure torch, and loading
    the file does not run the package's __init__ (which loads the native libraries)."""
    path = os.path.join(ROOT, "torchsoftdtw_b200", "workloads.py")
    spec = importlib.util.spec_from_file_location("sdtw_bench_workloads", path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod
    spec.loader.exec_module(mod)
    return mod


_WL = _load_workloads()
WORKLOADS, make_inputs = _WL.WORKLOADS, _WL.make_inputs

DATA_KIND = {"normal": "N(0,1)", "uniform": "U[-1,1]", "randwalk": "random walks", "sine": "noisy sines"}

L2_FLUSH_BYTES = 256 << 20


# ---------------------------------------------------------------------------------------------------
def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 100 ms in the background."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.tmp = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(gpu_index), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=self.tmp, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        self.marks = []

    def mark(self):
        self.tmp.flush()
        self.marks.append(self._count())

    def _count(self):
        try:
            with open(self.tmp.name) as f:
                return sum(1 for _ in f)
        except OSError:
            return 0

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        with open(self.tmp.name) as f:
            rows = [r.strip().split(", ") for r in f if r.strip()]
        os.unlink(self.tmp.name)
        return rows

    @staticmethod
    def summarize(rows, first: int):
        sel = rows[first:] if len(rows) > first else rows[-3:]
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in sel:
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
                for k, v in zip(names, r[5:9]):
                    if v.strip() == "Active":
                        reasons.add(k)
            except (ValueError, IndexError):
                continue
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------------------------------
# The reference's CPU path (timed baseline and reference arm). Only the oracle is loaded here: the
# reference's compiled CPU operator (oracle/_ref) under its module glue, restated in oracle/oracle.py.
# ---------------------------------------------------------------------------------------------------
def cpu_reference_measure(w, sample_pairs: int, steps: int, warmup: int, min_seconds: float = 0.0):
    """Cells/s of the reference CPU path on `sample_pairs` pairs of the workload, all host threads."""
    from oracle import oracle as O

    if not O.ref_available():
        O.build()
    O.load_ref()
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    X, Y, lx, ly, _ = make_inputs(w.name, seed=1000, batch=sample_pairs)
    cells = O.count_cells(lx.numpy(), ly.numpy(), w.bandwidth)
    for _ in range(warmup):
        O.reference_module_step(X, Y, lx, ly, w.gamma, w.bandwidth, w.normalize)
    times = []
    t_total = 0.0
    while len(times) < steps or t_total < min_seconds:
        t0 = time.perf_counter()
        O.reference_module_step(X, Y, lx, ly, w.gamma, w.bandwidth, w.normalize)
        dt = time.perf_counter() - t0
        times.append(dt)
        t_total += dt
    mean = sum(times) / len(times)
    return {"value": cells / mean, "unit": "cells/s", "cores": threads, "kind": "reference",
            "sample": f"{sample_pairs} pairs of the {w.name} workload ({cells} cells) per step, "
                      f"{len(times)} steps, module fwd+bwd (the reference's pairwise_l2_squared + its CPU op + "
                      f"torch autograd)",
            "s_per_step": mean}


def run_reference_arm(args, w, rank, world):
    if rank != 0:
        return
    sample = args.cpu_sample
    r = cpu_reference_measure(w, sample, max(args.steps, 1), max(args.warmup, 1))
    line = {
        "impl": "reference", "metric": metric_name(w), "value": r["value"], "unit": "cells/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": r["s_per_step"] * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": dtype_name(w),
        "data": "synthetic", "config": config_of(w, world),
        "cpu_baseline": {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": r["value"], "unit": "cells/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------------------------------
def metric_name(w):
    return f"Soft-DTW DP cells/sec fwd+bwd (B={w.B},N={w.N},M={w.M},d={w.d} {dtype_name(w)})"


def dtype_name(w):
    return "f64" if w.dtype == torch.float64 else "f32"


def config_of(w, world):
    return {"workload": w.name, "global_batch": w.B, "pairs_per_gpu": f"{w.B}/{world}", "N": w.N, "M": w.M,
            "d": w.d, "gamma": w.gamma, "bandwidth": w.bandwidth, "normalize": w.normalize,
            "parallelism": f"batch-shard x{world} (contiguous slices of one seeded global batch)",
            "step": "SoftDTW(X,Y).sum().backward(), grad_X only",
            "l2": "flushed between timed steps (256 MiB write, outside the timed events)"}


# Transcendental (MUFU) operations per DP cell of the north_star roofline: forward 2 exp + 1 log,
# backward 3 exp. SMs x 16 MUFU results per clock x the SM clock is the MUFU rate.
MUFU_PER_CELL = {"fwd": 3, "fwd+bwd": 6}


def step_roofline(w, value: float, kind: str, sms: int):
    """value (cells/s) against min(HBM / algorithmic bytes per cell, MUFU rate / MUFU ops per cell) of the
    whole step, D and E kept on chip: R written once (and read once by the backward), X and Y read by
    each pass, grad_X written."""
    es = 8 if w.dtype == torch.float64 else 4
    hbm, src = peaks()
    nm = float(w.N * w.M)
    if kind == "fwd":
        bpc = es + (w.N + w.M) * w.d * es / nm
    else:
        bpc = 2 * es + (2 * (w.N + w.M) + w.N) * w.d * es / nm
    hbm_cells = hbm * 1e9 / bpc
    out = {"bytes_per_cell": bpc, "hbm_gbs": hbm, "hbm_bound_cells_per_s": hbm_cells, "peak_source": src}
    peak = hbm_cells
    if w.dtype == torch.float32:
        mhz = sm_max_mhz()
        mufu = sms * 16 * mhz * 1e6
        out.update({"mufu_per_cell": MUFU_PER_CELL[kind], "mufu_per_s": mufu,
                    "mufu_bound_cells_per_s": mufu / MUFU_PER_CELL[kind]})
        peak = min(peak, mufu / MUFU_PER_CELL[kind])
    out["bound"] = "hbm" if peak == hbm_cells else "mufu"
    out["peak_cells_per_s"] = peak
    out["frac"] = value / peak
    return out


def sm_max_mhz() -> float:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            return float(json.load(f).get("sm_max_mhz", 1965.0))
    return 1965.0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="medium", choices=sorted(WORKLOADS))
    ap.add_argument("--cpu-sample", type=int, default=None,
                    help="pairs per CPU-baseline step (default: one per host thread, at least 16)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile", action="store_true", help="run for profilers: timed fwd+bwd steps only")
    ap.add_argument("--batch", type=int, default=None, help="global batch (default: the workload's B)")
    ap.add_argument("--no-weak", action="store_true", help="N > 1: skip the secondary weak-scaling timing")
    ap.add_argument("--loss-allreduce", action="store_true",
                    help="N > 1: also time the step followed by the global loss sum (NCCL all-reduce of one scalar)")
    args = ap.parse_args()
    rank, world, local = dist_env()
    w = WORKLOADS[args.workload]
    if args.cpu_sample is None:
        args.cpu_sample = max(16, os.cpu_count() or 1)
    if args.batch is not None:
        import dataclasses

        w = dataclasses.replace(w, B=args.batch)

    if args.impl == "reference":
        run_reference_arm(args, w, rank, world)
        return

    import torch.distributed as dist

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    import torchsoftdtw_b200 as T
    from torchsoftdtw_b200 import _ext, sharding
    from torchsoftdtw_b200.workloads import count_cells

    # One seeded global batch (the same on every rank); this rank keeps its contiguous slice.
    Xg, Yg, lxg, lyg, _ = make_inputs(w.name, seed=0, batch=w.B)
    b0, b1 = sharding.shard_bounds(w.B, world, rank)
    X, Y, lx, ly = Xg[b0:b1].contiguous(), Yg[b0:b1].contiguous(), lxg[b0:b1], lyg[b0:b1]
    cells_global = count_cells(lxg, lyg, w.bandwidth)
    cells_rank = count_cells(lx, ly, w.bandwidth)
    Xd, Yd, lxd, lyd = X.to(dev), Y.to(dev), lx.to(dev), ly.to(dev)
    Xd.requires_grad_(True)
    Xnd = Xd.detach()
    module = T.SoftDTW(gamma=w.gamma, bandwidth=w.bandwidth, normalize=w.normalize)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    capi = _ext.capi()

    def step():
        Xd.grad = None
        loss = module(Xd, Yd, lxd, lyd).sum()
        loss.backward()
        return loss

    def fwd_step():
        return module(Xnd, Yd, lxd, lyd)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    def max_over_ranks(v: float) -> float:
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def timed(fn, steps: int, warmup: int) -> tuple[float, int]:
        """Summed CUDA-event time (ms) of `steps` calls of fn after `warmup` untimed ones, L2 flushed before
        each call outside the events, max over ranks; and this library's kernel launches in the timed calls."""
        for _ in range(max(warmup, 1)):
            fn()
        torch.cuda.synchronize()
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        barrier()
        torch.cuda.synchronize()
        l0 = capi.sdtw_debug_kernel_launches()
        for k in range(steps):
            flush.fill_(float(k))
            starts[k].record()
            fn()
            ends[k].record()
        torch.cuda.synchronize()
        launches = capi.sdtw_debug_kernel_launches() - l0
        barrier()
        return max_over_ranks(sum(s.elapsed_time(e) for s, e in zip(starts, ends))), int(launches)

    sampler = None if args.profile else ClockSampler(local)
    if sampler:
        time.sleep(0.3)
        sampler.mark()
    steps = args.steps
    ms_max, launches = timed(step, steps, args.warmup)
    T.check_errors(dev)
    value = cells_global * steps / (ms_max / 1e3)
    result = {
        "metric": metric_name(w), "value": value, "unit": "cells/s", "n_gpus": world, "steps": steps,
        "warmup": args.warmup, "ms_per_step": ms_max / steps, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": dtype_name(w),
        "data": f"synthetic (one seeded global batch, {DATA_KIND[w.kind]}; no dataset)",
        "config": config_of(w, world), "gpu_launches": launches,
    }
    if args.profile:
        if rank == 0:
            print(json.dumps(result), flush=True)
        if world > 1:
            dist.destroy_process_group()
        return
    if sampler:
        sampler.mark()

    # ---- forward alone (cost matrix + forward wavefront + costs) ---------------------------------------
    ms_fwd, launches_fwd = timed(fwd_step, steps, args.warmup)
    T.check_errors(dev)
    value_fwd = cells_global * steps / (ms_fwd / 1e3)
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    result["fwd"] = {"value": value_fwd, "unit": "cells/s", "ms_per_step": ms_fwd / steps,
                     "gpu_launches": launches_fwd, "step_roofline": step_roofline(w, value_fwd, "fwd", sms)}
    result["step_roofline"] = step_roofline(w, value, "fwd+bwd", sms)

    if world > 1 and args.loss_allreduce:
        # The same steps with the global loss sum (sharding.all_reduce_loss: one fp32 scalar, all_reduce(SUM)
        # over NCCL). after_backward: the collective follows the step; overlapped: it starts when the forward
        # has produced the loss and runs beside the backward, joined before the step's end event.
        def step_global():
            return sharding.all_reduce_loss(step())

        def step_global_overlapped():
            Xd.grad = None
            loss = module(Xd, Yd, lxd, lyd).sum()
            pending = sharding.all_reduce_loss(loss, async_op=True)
            loss.backward()
            return pending.wait()

        ms2, _ = timed(step_global, steps, 2)
        ms3, _ = timed(step_global_overlapped, steps, 2)
        result["with_loss_allreduce"] = {"value": cells_global * steps / (ms2 / 1e3), "unit": "cells/s",
                                         "ms_per_step": ms2 / steps,
                                         "overlapped": {"value": cells_global * steps / (ms3 / 1e3),
                                                        "ms_per_step": ms3 / steps}}

    if world > 1 and not args.no_weak:
        # Secondary: weak scaling, every rank a full batch of B pairs of its own (seed = rank).
        Xw, Yw, lxw, lyw, _ = make_inputs(w.name, seed=rank, batch=w.B)
        cw = float(count_cells(lxw, lyw, w.bandwidth))
        Xwd, Ywd, lxwd, lywd = Xw.to(dev).requires_grad_(True), Yw.to(dev), lxw.to(dev), lyw.to(dev)

        def step_weak():
            Xwd.grad = None
            module(Xwd, Ywd, lxwd, lywd).sum().backward()

        weak_steps = max(5, steps // 4)
        ms_w, _ = timed(step_weak, weak_steps, 2)
        cw_t = torch.tensor([cw], dtype=torch.float64, device=dev)
        dist.all_reduce(cw_t, op=dist.ReduceOp.SUM)
        result["weak"] = {"value": float(cw_t.item()) * weak_steps / (ms_w / 1e3), "unit": "cells/s",
                          "ms_per_step": ms_w / weak_steps, "pairs_per_gpu": w.B, "global_batch": w.B * world,
                          "steps": weak_steps}
        del Xwd, Ywd

    # ---- e2e through the public API with host buffers ----------------------------------------------
    # Every step copies its X and Y slices from pinned host memory (H2D) and reads its loss back (D2H)
    # inside the timed region. The copies run on a second stream into two alternating device buffers, so
    # the copy of step k+1 overlaps the compute of step k (an input pipeline); step k waits for its own
    # copy, and the copy into a buffer waits for the step that last used it.
    Xh = X.pin_memory()
    Yh = Y.pin_memory()
    loss_h = torch.empty((), dtype=torch.float32).pin_memory()
    e2e_steps = max(10, steps // 4)
    copy_stream = torch.cuda.Stream(device=dev)
    main_stream = torch.cuda.current_stream(dev)
    xbuf = [torch.empty_like(Xnd) for _ in range(2)]
    ybuf = [torch.empty_like(Yd) for _ in range(2)]
    copied = [torch.cuda.Event() for _ in range(2)]
    used = [torch.cuda.Event() for _ in range(2)]
    h2d_bytes = Xh.numel() * Xh.element_size() + Yh.numel() * Yh.element_size()

    # Pinned host -> device bandwidth of this box for these buffers (the bound of the e2e figure).
    for _ in range(2):
        xbuf[0].copy_(Xh, non_blocking=True)
        ybuf[0].copy_(Yh, non_blocking=True)
    torch.cuda.synchronize()
    c0 = torch.cuda.Event(enable_timing=True)
    c1 = torch.cuda.Event(enable_timing=True)
    c0.record()
    for _ in range(5):
        xbuf[0].copy_(Xh, non_blocking=True)
        ybuf[0].copy_(Yh, non_blocking=True)
    c1.record()
    torch.cuda.synchronize()
    h2d_gbs = 5 * h2d_bytes / (c0.elapsed_time(c1) / 1e3) / 1e9

    def e2e_copy(k, after):
        j = k % 2
        with torch.cuda.stream(copy_stream):
            copy_stream.wait_event(after)
            xbuf[j].copy_(Xh, non_blocking=True)
            ybuf[j].copy_(Yh, non_blocking=True)
            copied[j].record(copy_stream)

    def e2e_step(k):
        j = k % 2
        main_stream.wait_event(copied[j])
        xs = xbuf[j].detach().requires_grad_(True)  # a fresh leaf over the buffer (the copies write the buffer)
        loss = module(xs, ybuf[j], lxd, lyd).sum()
        loss.backward()
        loss_h.copy_(loss.detach(), non_blocking=True)
        used[j].record(main_stream)

    for k in range(3):  # warm-up of the pipeline (allocator blocks, first launches)
        e2e_copy(k, used[k % 2] if k >= 2 else main_stream.record_event())
        e2e_step(k)
    barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(main_stream)
    e2e_copy(0, e0)
    for k in range(e2e_steps):
        if k + 1 < e2e_steps:
            e2e_copy(k + 1, used[(k + 1) % 2] if k >= 1 else e0)
        e2e_step(k)
    e1.record(main_stream)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1))
    e2e_value = cells_global * e2e_steps / (e2e_ms / 1e3)
    h2d_min = -max_over_ranks(-h2d_gbs)
    copy_bound = cells_global / (h2d_bytes / (h2d_min * 1e9))
    result["e2e"] = {"value": e2e_value, "unit": "cells/s", "h2d_bytes_per_step": h2d_bytes,
                     "d2h_bytes_per_step": loss_h.element_size(), "ms_per_step": e2e_ms / e2e_steps,
                     "h2d_gbs_measured": h2d_min, "copy_bound_cells_per_s": copy_bound,
                     "frac_of_copy_bound": e2e_value / copy_bound}

    # ---- per-kernel device time through the C ABI (dominant kernel -> roofline) --------------------
    kt = kernel_times(T, Xnd, Yd, lxd, lyd, w, dev, flush)
    clocks = sampler.summarize(sampler.stop(), sampler.marks[0]) if sampler else None
    if rank == 0:
        hbm, peak_kind = peaks()
        name, ms = max(kt.items(), key=lambda kv: kv[1])
        bytes_per_cell = ALGO_BYTES[name] * (8 if w.dtype == torch.float64 else 4)
        achieved = cells_rank * bytes_per_cell / (ms / 1e3) / 1e9
        traffic = measured_traffic(w, world, name)
        result["roofline"] = {"bound": "hbm", "kernel": name, "achieved": achieved, "peak": hbm,
                              "unit": "GB/s", "frac": achieved / hbm,
                              "traffic": traffic / (ms / 1e3) / 1e9 if traffic else None,
                              "traffic_bytes_per_launch": traffic,
                              "peak_source": peak_kind,
                              "algorithmic_bytes_per_cell": bytes_per_cell, "launch_ms": ms,
                              "per_kernel_ms": kt}
        result["clocks"] = clocks
        if not args.no_cpu_baseline and world == 1:
            r = cpu_reference_measure(w, args.cpu_sample, 2, 1, min_seconds=10.0)
            result["cpu_baseline"] = {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")}
        print(json.dumps(result), flush=True)
    if world > 1:
        dist.destroy_process_group()


def measured_traffic(w, world: int, name: str):
    """DRAM bytes (read + write) of one launch of the C-ABI call `name` on one rank's slice of workload `w`,
    as recorded from an ncu capture in profiles/dram_traffic_<workload>_b<pairs per GPU>.txt (lines:
    <call> <kernel> <bytes>), or None when no capture of that slice exists."""
    path = os.path.join(ROOT, "profiles", f"dram_traffic_{w.name}_b{(w.B + world - 1) // world}.txt")
    if not os.path.exists(path):
        return None
    with open(path) as f:
        for line in f:
            parts = line.split()
            if len(parts) == 3 and not line.startswith("#") and parts[0] == name:
                return int(parts[2])
    return None


# Algorithmic DRAM bytes per DP cell, in units of the element size, of each timed C-ABI call:
#   forward  : read D + write R                      = 2
#   backward : read R + write E                      = 2
#   pairwise : write D (X, Y reads are O((N+M)d/NM)) = 1
#   grad     : read E (D only for pairs with a clamped cell) = 1
ALGO_BYTES = {"sdtw_forward": 2, "sdtw_backward": 2, "sdtw_forward_tiles": 2, "sdtw_backward_tiles": 2,
              "sdtw_pairwise_l2": 1, "sdtw_grad_l2": 1, "sdtw_forward_band_r": 2, "sdtw_pairwise_l2_band": 1,
              "sdtw_grad_l2_band": 1}


def kernel_times(T, X, Y, lx, ly, w, dev, flush, reps: int = 20):
    """Average device time (ms) of each C-ABI call of one step, CUDA events on the launching stream,
    L2 flushed before each launch."""
    import ctypes

    from torchsoftdtw_b200 import _ext

    lib = _ext.capi()
    B, N, d = X.shape
    M = Y.shape[1]
    code = 1 if X.dtype == torch.float64 else 0
    D = torch.empty(B, N, M, device=dev, dtype=X.dtype)
    R = torch.empty(B, N + 2, M + 2, device=dev, dtype=X.dtype)
    E = torch.empty(B, N, M, device=dev, dtype=X.dtype)
    costs = torch.empty(B, device=dev, dtype=X.dtype)
    g = torch.ones(B, device=dev, dtype=X.dtype)
    flags = torch.zeros(B, device=dev, dtype=torch.int32)
    gX = torch.empty_like(X)
    err = torch.zeros(1, device=dev, dtype=torch.int32)
    wsf = lib.sdtw_forward_workspace_bytes(B, N, M, code)
    wsb = lib.sdtw_backward_workspace_bytes(B, N, M, code)
    ws = torch.empty(max(wsf, wsb), device=dev, dtype=torch.uint8)
    stream = torch.cuda.current_stream()
    sp = ctypes.c_void_p(stream.cuda_stream)
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    is32 = 1 if lx.dtype == torch.int32 else 0
    calls = {
        "sdtw_pairwise_l2": lambda: lib.sdtw_pairwise_l2(code, p(X), p(Y), B, N, M, d, p(D), p(flags), sp),
        "sdtw_forward": lambda: lib.sdtw_forward(code, p(D), B, N, M, p(lx), p(ly), is32, w.gamma, w.bandwidth,
                                                 p(R), p(costs), p(ws), wsf, p(err), sp),
        "sdtw_backward": lambda: lib.sdtw_backward(code, p(D), p(R), B, N, M, p(lx), p(ly), is32, w.gamma,
                                                   w.bandwidth, p(E), p(ws), wsb, p(err), sp),
        "sdtw_grad_l2": lambda: lib.sdtw_grad_l2(code, p(X), p(Y), p(D), p(E), p(g), p(flags), B, N, M, d, p(gX),
                                                 None, sp),
    }
    if lib.sdtw_r_tiled(B, N, M, code):
        # The module path hands R over as strip tiles for this shape: time the calls it makes.
        Rt = torch.empty(lib.sdtw_r_tiles_elems(B, N, M), device=dev, dtype=X.dtype)
        calls["sdtw_forward_tiles"] = lambda: lib.sdtw_forward_tiles(code, p(D), B, N, M, p(lx), p(ly), is32, w.gamma,
                                                                     w.bandwidth, p(Rt), p(costs), p(ws), wsf, p(err),
                                                                     sp)
        calls["sdtw_backward_tiles"] = lambda: lib.sdtw_backward_tiles(code, p(Rt), B, N, M, p(lx), p(ly), is32,
                                                                       w.gamma, w.bandwidth, p(E), p(ws), wsb, p(err),
                                                                       sp)
        del calls["sdtw_forward"], calls["sdtw_backward"]
    if w.bandwidth >= 0:
        # With a band the module computes only the cost tiles and E chunks its wavefronts read, and (on the
        # strip-ticket kernels) prefills only the part of R the backward loads: time those calls.
        wsp = lib.sdtw_pairwise_l2_band_workspace_bytes(B, N, M)
        wsbuf = torch.empty(wsp, device=dev, dtype=torch.uint8)
        band = {
            "sdtw_pairwise_l2_band": lambda: lib.sdtw_pairwise_l2_band(code, p(X), p(Y), B, N, M, d, p(lx), p(ly),
                                                                       is32, w.bandwidth, p(D), p(flags),
                                                                       p(wsbuf), wsp, sp),
        }
        for name in list(calls):
            if name == "sdtw_forward":
                band["sdtw_forward_band_r"] = lambda: lib.sdtw_forward_band_r(
                    code, p(D), B, N, M, p(lx), p(ly), is32, w.gamma, w.bandwidth, p(R), p(costs), p(ws), wsf,
                    p(err), sp)
            elif name not in ("sdtw_pairwise_l2", "sdtw_grad_l2"):
                band[name] = calls[name]
        band["sdtw_grad_l2_band"] = lambda: lib.sdtw_grad_l2_band(code, p(X), p(Y), p(D), p(E), p(g), p(flags), B,
                                                                  N, M, d, p(lx), p(ly), is32, w.bandwidth, p(gX),
                                                                  None, sp)
        calls = band
    out = {}
    for name, fn in calls.items():
        st = fn()
        assert st == 0, (name, lib.sdtw_status_string(st))
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
        for a, b in ev:
            flush.fill_(1.0)
            a.record(stream)
            fn()
            b.record(stream)
        torch.cuda.synchronize()
        out[name] = sum(a.elapsed_time(b) for a, b in ev) / reps
    assert lib.sdtw_read_error_word(p(err), sp) == 0
    return out


if __name__ == "__main__":
    main()
