#!/usr/bin/env python
"""Benchmark of the SpMM hot path (driver contract).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config 2] [--op csr|mixed]

One step = one SpMM C = A @ B of BASELINE config 2 (1M x 1M power-law graph,
~16 nonzeros/row, fp16, N = 256) with its inputs resident in HBM.  With N
GPUs (torchrun, one rank per GPU) A is row-partitioned, B is replicated and C
stays row-sharded: no collective runs in the timed region.

``--scaling weak`` (default): every rank owns one config-sized row block of a
global A of N blocks (rank r's block is the config generated with seed
2027 + r; rank 0's block is the 1-GPU workload) times the shared B (seed
2027), so the work per GPU is fixed as N grows.  ``--scaling strong``: the
single config matrix is cut into N row ranges balanced by nonzeros at 16-row
window boundaries (spmm_dist.shard_bounds).

``--impl reference`` times the reference's own CPU path for SpMM
(tests/aic_aiv_ablation/common.py:173-177: torch.sparse.mm in fp32, all
host threads) on a bounded row sample of the same workload, on rank 0 only.

Rank 0 prints one JSON line.  Inputs (B is 537 MB) are larger than the
126 MB L2, so no flush runs between steps.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from datetime import datetime, timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent
PKG = ROOT / "ascend-spmm_b200"
for _p in (PKG, ROOT, ROOT / "oracle"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

import torch  # noqa: E402

import workloads  # noqa: E402

METRIC = "SpMM GFLOP/s (2*nnz*N) and HBM GB/s vs roofline at 1/2/4/8 B200"
UNIT = "GFLOP/s"
FALLBACK_HBM_GBS = 6650.0


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=1000)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--config", type=int, default=2)
    p.add_argument("--scale", type=float, default=1.0)
    p.add_argument("--op", choices=("csr", "mixed"), default="csr")
    p.add_argument("--scaling", choices=("weak", "strong"), default="weak")
    p.add_argument("--e2e-steps", type=int, default=24)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-e2e", action="store_true", help="skip the host-buffer end-to-end leg")
    p.add_argument("--gather", action="store_true",
                   help="also time the optional NCCL all-gather of the row-sharded C (reported separately)")
    return p.parse_args()


# --------------------------------------------------------------------------
# distributed plumbing
# --------------------------------------------------------------------------

def dist_setup(gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def allreduce_max(x: float, world) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def allreduce_sum(x: float, world) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


# --------------------------------------------------------------------------
# clocks during the timed region
# --------------------------------------------------------------------------

class ClockSampler:
    """nvidia-smi clock/throttle samples (every 50 ms) of one GPU.  Entering
    starts the sampler and waits (up to 5 s) for its first sample; mark(t0)
    and mark(t1) bracket the timed region, and summary() keeps the samples
    from 0.3 s before it (the warm-up steps that run under the sampler right
    before timing) to its end."""
    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.file = None
        self.t0 = self.t1 = None

    def __enter__(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=self.file, stderr=subprocess.DEVNULL)
            t_end = time.time() + 5.0
            while time.time() < t_end and os.path.getsize(self.file.name) == 0 and self.proc.poll() is None:
                time.sleep(0.02)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def mark(self, start):
        if start:
            self.t0 = datetime.now()
        else:
            self.t1 = datetime.now()

    def summary(self):
        if self.proc is None or self.file is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.file.flush()
        rows, every = [], []
        with open(self.file.name) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) < 10:
                    continue
                every.append(parts[1:])
                try:
                    ts = datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f")
                except ValueError:
                    continue
                if self.t0 is None or self.t1 is None or \
                        self.t0 - timedelta(seconds=0.3) <= ts <= self.t1 + timedelta(seconds=0.05):
                    rows.append(parts[1:])
        os.unlink(self.file.name)
        window = "timed region and the 0.3 s of warm-up before it"
        if not rows and every:   # timestamps unreadable: keep the whole sampler run
            rows, window = every, "warm-up and timed region"
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        pw = [float(r[3]) for r in rows if r[3].replace(".", "").isdigit()]
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows), "power_w_max": max(pw) if pw else None,
                "window": window}


def peak_hbm():
    try:
        d = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def traffic_per_launch(key: str, units: float):
    """DRAM bytes per launch from a committed ncu summary, scaled by units."""
    try:
        d = json.loads((ROOT / "profiles" / "traffic.json").read_text())
        e = d[key]
        return e["dram_bytes_per_unit"] * units
    except Exception:
        return None


# --------------------------------------------------------------------------
# CPU baseline: the reference's CPU SpMM (torch.sparse.mm, fp32, all threads)
# --------------------------------------------------------------------------

def cpu_reference_rate(w: "workloads.Workload", target_s=1.0, max_rows=None):
    import oracle

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    rowptr = w.rowptr.cpu()
    col, val, B = w.col.cpu(), w.val.cpu(), w.B.cpu()
    Bf = B.float()

    def run(rows):
        rp, c, v = workloads.row_slice(workloads.Workload(w.name, w.M, w.K, w.N, w.dtype, rowptr, col, val, B, {}),
                                        0, rows)
        t = time.perf_counter()
        oracle.cpu_reference(rows, w.K, rp.to(torch.int64), c.to(torch.int64), v, Bf)
        return time.perf_counter() - t, int(rp[-1])

    rows = min(w.M, max_rows or w.M, 4096)
    dt, nz = run(rows)
    while dt < 0.2 and rows < w.M:
        rows = min(w.M, rows * 4)
        dt, nz = run(rows)
    rows = min(w.M, max(1, int(rows * target_s / max(dt, 1e-6))))
    return rows, threads, Bf, rowptr, col, val


# --------------------------------------------------------------------------
# our arm
# --------------------------------------------------------------------------

def run_ours(args, rank, world, local):
    import spmm_npu

    dev = torch.device("cuda", local)
    from spmm_dist import allgather_rows, shard_bounds

    if args.scaling == "weak":
        w = workloads.make(args.config, device=dev, scale=args.scale, seed=workloads.DEFAULT_SEED + rank)
        B = w.B if rank == 0 else workloads.make(args.config, device=dev, scale=args.scale).B
        rp, col, val = w.rowptr, w.col, w.val
        bounds = [(k * w.M, (k + 1) * w.M) for k in range(world)]
        nnz_global = int(allreduce_sum(float(w.nnz), world))
    else:
        w = workloads.make(args.config, device=dev, scale=args.scale)
        bounds = shard_bounds(w.rowptr, world)
        r0, r1 = bounds[rank]
        rp, col, val = workloads.row_slice(w, r0, r1)
        B = w.B
        nnz_global = w.nnz
    rp, col, val = rp.contiguous(), col.contiguous(), val.contiguous()
    M_local, nnz_local = int(rp.numel()) - 1, int(col.numel())
    start = torch.zeros(40, dtype=torch.int32, device=dev)

    mixed = None
    if args.op == "mixed":
        m = spmm_npu.preprocess(rp, col, val, M_local, w.K, 16, False)
        mixed = [m[k] for k in ("crow_window_ptr", "unique_col_ids", "value", "vrow_window_ptr",
                                "vcol_indices", "vvalue")]

    def step():
        if mixed is None:
            return spmm_npu.spmm_csr(rp, col, val, B, start)
        return spmm_npu.spmm_ascend_cube(*mixed, B, start[:20], start)

    stream = torch.cuda.current_stream()
    with ClockSampler(local) as clk:   # sampling from before the warm-up on
        for _ in range(max(3, args.warmup)):
            step()
        torch.cuda.synchronize()
        code, detail = spmm_npu.device_status(True)
        assert code == 0, (code, detail)

        # ---- device-timed region ---------------------------------------
        barrier(world)
        torch.cuda.synchronize()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        clk.mark(True)
        ev0.record(stream)
        for _ in range(args.steps):
            step()
        ev1.record(stream)
        torch.cuda.synchronize()
        clk.mark(False)
    barrier(world)
    ms_local = ev0.elapsed_time(ev1)
    ms_total = allreduce_max(ms_local, world)
    ms_step = ms_total / args.steps
    flops = 2.0 * nnz_global * w.N
    value = flops * args.steps / (ms_total * 1e-3) / 1e9

    # roofline of the dominant kernel (this rank's launches)
    s = torch.finfo(w.dtype).bits // 8
    bytes_local = 4 * (M_local + 1) + nnz_local * (4 + s) + nnz_local * w.N * s + M_local * w.N * s
    achieved = bytes_local / (ms_local / args.steps * 1e-3) / 1e9
    peak, peak_kind = peak_hbm()
    traffic = traffic_per_launch(f"{w.name}:{args.op}", nnz_local)

    out = {}
    if args.gather and world > 1:
        y = step()
        allgather_rows(y, bounds)
        torch.cuda.synchronize()
        barrier(world)
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record(stream)
        for _ in range(5):
            full = allgather_rows(y, bounds)
        g1.record(stream)
        torch.cuda.synchronize()
        gms = allreduce_max(g0.elapsed_time(g1), world) / 5
        out["allgather"] = {"ms": round(gms, 3), "bytes": int(full.numel() * full.element_size()),
                            "note": "optional full-C all-gather over NCCL, not part of value"}
    if not args.no_e2e:
        out["e2e"] = run_e2e(args, w, rp, col, val, B, start, step, dev, world, flops)

    launches_per_step = count_own_kernels(step)
    out = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True,
        "scaling": args.scaling, "vs_baseline": None, "dtype": "f16 (fp32 accumulate)" if s == 2 else "f32",
        "data": "synthetic (seeded generator, BASELINE config shapes)",
        "config": {"workload": (f"{w.name} M=K={w.M} nnz={w.nnz} N={w.N}" if args.scaling == "strong" or world == 1
                                else f"{world} row blocks of {w.name} (M=K={w.M}, seeds {workloads.DEFAULT_SEED}"
                                     f"+rank), {nnz_global} nnz in all, N={w.N}"),
                   "op": "spmm_csr" if mixed is None else "spmm_ascend_cube(preprocess)",
                   "parallelism": f"row-shard x{world} (B replicated, C row-sharded)",
                   "l2": f"inputs larger than L2 (B {B.numel() * B.element_size() / 1e6:.0f} MB), no flush",
                   "generator": w.params},
        "gb_per_s": round(bytes_local / (ms_step * 1e-3) / 1e9, 1) if world == 1 else None,
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": traffic,
                     "peak_source": f"{peak_kind} hbm_gbs", "algorithmic_bytes_per_launch": bytes_local},
        **out,
        "gpu_launches": launches_per_step * args.steps if launches_per_step is not None else None,
        "clocks": clk.summary(),
    }

    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_baseline(w)
    if rank == 0:
        print(json.dumps(out), flush=True)


def count_own_kernels(step):
    """Kernels of this library (namespace spmmb) that one step launches,
    counted from the CUDA activity trace of one untimed step."""
    import warnings

    from torch.profiler import ProfilerActivity, profile

    torch.cuda.synchronize()
    try:
        with warnings.catch_warnings():
            warnings.simplefilter("ignore")
            with profile(activities=[ProfilerActivity.CUDA]) as prof:
                step()
                torch.cuda.synchronize()
        names = [e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA]
    except Exception as exc:   # no CUDA activity tracing in this process
        print(f"gpu_launches: kernel trace unavailable ({exc})", file=sys.stderr)
        return None
    return sum(1 for n in names if "spmmb::" in n)


def run_e2e(args, w, rp, col, val, B, start, step, dev, world, flops):
    """Same SpMM through the public API with HOST inputs: every step copies
    A (rowptr, col, val) and B from pinned host memory, runs spmm_csr and
    reads C back into pinned host memory, all inside the timed region.

    Steps are pipelined two deep, as a serving loop would run them: step i's
    host-to-device copies (copy stream) overlap step i-1's kernel and its
    device-to-host copy of C (a second copy stream), each step with its own
    buffer set; PCIe carries both directions at once."""
    import spmm_npu

    M_local = rp.numel() - 1
    pin = lambda t: t.cpu().pin_memory()  # noqa: E731
    h_in = [pin(t) for t in (rp, col, val, B)]
    h_out = [torch.empty((M_local, w.N), dtype=w.dtype).pin_memory() for _ in range(2)]
    d_in = [[torch.empty_like(t, device=dev) for t in (rp, col, val, B)] for _ in range(2)]
    s_in, s_comp, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    comp_done = [torch.cuda.Event() for _ in range(2)]
    d2h_done = [torch.cuda.Event() for _ in range(2)]
    started = [False, False]
    ys = [None, None]

    # Buffer reuse is ordered by events (no record_stream): step i's result
    # replaces that of step i-2 only after its device-to-host copy is done,
    # so the caching allocator hands the same block back without new
    # allocations inside the timed region.
    def e2e_step(i):
        k = i % 2
        with torch.cuda.stream(s_in):
            if started[k]:
                s_in.wait_event(comp_done[k])          # the kernel of step i-2 has read buffer set k
            for d, h in zip(d_in[k], h_in):
                d.copy_(h, non_blocking=True)
        s_comp.wait_stream(s_in)
        with torch.cuda.stream(s_comp):
            if started[k]:
                s_comp.wait_event(d2h_done[k])         # step i-2's result has been read back
            ys[k] = None
            ys[k] = spmm_npu.spmm_csr(*d_in[k][:3], d_in[k][3], start)
            comp_done[k].record(s_comp)
        started[k] = True
        s_out.wait_stream(s_comp)
        with torch.cuda.stream(s_out):
            h_out[k].copy_(ys[k], non_blocking=True)
            d2h_done[k].record(s_out)

    for i in range(2):
        e2e_step(i)
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s_in)
    s_comp.wait_stream(s_in)
    s_out.wait_stream(s_in)
    for i in range(args.e2e_steps):
        e2e_step(i)
    s_out.wait_stream(s_in)
    s_out.wait_stream(s_comp)
    e1.record(s_out)
    torch.cuda.synchronize()
    barrier(world)
    e2e_ms = allreduce_max(e0.elapsed_time(e1), world)
    e2e_value = flops * args.e2e_steps / (e2e_ms * 1e-3) / 1e9
    h2d = allreduce_sum(float(sum(t.numel() * t.element_size() for t in h_in)), world)
    d2h = allreduce_sum(float(h_out[0].numel() * h_out[0].element_size()), world)
    ref = spmm_npu.spmm_csr(rp, col, val, B, start)
    torch.cuda.synchronize()
    assert torch.equal(h_out[(args.e2e_steps - 1) % 2].to(dev), ref), "e2e result differs from the resident run"
    return {"value": round(e2e_value, 2), "unit": UNIT, "h2d_bytes_per_step": int(h2d),
            "d2h_bytes_per_step": int(d2h), "steps": args.e2e_steps,
            "pipeline": "2 steps in flight: H2D of step i overlaps kernel + D2H of step i-1 (pinned host buffers)"}


def cpu_baseline(w):
    import oracle

    rows, threads, Bf, rowptr, col, val = cpu_reference_rate(w, target_s=1.5)
    rp, c, v = workloads.row_slice(workloads.Workload(w.name, w.M, w.K, w.N, w.dtype, rowptr, col, val, w.B.cpu(),
                                                      {}), 0, rows)
    rp64, c64 = rp.to(torch.int64), c.to(torch.int64)
    times = []
    t_end = time.perf_counter() + 12.0
    while time.perf_counter() < t_end or len(times) < 3:
        t = time.perf_counter()
        oracle.cpu_reference(rows, w.K, rp64, c64, v, Bf)
        times.append(time.perf_counter() - t)
        if len(times) >= 20:
            break
    t = statistics.median(times)
    gflops = 2.0 * int(rp[-1]) * w.N / t / 1e9
    return {"value": round(gflops, 3), "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"rows [0, {rows}) of {w.name} ({int(rp[-1])} nnz, N={w.N}), torch.sparse.mm fp32, "
                      f"median of {len(times)} runs",
            "impl": "tests/aic_aiv_ablation/common.py:173-177 cpu_reference restated"}


# --------------------------------------------------------------------------
# reference arm
# --------------------------------------------------------------------------

def run_reference(args, rank, world):
    if rank != 0:
        return
    import oracle

    dev = "cuda" if torch.cuda.is_available() else "cpu"
    w = workloads.make(args.config, device=dev, scale=args.scale)
    rows, threads, Bf, rowptr, col, val = cpu_reference_rate(w, target_s=0.5)
    rp, c, v = workloads.row_slice(workloads.Workload(w.name, w.M, w.K, w.N, w.dtype, rowptr, col, val, w.B.cpu(),
                                                      {}), 0, rows)
    rp64, c64 = rp.to(torch.int64), c.to(torch.int64)
    for _ in range(args.warmup):
        oracle.cpu_reference(rows, w.K, rp64, c64, v, Bf)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        oracle.cpu_reference(rows, w.K, rp64, c64, v, Bf)
    dt = time.perf_counter() - t0
    nz = int(rp[-1])
    value = 2.0 * nz * w.N * args.steps / dt / 1e9
    sample = f"rows [0, {rows}) of {w.name} ({nz} of {w.nnz} nnz, N={w.N}) per step"
    out = {
        "metric": METRIC, "value": round(value, 3), "unit": UNIT, "impl": "reference", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 3),
        "higher_is_better": True, "scaling": args.scaling, "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded generator, BASELINE config shapes)",
        "config": {"workload": f"{w.name} M=K={w.M} nnz={w.nnz} N={w.N}", "op": "torch.sparse.mm (cpu_reference)",
                   "parallelism": f"host CPU, {threads} threads"},
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(out), flush=True)


def main():
    args = parse_args()
    rank, world, local = dist_setup(args.gpus)
    try:
        if args.impl == "reference":
            run_reference(args, rank, world)
        else:
            run_ours(args, rank, world, local)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
