#!/usr/bin/env python
"""Benchmark of the SpMM hot path (driver contract).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config 5] [--op csr|mixed|preprocess] [--scaling strong|weak]

Default step: one SpMM C = A @ B of BASELINE config 5, the largest
configuration that fits one B200 (16.8M x 16.8M power-law matrix, ~469M
nonzeros after de-duplication, fp16 values, B = 16.8M x 1024 fp16, about
72 GB with C), inputs resident in HBM, through ``spmm_csr``.  With N GPUs
(torchrun, one rank per GPU) the matrix is cut into N row ranges balanced by
nonzeros at 16-row window boundaries (``--scaling strong``, the default:
total work fixed) or every rank owns one config-sized row block of a global
matrix (``--scaling weak``); B is replicated and C stays row-sharded, so no
collective runs in the timed region.  ``--gather`` times the optional full-C
all-gather separately.

The JSON line carries, besides the contract keys:
* ``roofline``: per-nnz-model bytes (the graded algorithmic figure) over the
  dominant kernel's time, the compulsory bytes (A and C once, each distinct
  B row once) over the same time, and the DRAM traffic of one launch from a
  committed ncu capture (``profiles/traffic.json``) over that time;
* ``kernels``: per-kernel share of a step from a CUDA activity trace of
  untimed steps (the dominant kernel's time is the step time times its
  share);
* ``e2e``: the same SpMM through ``spmm_csr`` with the inputs copied from
  pinned host memory and C copied back every step;
* ``cpu_baseline``: the reference's CPU SpMM path on the box's host cores on
  a leading-row sample: torch.sparse.mm in fp32 on all threads (the
  reference's ``cpu_reference``, tests/aic_aiv_ablation/common.py:173-177)
  and SciPy CSR @ dense single-threaded; the faster one is the value;
* ``preprocess``: the GPU layout builders against the reference's own
  compiled CPU preprocessing (single-threaded) on config 2.

``--impl reference`` times the reference's CPU SpMM path (torch.sparse.mm,
fp32, all host threads) on the same leading-row sample, on rank 0 only.
B (34 GB) is far larger than the 126 MB L2, so no flush runs between steps.
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
CPU_SAMPLE_NNZ = 8_000_000      # nonzeros of the leading-row CPU sample


def parse_args(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=100)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--config", type=int, default=5)
    p.add_argument("--scale", type=float, default=1.0)
    p.add_argument("--op", choices=("csr", "mixed", "preprocess"), default="csr")
    p.add_argument("--scaling", choices=("strong", "weak"), default="strong")
    p.add_argument("--e2e-steps", type=int, default=16)
    p.add_argument("--e2e-outputs", type=int, choices=(1, 2), default=2,
                   help="device outputs in the e2e pipeline (1: a step's kernel waits for the previous read-back)")
    p.add_argument("--preprocess-config", type=int, default=2)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-e2e", action="store_true", help="skip the host-buffer end-to-end leg")
    p.add_argument("--no-preprocess", action="store_true", help="skip the layout-builder leg")
    p.add_argument("--gather", action="store_true",
                   help="also time the optional NCCL all-gather of the row-sharded C (reported separately)")
    return p.parse_args(argv)


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


def allreduce(x: float, world, op="max") -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op={"max": dist.ReduceOp.MAX, "min": dist.ReduceOp.MIN, "sum": dist.ReduceOp.SUM}[op])
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
    """DRAM bytes of one launch of the dominant kernel, from a committed ncu
    capture (``profiles/traffic.json``: bytes per nonzero), times units."""
    try:
        e = json.loads((ROOT / "profiles" / "traffic.json").read_text())[key]
        return e["dram_bytes_per_unit"] * units, e.get("source")
    except Exception:
        return None, None


def l2_plan_probe(rp, col, val, B, out):
    """The L2 residency plan of one spmm_csr launch (untimed), read back
    through the C ABI: whether this problem reserves a plan, whether it
    engaged (hot columns hold at least a quarter of the sampled nonzeros),
    the hot column bins and their share of the samples.  ``out`` receives
    the product (the same bits as the timed steps)."""
    import ctypes

    import build

    L = ctypes.CDLL(str(build.LIB))
    V, I64, INT, SZ = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_size_t
    L.spmm_csr_l2_plan_offset.restype = SZ
    L.spmm_csr_l2_plan_offset.argtypes = [I64, I64, I64, INT]
    L.spmm_csr_workspace_bytes.restype = SZ
    L.spmm_csr_workspace_bytes.argtypes = [I64, I64, I64, INT]
    L.spmm_csr_launch.restype = INT
    L.spmm_csr_launch.argtypes = [V, V, V, V, V, I64, V, I64, I64, I64, I64, INT, INT, V, SZ, V]
    M, K, N, nnz = rp.numel() - 1, B.shape[0], B.shape[1], col.numel()
    dt = 0 if B.dtype == torch.float16 else 1
    it = 0 if rp.dtype == torch.int32 else 1
    off = L.spmm_csr_l2_plan_offset(M, N, nnz, dt)
    if off == ctypes.c_size_t(-1).value:
        return {"reserved": False, "engaged": False}
    wb = L.spmm_csr_workspace_bytes(M, N, nnz, dt)
    ws = torch.empty(wb, dtype=torch.uint8, device=B.device)
    rc = L.spmm_csr_launch(rp.data_ptr(), col.data_ptr(), val.data_ptr(), B.data_ptr(), None, 0, out.data_ptr(),
                           M, K, N, nnz, it, dt, ws.data_ptr(), wb, torch.cuda.current_stream().cuda_stream)
    if rc != 0:
        return {"reserved": True, "error": rc}
    h = ws[off: off + 32].cpu().numpy().view("<u4")
    threshold, hot_bins, budget = int(h[0]), int(h[1]), int(h[2])
    samples, hot = int(h[4]) | (int(h[5]) << 32), int(h[6]) | (int(h[7]) << 32)
    del ws
    return {"reserved": True, "engaged": bool(threshold > 0 and samples > 0 and 4 * hot >= samples),
            "hot_column_bins": hot_bins, "budget_bins": budget, "threshold_samples": threshold,
            "samples": samples, "hot_sample_fraction": round(hot / samples, 4) if samples else 0.0}


def value_bytes(dtype) -> int:
    return torch.finfo(dtype).bits // 8


def algorithmic_bytes(M, nnz, N, s) -> int:
    """Per-nnz gather model: 4(M+1) + nnz(4 + s) + nnz*N*s + M*N*s."""
    return 4 * (M + 1) + nnz * (4 + s) + nnz * N * s + M * N * s


def compulsory_bytes(M, col, N, s, K) -> int:
    """A once, C once and each distinct B row once."""
    nnz = int(col.numel())
    distinct = int((torch.bincount(col.to(torch.int64), minlength=K) > 0).sum()) if nnz else 0
    return 4 * (M + 1) + nnz * (4 + s) + distinct * N * s + M * N * s


# --------------------------------------------------------------------------
# per-kernel shares from a CUDA activity trace
# --------------------------------------------------------------------------

def kernel_trace(step, steps=3):
    """Device time per kernel name of this library (namespace spmmb) over a
    few untimed steps: {name: (launches per step, microseconds per step)}."""
    import warnings

    from torch.profiler import ProfilerActivity, profile

    torch.cuda.synchronize()
    try:
        with warnings.catch_warnings():
            warnings.simplefilter("ignore")
            with profile(activities=[ProfilerActivity.CUDA]) as prof:
                for _ in range(steps):
                    step()
                torch.cuda.synchronize()
        out = {}
        for e in prof.key_averages():
            if "spmmb::" not in e.key:
                continue
            us = getattr(e, "device_time_total", None)
            if us is None:
                us = getattr(e, "cuda_time_total", 0.0)
            n, t = out.get(e.key, (0, 0.0))
            out[e.key] = (n + e.count / steps, t + us / steps)
        return out
    except Exception as exc:   # no CUDA activity tracing in this process (e.g. under ncu)
        print(f"kernel trace unavailable ({exc})", file=sys.stderr)
        return None


def short_name(kernel: str) -> str:
    """Kernel name without return type, namespaces and parameter list."""
    k = kernel.replace("void ", "").replace("(anonymous namespace)::", "").replace("spmmb::", "")
    k = k.replace("unnamed>::", "")
    depth, out = 0, []
    for ch in k:   # cut at the parameter list: the first "(" outside template brackets
        if ch == "<":
            depth += 1
        elif ch == ">":
            depth -= 1
        elif ch == "(" and depth == 0:
            break
        out.append(ch)
    return "".join(out).strip()


# --------------------------------------------------------------------------
# CPU baseline: the reference's CPU SpMM on a leading-row sample
# --------------------------------------------------------------------------

def cpu_sample(w, target_nnz=CPU_SAMPLE_NNZ):
    """Rows [0, R) of w holding about target_nnz nonzeros, on the host in
    fp32, with only the B rows the sample touches (columns relabelled to
    compact ids; the work - nonzeros and features - is unchanged)."""
    rp64 = w.rowptr.to(torch.int64)
    R = int(torch.searchsorted(rp64, torch.tensor([target_nnz], device=rp64.device)).item())
    R = max(1, min(w.M, R))
    rp, c, v = workloads.row_slice(w, 0, R)
    uniq, inv = torch.unique(c.to(torch.int64), return_inverse=True)
    Bs = w.B.index_select(0, uniq).float().cpu()
    return {"rows": R, "rowptr": rp.to(torch.int64).cpu(), "col": inv.to(torch.int64).cpu(),
            "val": v.float().cpu(), "B": Bs, "nnz": int(c.numel()), "distinct_cols": int(uniq.numel()),
            "desc": f"rows [0, {R}) of {w.name} ({int(c.numel())} of {w.nnz} nonzeros, "
                    f"{int(uniq.numel())} distinct B rows gathered, N={w.N}); GFLOP/s is "
                    f"extrapolated to the whole matrix linearly in nonzeros"}


FEATURE_CHUNK = 128   # dense columns per CPU library call


def feature_chunks(Bs):
    """B split into contiguous feature blocks: the host libraries address the
    dense operand with 32-bit offsets (torch.sparse.mm's MKL kernel segfaults
    past 2^31 elements), so each call gets one block of FEATURE_CHUNK
    features; the work (2 * nnz * N) is unchanged."""
    return [Bs[:, f:f + FEATURE_CHUNK].contiguous() for f in range(0, Bs.shape[1], FEATURE_CHUNK)]


def torch_cpu_spmm(smp, chunks):
    import oracle

    for Bc in chunks:
        oracle.cpu_reference(smp["rows"], Bc.shape[0], smp["rowptr"], smp["col"], smp["val"], Bc)


def time_runs(fn, budget_s, min_runs=3, max_runs=50):
    fn()   # warm
    times = []
    t_end = time.perf_counter() + budget_s
    while (time.perf_counter() < t_end or len(times) < min_runs) and len(times) < max_runs:
        t = time.perf_counter()
        fn()
        times.append(time.perf_counter() - t)
    return statistics.median(times), len(times)


def cpu_baseline(w):
    import scipy.sparse as sp

    smp = cpu_sample(w)
    chunks = feature_chunks(smp.pop("B"))
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    flops = 2.0 * smp["nnz"] * w.N
    t_torch, n_torch = time_runs(lambda: torch_cpu_spmm(smp, chunks), 6.0)
    A = sp.csr_matrix((smp["val"].numpy(), smp["col"].numpy().astype("int64"), smp["rowptr"].numpy().astype("int64")),
                      shape=(smp["rows"], chunks[0].shape[0]))
    Bn = [c.numpy() for c in chunks]
    t_scipy, n_scipy = time_runs(lambda: [A @ b for b in Bn], 6.0, min_runs=2)
    legs = {"torch.sparse.mm": {"gflops": round(flops / t_torch / 1e9, 3), "threads": threads, "runs": n_torch},
            "scipy.csr@dense": {"gflops": round(flops / t_scipy / 1e9, 3), "threads": 1, "runs": n_scipy}}
    best = max(legs, key=lambda k: legs[k]["gflops"])
    return {"value": legs[best]["gflops"], "unit": UNIT, "cores": legs[best]["threads"], "kind": "port",
            "impl": best, "legs": legs, "host_cpus": threads,
            "sample": smp["desc"] + f"; fp32, dense operand in blocks of {FEATURE_CHUNK} features per call; "
                                    "median of timed runs",
            "reference": "tests/aic_aiv_ablation/common.py:173-177 cpu_reference restated (torch.sparse.mm); "
                         "SciPy single-threaded alongside"}


# --------------------------------------------------------------------------
# preprocessing: GPU layout builders vs the reference's compiled CPU code
# --------------------------------------------------------------------------

class native_stdout_silenced:
    """Sends file descriptor 1 to /dev/null while the reference's compiled
    builders run (they print block counts from C++), so the bench's JSON
    line stays the only output."""

    def __enter__(self):
        sys.stdout.flush()
        self.saved = os.dup(1)
        self.null = os.open(os.devnull, os.O_WRONLY)
        os.dup2(self.null, 1)
        return self

    def __exit__(self, *exc):
        sys.stdout.flush()
        os.dup2(self.saved, 1)
        os.close(self.saved)
        os.close(self.null)


def preprocess_leg(cfg, dev):
    """Times each GPU layout builder (CUDA events, median of 5) on config
    ``cfg`` against the same function of the reference's compiled CPU code
    (oracle/_ref, single-threaded; the C restatement when it is absent) on
    the same input, and checks that the layouts agree."""
    import spmm_npu

    w = workloads.make(cfg, device=dev)
    M, K = w.M, w.K
    rp, col, val = w.rowptr, w.col, w.val
    ratio = (222.0 / 190.0) * 0.5
    gpu_fns = {
        "preprocess": lambda: spmm_npu.preprocess(rp, col, val, M, K, 16, False),
        "preprocess(graph_layout)": lambda: spmm_npu.preprocess(rp, col, val, M, K, 16, True),
        "csr_to_bcsr": lambda: spmm_npu.csr_to_bcsr(rp, col, val, M, K, 16),
        "block_level_split": lambda: spmm_npu.block_level_split(rp, col, val, M, K, ratio, 16),
    }
    ref, kind = None, "reference"
    try:
        import build_ref

        ref = build_ref.load()
    except Exception as exc:   # the compiled reference could not be loaded here
        print(f"oracle/_ref unavailable ({exc}); timing the C restatement", file=sys.stderr)
    if ref is None:
        import oracle as ref
        kind = "port"
    h = [t.cpu() for t in (rp, col, val)]
    cpu_fns = {
        "preprocess": lambda: ref.preprocess(*h, M, K, 16, False),
        "preprocess(graph_layout)": lambda: ref.preprocess(*h, M, K, 16, True),
        "csr_to_bcsr": lambda: ref.csr_to_bcsr(*h, M, K, 16),
        "block_level_split": lambda: ref.block_level_split(*h, M, K, ratio, 16),
    }
    torch.set_num_threads(1)
    out = {"config": f"{w.name} M=K={M} nnz={w.nnz} ({w.dtype})", "cpu_kind": kind, "cpu_threads": 1,
           "builders": {}}
    for name, fn in gpu_fns.items():
        got = fn()
        torch.cuda.synchronize()
        times = []
        for _ in range(5):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            times.append(e0.elapsed_time(e1))
        gms = statistics.median(times)
        with native_stdout_silenced():
            t = time.perf_counter()
            want = cpu_fns[name]()
            cms = (time.perf_counter() - t) * 1e3
        same = all(torch.equal(got[k].cpu(), want[k].cpu()) for k in want
                   if torch.is_tensor(want[k]) and k in got)
        out["builders"][name] = {"gpu_ms": round(gms, 3), "cpu_ms": round(cms, 1),
                                 "speedup": round(cms / gms, 1), "layouts_equal": bool(same)}
    return out


# --------------------------------------------------------------------------
# our arm
# --------------------------------------------------------------------------

def local_problem(args, rank, world, dev):
    """This rank's CSR rows, B and the global nonzero count."""
    from spmm_dist import shard_bounds

    if args.scaling == "weak":
        w = workloads.make(args.config, device=dev, scale=args.scale, seed=workloads.DEFAULT_SEED + rank)
        if rank != 0:   # B is the seed-2027 operand on every rank
            w.B = workloads.make(args.config, device=dev, scale=args.scale).B
        rp, col, val = w.rowptr, w.col, w.val
        bounds = [(k * w.M, (k + 1) * w.M) for k in range(world)]
        nnz_global = int(allreduce(float(w.nnz), world, "sum"))
    else:
        w = workloads.make(args.config, device=dev, scale=args.scale)
        bounds = shard_bounds(w.rowptr, world)
        r0, r1 = bounds[rank]
        rp, col, val = workloads.row_slice(w, r0, r1)
        nnz_global = w.nnz
    return w, rp.contiguous(), col.contiguous(), val.contiguous(), bounds, nnz_global


def run_ours(args, rank, world, local):
    import spmm_npu
    from spmm_dist import allgather_rows

    dev = torch.device("cuda", local)
    w, rp, col, val, bounds, nnz_global = local_problem(args, rank, world, dev)
    B = w.B
    M_local, nnz_local = int(rp.numel()) - 1, int(col.numel())
    start = torch.zeros(40, dtype=torch.int32, device=dev)

    mixed = None
    if args.op == "mixed":
        m = spmm_npu.preprocess(rp, col, val, M_local, w.K, 16, False)
        mixed = [m[k] for k in ("crow_window_ptr", "unique_col_ids", "value", "vrow_window_ptr",
                                "vcol_indices", "vvalue")]
        del m

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
    ms_total = allreduce(ms_local, world, "max")
    ms_step = ms_total / args.steps
    flops = 2.0 * nnz_global * w.N
    value = flops * args.steps / (ms_total * 1e-3) / 1e9

    # ---- per-kernel shares (untimed steps) and the roofline of the dominant kernel
    trace = kernel_trace(step)
    kernels = None
    dom_name, dom_share = None, 1.0
    if trace:
        tot = sum(t for _, t in trace.values()) or 1.0
        kernels = {short_name(k): {"launches_per_step": round(n, 2), "us_per_step": round(t, 1),
                                   "share": round(t / tot, 4)} for k, (n, t) in trace.items()}
        dom = max(trace, key=lambda k: trace[k][1])
        dom_name, dom_share = short_name(dom), trace[dom][1] / tot
    launches_per_step = sum(n for n, _ in trace.values()) if trace else None
    s = value_bytes(w.dtype)
    kernel_s = ms_local / args.steps * 1e-3 * dom_share
    algo = algorithmic_bytes(M_local, nnz_local, w.N, s)
    comp = compulsory_bytes(M_local, col, w.N, s, w.K)
    peak, peak_kind = peak_hbm()
    key = f"{w.name}:{args.op}"
    l2_plan = None
    if mixed is None:   # spmm_csr: did the L2 residency plan engage (its traffic was measured apart)
        l2_plan = l2_plan_probe(rp, col, val, B, step())
        torch.cuda.synchronize()
        if not l2_plan.get("engaged"):
            key += ":no_l2_plan"
    traffic, traffic_src = traffic_per_launch(key, nnz_local)
    roofline = {
        "bound": "hbm", "achieved": round(algo / kernel_s / 1e9, 1), "peak": peak, "unit": "GB/s",
        "frac": round(algo / kernel_s / 1e9 / peak, 4),
        "traffic": round(traffic) if traffic else None,
        "kernel": dom_name, "kernel_ms": round(kernel_s * 1e3, 4),
        "peak_source": f"{peak_kind} hbm_gbs (MEASURED_PEAKS.json)",
        "algorithmic_bytes": algo,
        "algorithmic_model": "per-nnz gather: 4(M+1) + nnz(4+s) + nnz*N*s + M*N*s",
        "compulsory_bytes": comp,
        "compulsory_frac": round(comp / kernel_s / 1e9 / peak, 4),
        "dram_gbs": round(traffic / kernel_s / 1e9, 1) if traffic else None,
        "dram_frac": round(traffic / kernel_s / 1e9 / peak, 4) if traffic else None,
        "traffic_source": traffic_src,
    }
    if l2_plan is not None:
        roofline["l2_plan"] = l2_plan

    extra = {}
    if args.gather and world > 1:
        y = step()
        allgather_rows(y, bounds)
        torch.cuda.synchronize()
        barrier(world)
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record(stream)
        for _ in range(3):
            full = allgather_rows(y, bounds)
        g1.record(stream)
        torch.cuda.synchronize()
        gms = allreduce(g0.elapsed_time(g1), world, "max") / 3
        extra["allgather"] = {"ms": round(gms, 3), "bytes": int(full.numel() * full.element_size()),
                              "note": "optional full-C all-gather over NCCL, not part of value"}
        del y
        extra["allgather"]["fused_multicast"] = fused_multicast_leg(rp, col, val, B, bounds, rank, world, dev,
                                                                    full, stream)
        del full
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        extra["cpu_baseline"] = cpu_baseline(w)
    if not args.no_e2e:
        inputs = [rp, col, val, B] if mixed is None else [*mixed, B]
        op = ((lambda a: spmm_npu.spmm_csr(*a[:3], a[3], start)) if mixed is None
              else (lambda a: spmm_npu.spmm_ascend_cube(*a[:6], a[6], start[:20], start)))
        extra["e2e"] = run_e2e(args, w, inputs, op, dev, world, flops)
    if rank == 0 and not args.no_preprocess and args.op != "preprocess":
        extra["preprocess"] = preprocess_leg(args.preprocess_config, dev)

    out = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True,
        "scaling": args.scaling, "vs_baseline": None, "dtype": "f16 (fp32 accumulate)" if s == 2 else "f32",
        "data": "synthetic (seeded generator, BASELINE config shapes)",
        "config": {"workload": (f"{w.name} M=K={w.M} nnz={w.nnz} N={w.N}" if args.scaling == "strong"
                                else f"{world} row blocks of {w.name} (M=K={w.M}, seeds {workloads.DEFAULT_SEED}"
                                     f"+rank), {nnz_global} nnz in all, N={w.N}"),
                   "op": "spmm_csr" if mixed is None else "spmm_ascend_cube(preprocess)",
                   "parallelism": f"row-shard x{world} (B replicated, C row-sharded, no collective timed)",
                   "rank0_rows": M_local, "rank0_nnz": nnz_local,
                   "l2": f"inputs larger than L2 (B {B.numel() * B.element_size() / 1e6:.0f} MB), no flush",
                   "generator": w.params},
        "gb_per_s": round(algorithmic_bytes(M_local, nnz_local, w.N, s) / (ms_step * 1e-3) / 1e9, 1),
        "roofline": roofline,
        "kernels": kernels,
        **extra,
        "gpu_launches": round(launches_per_step * args.steps) if launches_per_step is not None else None,
        "clocks": clk.summary(),
    }
    if rank == 0:
        print(json.dumps(out), flush=True)


def fused_multicast_leg(rp, col, val, B, bounds, rank, world, dev, full_nccl, stream):
    """The SpMM with the full-C gather fused into it: this rank's rows are
    stored by the CSR kernels through the NVLink multicast address of a
    symmetric-memory replica of C (``spmm_dist.MulticastRows``), between two
    stream-ordered barriers.  Timed like the NCCL leg (3 calls, max over
    ranks) and checked bit for bit against the NCCL all-gather result."""
    import custom_ops_lib
    from spmm_dist import MulticastRows, group_barrier

    r0, r1 = bounds[rank]
    rep, why = None, ""
    torch.cuda.empty_cache()   # the replica comes from the driver, not from torch's cache
    try:
        rep = MulticastRows(full_nccl.shape[0], full_nccl.shape[1], full_nccl.dtype, dev)
        ok = 1.0
    except RuntimeError as e:
        why, ok = str(e), 0.0
    if allreduce(ok, world, "min") < 1.0:
        if rep is not None:
            rep.close()
        barrier(world)
        return {"unavailable": why if not ok else "multicast replica unavailable on another rank"}
    out = rep.buf[r0:r1]

    def fused():
        group_barrier(device=dev)
        custom_ops_lib.spmm_csr_multicast(rp, col, val, B, out, rep.rows_mc(r0))
        group_barrier(device=dev)

    fused()
    torch.cuda.synchronize()
    same = allreduce(1.0 if torch.equal(rep.buf, full_nccl) else 0.0, world, "min") >= 1.0
    barrier(world)
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for _ in range(3):
        fused()
    f1.record(stream)
    torch.cuda.synchronize()
    fms = allreduce(f0.elapsed_time(f1), world, "max") / 3
    del out
    barrier(world)     # no rank writes the replicas any more
    rep.close()
    torch.cuda.synchronize()
    barrier(world)
    return {"ms": round(fms, 3), "equal_to_nccl_gather": same,
            "note": "SpMM + full-C replication in one kernel (multimem.st through NVSwitch), barriers included"}


def run_e2e(args, w, inputs, op, dev, world, flops):
    """The same SpMM through the public API with HOST buffers: every step
    copies the operator's inputs from pinned host memory into device memory,
    runs the operator and copies C back into pinned host memory, all inside
    the timed region.

    One pinned host set (config 5: 37 GB of inputs, 34 GB of output) and,
    device memory permitting, two device input sets (the resident tensors and
    one copy) and two device outputs, used alternately: step i+1's
    host-to-device copy overlaps step i's kernel and its device-to-host copy
    of C, and the kernel of step i+1 waits only for its inputs and for the
    read-back of C of step i-1 (whose output block it reuses), so in steady
    state a step costs the slower of the two host-link directions.  With one
    device input set the copy of step i+1 waits for the kernel of step i and
    the kernel waits for the read-back of step i.

    With several ranks, B (the last input, the same on every rank) crosses
    the host link once per step for the whole job: each rank uploads its
    1/N row block and an NCCL all-gather over NVLink assembles B on every
    GPU (in place), inside the timed step."""
    import psutil

    import torch.distributed as dist

    B = inputs[-1]
    rank = dist.get_rank() if world > 1 else 0
    shard_b = world > 1 and B.shape[0] % world == 0
    kb = B.shape[0] // world if shard_b else B.shape[0]
    b_rows = slice(rank * kb, (rank + 1) * kb) if shard_b else slice(0, B.shape[0])
    host_bytes = sum(t.numel() * t.element_size() for t in inputs[:-1]) + \
        B[b_rows].numel() * B.element_size()
    y0 = op(inputs)
    torch.cuda.synchronize()
    out_bytes = y0.numel() * y0.element_size()
    local_world = int(os.environ.get("LOCAL_WORLD_SIZE", str(world)))
    need = (host_bytes + out_bytes) * local_world
    avail = psutil.virtual_memory().available
    # one decision for all ranks (each then takes the same collective steps)
    fits = allreduce(1.0 if need <= 0.8 * avail else 0.0, world, "min")
    if fits < 1.0:
        del y0
        return {"skipped": f"pinned host buffers of {need / 1e9:.0f} GB for {local_world} local ranks exceed "
                           f"80% of the {avail / 1e9:.0f} GB of available host memory"}

    def pinned_copy(t):
        h = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
        h.copy_(t)
        return h

    h_in = [pinned_copy(t) for t in inputs[:-1]] + [pinned_copy(B[b_rows])]
    h_out = torch.empty(y0.shape, dtype=y0.dtype, pin_memory=True)
    del y0
    torch.cuda.empty_cache()
    free, _ = torch.cuda.mem_get_info(dev)
    set_bytes = sum(t.numel() * t.element_size() for t in inputs)
    two = allreduce(1.0 if free > set_bytes + 2 * out_bytes + (4 << 30) else 0.0, world, "min") >= 1.0
    sets = [inputs] + ([[torch.empty_like(t) for t in inputs]] if two else [])
    nset = len(sets)
    nout = min(nset, args.e2e_outputs)   # 2: the kernel of step i+1 never waits on the D2H of step i
    s_in, s_comp, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    in_done = [torch.cuda.Event() for _ in range(nset)]
    comp_done = [torch.cuda.Event() for _ in range(nset)]
    d2h_done = [torch.cuda.Event() for _ in range(nout)]
    state = {"y": [None] * nout, "step": 0, "used": [False] * nset, "out_used": [False] * nout}

    def e2e_step():
        k = state["step"] % nset
        o = state["step"] % nout
        with torch.cuda.stream(s_in):
            if state["used"][k]:
                s_in.wait_event(comp_done[k])    # the last kernel that read set k is done
            for d, h in zip(sets[k][:-1], h_in[:-1]):
                d.copy_(h, non_blocking=True)
            Bd = sets[k][-1]
            Bd[b_rows].copy_(h_in[-1], non_blocking=True)
            if shard_b:   # every rank's block to every GPU, over NVLink (in place)
                dist.all_gather_into_tensor(Bd, Bd[b_rows])
            in_done[k].record(s_in)
        with torch.cuda.stream(s_comp):
            s_comp.wait_event(in_done[k])
            if state["out_used"][o]:
                s_comp.wait_event(d2h_done[o])   # the result held in slot o has been read back
            state["y"][o] = None                 # its block may now be handed out again on s_comp
            state["y"][o] = op(sets[k])
            comp_done[k].record(s_comp)
        with torch.cuda.stream(s_out):
            s_out.wait_event(comp_done[k])
            h_out.copy_(state["y"][o], non_blocking=True)
            d2h_done[o].record(s_out)
        state["used"][k] = True
        state["out_used"][o] = True
        state["step"] += 1

    e2e_step()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s_in)
    s_comp.wait_stream(s_in)
    s_out.wait_stream(s_in)
    for _ in range(args.e2e_steps):
        e2e_step()
    s_out.wait_stream(s_in)
    s_out.wait_stream(s_comp)
    e1.record(s_out)
    torch.cuda.synchronize()
    barrier(world)
    e2e_ms = allreduce(e0.elapsed_time(e1), world, "max")
    e2e_value = flops * args.e2e_steps / (e2e_ms * 1e-3) / 1e9
    h2d = allreduce(float(host_bytes), world, "sum")
    d2h = allreduce(float(out_bytes), world, "sum")
    # the host copy of the last step equals a resident run (compared in slabs)
    state["y"] = [None] * nout
    del sets[1:]
    ref = op(inputs)
    torch.cuda.synchronize()
    slab = max(1, (1 << 30) // max(1, ref[0].numel() * ref.element_size()))
    for r in range(0, ref.shape[0], slab):
        assert torch.equal(h_out[r:r + slab].to(dev), ref[r:r + slab]), "e2e result differs from the resident run"
    del ref, h_in, h_out
    return {"value": round(e2e_value, 2), "unit": UNIT, "h2d_bytes_per_step": int(h2d),
            "d2h_bytes_per_step": int(d2h), "steps": args.e2e_steps, "ms_per_step": round(e2e_ms / args.e2e_steps, 2),
            "pipeline": f"pinned host buffers, {nset} device input set(s), {nout} output(s): H2D of step i+1 overlaps "
                        f"{'the kernel and ' if nset == 2 else ''}D2H of step i"
                        + (f"; B uploaded as {world} row blocks (one per rank) and all-gathered over NCCL"
                           if shard_b else "")}


def run_preprocess_only(args, rank, world, local):
    if rank != 0:
        return
    leg = preprocess_leg(args.preprocess_config, torch.device("cuda", local))
    print(json.dumps({"metric": "layout builders: GPU vs the reference's CPU preprocessing", "unit": "ms",
                      "higher_is_better": False, "n_gpus": 1, "preprocess": leg}), flush=True)


# --------------------------------------------------------------------------
# reference arm
# --------------------------------------------------------------------------

def run_reference(args, rank, world):
    if rank != 0:
        return
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    w = workloads.make(args.config, device=dev, scale=args.scale)
    smp = cpu_sample(w)
    workload = f"{w.name} M=K={w.M} nnz={w.nnz} N={w.N}"
    N = w.N
    del w
    chunks = feature_chunks(smp.pop("B"))
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)

    def one():
        torch_cpu_spmm(smp, chunks)

    for _ in range(args.warmup):
        one()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        one()
    dt = time.perf_counter() - t0
    value = 2.0 * smp["nnz"] * N * args.steps / dt / 1e9
    out = {
        "metric": METRIC, "value": round(value, 3), "unit": UNIT, "impl": "reference", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 3),
        "higher_is_better": True, "scaling": args.scaling, "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded generator, BASELINE config shapes)",
        "config": {"workload": workload, "sample": smp["desc"],
                   "op": "torch.sparse.mm (the reference's cpu_reference, tests/aic_aiv_ablation/common.py:173-177)",
                   "parallelism": f"host CPU, {threads} threads"},
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": smp["desc"] + f" per step; dense operand in blocks of {FEATURE_CHUNK} features"},
        "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(out), flush=True)


def main():
    args = parse_args()
    rank, world, local = dist_setup(args.gpus)
    try:
        if args.impl == "reference":
            run_reference(args, rank, world)
        elif args.op == "preprocess":
            run_preprocess_only(args, rank, world, local)
        else:
            run_ours(args, rank, world, local)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
