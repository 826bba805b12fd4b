"""Host logic of bench.py that needs no GPU: the clock record keeps only the
nvidia-smi samples of the timed region (plus the warm-up just before it) and
reports throttle reasons from them; unreadable timestamps fall back to every
sample; an empty record says so."""

import importlib.util
import sys
import tempfile
from datetime import datetime, timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def load_bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    argv = sys.argv
    sys.argv = ["bench.py"]
    try:
        spec.loader.exec_module(mod)
    finally:
        sys.argv = argv
    return mod


def sampler_with(lines, t0, t1):
    bench = load_bench()
    c = bench.ClockSampler(0)
    c.proc = object()   # a sampler that ran; only its output file matters here
    c.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
    c.file.write("".join(lines))
    c.file.flush()
    c.t0, c.t1 = t0, t1
    return c


def line(ts, mhz, power, cap):
    stamp = ts.strftime("%Y/%m/%d %H:%M:%S.%f")[:-3] if isinstance(ts, datetime) else ts
    return (f"{stamp}, 0, {mhz}, 1965, {power}, 0x0, Not Active, Not Active, Not Active, "
            f"{'Active' if cap else 'Not Active'}\n")


def test_samples_outside_the_timed_region_are_dropped():
    t0 = datetime(2026, 1, 1, 12, 0, 0)
    t1 = t0 + timedelta(seconds=1)
    lines = [line(t0 - timedelta(seconds=5), 345, 120.0, False),    # idle, long before
             line(t0 - timedelta(seconds=0.1), 1965, 400.0, False),  # warm-up just before
             line(t0 + timedelta(seconds=0.5), 1700, 990.0, True),
             line(t0 + timedelta(seconds=0.9), 1690, 995.0, True),
             line(t1 + timedelta(seconds=3), 500, 150.0, False)]     # after
    s = sampler_with(lines, t0, t1).summary()
    assert s["samples"] == 3
    assert s["sm_mhz"] == 1700.0 and s["sm_max_mhz"] == 1965.0
    assert s["reasons"] == ["sw_power_cap"] and s["power_w_max"] == 995.0


def test_unreadable_timestamps_keep_every_sample():
    t0 = datetime(2026, 1, 1, 12, 0, 0)
    s = sampler_with([line("n/a", 1800, 500.0, False), line("n/a", 1900, 600.0, False)], t0,
                     t0 + timedelta(seconds=1)).summary()
    assert s["samples"] == 2 and s["sm_mhz"] == 1850.0 and s["window"] == "warm-up and timed region"


def test_no_samples_is_reported():
    t0 = datetime(2026, 1, 1, 12, 0, 0)
    s = sampler_with([], t0, t0).summary()
    assert s["sm_mhz"] is None and s["reasons"] == ["no samples"]


def test_cpu_sample_keeps_the_product():
    """The CPU baseline's leading-row sample relabels columns to the B rows it
    touches; its product equals those rows of A @ B."""
    import torch

    import oracle
    import workloads

    bench = load_bench()
    w = workloads.make(2, scale=0.004)
    smp = bench.cpu_sample(w, target_nnz=5000)
    R = smp["rows"]
    assert smp["nnz"] == int(w.rowptr[R]) and smp["distinct_cols"] == smp["B"].shape[0] <= smp["nnz"]
    got = oracle.cpu_reference(R, smp["B"].shape[0], smp["rowptr"], smp["col"], smp["val"], smp["B"])
    rp, c, v = workloads.row_slice(w, 0, R)
    want = torch.from_numpy(oracle.spmm_csr_f64(rp, c, v, w.B))
    assert torch.allclose(got.double(), want, atol=1e-4, rtol=1e-4)
    # the blocked form the bench times computes the same product
    chunks = bench.feature_chunks(smp["B"])
    assert sum(b.shape[1] for b in chunks) == w.N and all(b.is_contiguous() for b in chunks)
    blocked = torch.cat([oracle.cpu_reference(R, b.shape[0], smp["rowptr"], smp["col"], smp["val"], b)
                         for b in chunks], 1)
    assert torch.allclose(blocked.double(), want, atol=1e-4, rtol=1e-4)


def test_bench_defaults_are_the_headline():
    bench = load_bench()
    a = bench.parse_args([])
    assert (a.config, a.scaling, a.op, a.gpus) == (5, "strong", "csr", 1)
    assert a.warmup >= 3


def test_kernel_names_from_the_trace():
    bench = load_bench()
    assert bench.short_name("void spmmb::(anonymous namespace)::csr_ring_kernel<__half, int, 32, 4, 2, 2, true>"
                            "(spmmb::GatherArgs)") == "csr_ring_kernel<__half, int, 32, 4, 2, 2, true>"
    assert bench.short_name("void unnamed>::csr_fixup_kernel<__half, int>(GatherArgs)") == "csr_fixup_kernel<__half, int>"
