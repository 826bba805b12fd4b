"""The tcgen05 window kernel (window_tc.cu: TMEM accumulators, fp16, 128-feature
slices) against the float64 oracle: every mixed-operator test module is rerun
in a child process with SPMM_B200_WINDOW=tc, so the
golden layouts of the reference, random windows, graph layouts, spmm_cube and
tile consumers, config-shaped matrices and B offsets beyond 2^32 elements all
go through it wherever the width is a multiple of 128 (other widths keep the
default kernel).  Also checks directly that the kernel ran, bit for bit
against itself across launches, and within tolerance of the default kernel."""

import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def _rerun(args, timeout=1200):
    env = dict(os.environ, SPMM_B200_WINDOW="tc")
    r = subprocess.run([sys.executable, "-m", "pytest", "-x", "-q", "-p", "no:cacheprovider", *args], env=env,
                       cwd=os.path.dirname(HERE), capture_output=True, text=True, timeout=timeout)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]


def test_mixed_operator_suites_on_the_tcgen05_kernel():
    if os.environ.get("SPMM_B200_WINDOW"):
        pytest.skip("already running with a forced window kernel")
    _rerun([os.path.join(HERE, "test_spmm_gpu.py"), "-k", "mixed or golden or cube or graph",
            os.path.join(HERE, "test_cube_gpu.py"), os.path.join(HERE, "test_graph_gpu.py")])


def test_full_size_mixed_cases_on_the_tcgen05_kernel():
    if os.environ.get("SPMM_B200_WINDOW"):
        pytest.skip("already running with a forced window kernel")
    _rerun([os.path.join(HERE, "test_full_size_gpu.py"), "-k", "b_offsets or config4",
            os.path.join(HERE, "test_task_mapping_gpu.py")])


def _child_product():
    """Mixed SpMM of config 3 at scale 0.1 in this process (the window kernel
    is whatever SPMM_B200_WINDOW selects)."""
    code = r'''
import sys, torch
sys.path[:0] = ["ascend-spmm_b200", "oracle", "tests", "."]
import workloads, spmm_npu
w = workloads.make(3, device="cuda", scale=0.1)
m = spmm_npu.preprocess(w.rowptr, w.col, w.val, w.M, w.K, 16, False)
z = torch.zeros(40, dtype=torch.int32, device="cuda")
args = [m[k] for k in ("crow_window_ptr", "unique_col_ids", "value", "vrow_window_ptr", "vcol_indices", "vvalue")]
y1 = spmm_npu.spmm_ascend_cube(*args, w.B, z[:20], z)
y2 = spmm_npu.spmm_ascend_cube(*args, w.B, z[:20], z)
torch.cuda.synchronize()
assert spmm_npu.device_status(True)[0] == 0
assert torch.equal(y1, y2)
torch.save(y1.cpu(), sys.argv[1])
'''
    return code


def test_tcgen05_kernel_repeatable_and_close_to_default(tmp_path):
    if os.environ.get("SPMM_B200_WINDOW"):
        pytest.skip("already running with a forced window kernel")
    outs = {}
    for kind in ("tc", "warp"):
        path = tmp_path / f"{kind}.pt"
        env = dict(os.environ, SPMM_B200_WINDOW=kind)
        r = subprocess.run([sys.executable, "-c", _child_product(), str(path)], env=env, cwd=os.path.dirname(HERE),
                           capture_output=True, text=True, timeout=600)
        assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
        outs[kind] = torch.load(path)
    a, b = outs["tc"].float(), outs["warp"].float()
    assert torch.isclose(a, b, atol=2e-2, rtol=2e-2).all()
