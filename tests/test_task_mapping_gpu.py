"""Table 6 correctness on the GPU: every task-mapping method's layout, run
through spmm_ascend_cube, matches spmm_csr on the same matrix within the
reference's tolerance (tests/task_mapping/correctness.py:34-64, 140-143,
175-200), and the float64 oracle."""

import pytest
import torch

import oracle
import workloads
from helpers import assert_close

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tm():
    import build

    build.build()
    import task_mapping

    assert torch.cuda.is_available()
    return task_mapping


def _matrices():
    w = workloads.make(2, scale=0.01)
    yield "powerlaw", w.M, w.K, w.rowptr, w.col
    w = workloads.make(3, scale=0.01)
    yield "fem", w.M, w.K, w.rowptr, w.col
    w = workloads.make(4, scale=0.004)
    yield "cluster", w.M, w.K, w.rowptr, w.col


@pytest.mark.parametrize("dtype,dim", [(torch.float16, 128), (torch.float32, 64)])
@pytest.mark.parametrize("method", ["ours", "naive", "neutronsparse", "block-split"])
def test_method_matches_csr(tm, method, dtype, dim):
    for name, rows, cols, crow, col in _matrices():
        seed = tm.stable_seed(2027, name)
        values = tm.make_values(col.numel(), dtype, seed)
        mapping, meta = tm.prepare_partition(method, rows, cols, crow, col, values)
        assert meta["aic_nnz"] + meta["aiv_nnz"] == col.numel()
        assert all(t.is_cuda for t in mapping.values() if torch.is_tensor(t))
        dense = tm.make_dense(cols, dim, dtype, seed + dim)
        ref = tm.build_reference_invoker(crow, col, values, dense)()[:rows]
        out = tm.build_mixed_invoker(mapping, dense)()
        torch.cuda.synchronize()
        if method == "ours":   # packed row order: restore original rows
            import spmm_npu

            out = spmm_npu.restore_node_tensor(out, mapping["inv_permutation"])
        out = out[:rows]
        assert torch.isfinite(out.float()).all()
        atol, rtol = (2e-2, 2e-2) if dtype == torch.float16 else (1e-4, 1e-4)
        assert torch.isclose(out.float().cpu(), ref.float().cpu(), atol=atol, rtol=rtol).all(), (method, name)
        assert_close(out, oracle.spmm_csr_f64(crow, col, values, dense), dtype, f"{method}/{name}")
