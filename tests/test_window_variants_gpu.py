"""The fp16 window kernel of window_warp.cu under every launch shape that
SPMM_B200_WW selects (read at every launch), against the float64 oracle.

Every warp gets several items (more items than warps in the grid), with
empty windows, windows of one block, windows whose stream is only CSR
entries and long windows side by side."""

import functools
import os

import numpy as np
import pytest
import torch

import oracle
from helpers import assert_close, rand_csr

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(bool(os.environ.get("SPMM_B200_WINDOW")), reason="another window kernel forced")]

DEV = "cuda"
VARIANTS = ["", "128s4w2", "128s5w2", "128s6w2", "128s5w1", "64s6w2", "64s5w4", "128s4w4", "64s3w4",
            "256s3w4", "256s3w2", "256s4w2", "128s3w4"]


@pytest.fixture(scope="module")
def npu():
    import build

    build.build()
    import spmm_npu

    assert torch.cuda.is_available()
    return spmm_npu


@functools.lru_cache(maxsize=4)
def _layout(nwin, K, seed, dtype):
    g = np.random.default_rng(seed)
    nb = g.integers(0, 70, nwin)
    nb[g.random(nwin) < 0.1] = 0          # empty block streams
    nb[g.random(nwin) < 0.1] = 1          # one block
    nb[::97] = 400                        # long windows (25 chunks)
    cptr = torch.from_numpy(np.concatenate([[0], np.cumsum(nb)])).to(torch.int32)
    ccol = torch.from_numpy(np.concatenate([np.sort(g.choice(K, int(n), replace=False)) for n in nb])).to(torch.int32)
    gen = torch.Generator().manual_seed(seed)
    cval = (torch.rand(16 * int(nb.sum()), generator=gen) * 2 - 1).to(dtype)
    cval[torch.rand(cval.numel(), generator=gen) < 0.5] = 0
    vrows = 16 * nwin + 123
    vcrow, vcol = rand_csr(vrows, K, 0.004, seed=seed, long_rows={5: 300, 16 * nwin + 7: 900}, empty_every=3)
    vval = (torch.rand(vcol.numel(), generator=gen) * 2 - 1).to(dtype)
    return cptr, ccol, cval, vcrow, vcol, vval


@pytest.mark.parametrize("variant", VARIANTS)
@pytest.mark.parametrize("N", [64, 128, 256])
def test_window_variants_match_oracle(npu, variant, N):
    dtype = torch.float16
    nwin, K = 3000, 4000
    cptr, ccol, cval, vcrow, vcol, vval = _layout(nwin, K, seed=N + 7, dtype=dtype)
    B = torch.randn(K, N, generator=torch.Generator().manual_seed(N)).to(dtype)
    ref = oracle.spmm_mixed_f64(cptr, ccol, cval, vcrow, vcol, vval, B)
    old = os.environ.get("SPMM_B200_WW")
    os.environ["SPMM_B200_WW"] = variant
    try:
        args = [x.to(DEV) for x in (cptr, ccol, cval, vcrow, vcol, vval)]
        z = torch.zeros(40, dtype=torch.int32, device=DEV)
        y = npu.spmm_ascend_cube(*args, B.to(DEV), z[:20], z)
        y2 = npu.spmm_ascend_cube(*args, B.to(DEV), z[:20], z)
        torch.cuda.synchronize()
    finally:
        if old is None:
            os.environ.pop("SPMM_B200_WW", None)
        else:
            os.environ["SPMM_B200_WW"] = old
    code, detail = npu.device_status(True)
    assert code == 0, f"device status {code} at {detail}"
    assert torch.equal(y, y2), "window kernel not repeatable"
    assert_close(y.cpu(), ref, dtype, f"window variant {variant or 'default'} N={N}")
