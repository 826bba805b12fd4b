"""Shared test helpers: golden-fixture loading and the reference's
tolerance comparison (tests/task_mapping/correctness.py:34-64)."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"


def load_golden(name):
    z = np.load(GOLDEN / f"{name}.npz")
    idt = torch.int32 if z["crow"].dtype == np.int32 else torch.int64
    case = {
        "z": z,
        "nrows": int(z["nrows"]),
        "ncols": int(z["ncols"]),
        "crow": torch.from_numpy(z["crow"]).to(idt),
        "col": torch.from_numpy(z["col"]).to(idt),
        "values": torch.from_numpy(z["values"]),
        "dense": torch.from_numpy(z["dense"]),
    }
    return case


def golden_layout(case, fn):
    z = case["z"]
    return {k.split("/", 1)[1]: torch.from_numpy(np.ascontiguousarray(z[k]))
            for k in z.files if k.startswith(fn + "/")}


def tol(dtype):
    """atol = rtol = 2e-2 for fp16, 1e-4 for fp32 (correctness.py:140-143)."""
    return (2e-2, 2e-2) if dtype == torch.float16 else (1e-4, 1e-4)


def assert_close(actual: torch.Tensor, expected, dtype, what=""):
    """torch.isclose with the reference's tolerances; expected is float64."""
    a = actual.detach().double().cpu()
    e = torch.as_tensor(expected, dtype=torch.float64)
    assert a.shape == e.shape, (what, tuple(a.shape), tuple(e.shape))
    assert bool(torch.isfinite(a).all()), f"{what}: non-finite output"
    atol, rtol = tol(dtype)
    close = torch.isclose(a, e, atol=atol, rtol=rtol)
    bad = int((~close).sum())
    if bad:
        i = torch.nonzero(~close)[0].tolist()
        raise AssertionError(f"{what}: {bad} mismatches, first at {i}: {a[tuple(i)].item()} vs {e[tuple(i)].item()}")


def rand_csr(M, K, density, seed, long_rows=(), empty_every=0, device="cpu", idt=torch.int32):
    """Random sorted, duplicate-free CSR with optional long rows and empty rows."""
    g = np.random.default_rng(seed)
    rows = []
    for r in range(M):
        k = int(g.binomial(K, density))
        if r in long_rows:
            k = min(K, long_rows[r] if isinstance(long_rows, dict) else K // 2)
        if empty_every and r % empty_every == 0:
            k = 0
        rows.append(np.sort(g.choice(K, size=k, replace=False)))
    crow = np.zeros(M + 1, np.int64)
    crow[1:] = np.cumsum([len(c) for c in rows])
    col = np.concatenate(rows) if rows else np.zeros(0, np.int64)
    return torch.from_numpy(crow).to(idt).to(device), torch.from_numpy(col).to(idt).to(device)


def sample_oracle(rowptr, col, val, B, rows) -> np.ndarray:
    """float64 oracle rows ``rows`` of A @ B, gathering only the B rows those
    rows touch (B may be a large device tensor)."""
    import oracle

    rp = rowptr.to(torch.int64)
    starts, ends = rp[rows].cpu(), rp[rows + 1].cpu()
    pos = torch.cat([torch.arange(int(a), int(b)) for a, b in zip(starts, ends)]) if len(rows) else \
        torch.zeros(0, dtype=torch.int64)
    cols = col[pos.to(col.device)].to(torch.int64)
    uniq, inv = torch.unique(cols, return_inverse=True)
    sub_ptr = torch.zeros(len(rows) + 1, dtype=torch.int64)
    sub_ptr[1:] = torch.cumsum(ends - starts, 0)
    Bsub = B.index_select(0, uniq.to(B.device)).cpu()
    return oracle.spmm_csr_f64(sub_ptr, inv.cpu(), val[pos.to(val.device)].cpu(), Bsub)


def assert_linear(y, rowptr, col, val, B, what="", seed=0, sigmas=8.0):
    """Whole-matrix probe, size-independent: with a random sign vector x,
    (C x)_i must equal (A (B x))_i (float64, on the device) up to the
    rounding of C's elements to its dtype.  Each element of C carries at
    most half an ulp of rounding error, independent across features, so the
    residual of row i has standard deviation <= ulp/2 * ||C_i|| / sqrt(3);
    the check allows ``sigmas`` of it (plus 1e-6).  A dropped, duplicated or
    misplaced nonzero moves a row by |a| * |B_c . x| ~ |a| sqrt(N), far
    beyond the bound.  For fp16 outputs only: there the final rounding
    (2^-11 relative) dominates the fp32 accumulation error (sqrt(nnz) *
    2^-24 relative), which the bound covers with a factor of two."""
    assert y.dtype == torch.float16, "the probe models fp16 output rounding"
    dev = B.device
    M, N = y.shape
    g = torch.Generator(device=dev).manual_seed(seed)
    x = (torch.randint(0, 2, (N,), generator=g, device=dev, dtype=torch.int64) * 2 - 1).double()
    slab = max(1, (1 << 28) // max(1, N))
    bx = torch.empty(B.shape[0], dtype=torch.float64, device=dev)
    for r in range(0, B.shape[0], slab):
        bx[r:r + slab] = B[r:r + slab].double() @ x
    rp = rowptr.to(torch.int64)
    owner = torch.repeat_interleave(torch.arange(M, device=dev), rp[1:] - rp[:-1], output_size=int(col.numel()))
    axb = torch.zeros(M, dtype=torch.float64, device=dev)
    axb.index_add_(0, owner, val.double() * bx[col.to(torch.int64)])
    del owner
    cx = torch.empty(M, dtype=torch.float64, device=dev)
    c2 = torch.empty(M, dtype=torch.float64, device=dev)
    for r in range(0, M, slab):
        yy = y[r:r + slab].double()
        cx[r:r + slab] = yy @ x
        c2[r:r + slab] = (yy * yy).sum(1)
    bound = sigmas * 2.0 * 2.0 ** -11 * torch.sqrt(c2 / 3) + 1e-6
    bad = (cx - axb).abs() > bound
    assert bool(torch.isfinite(cx).all()), f"{what}: non-finite output"
    nbad = int(bad.sum())
    if nbad:
        i = int(torch.nonzero(bad)[0])
        raise AssertionError(f"{what}: {nbad} rows fail the linearity probe, first row {i}: "
                             f"{float(cx[i])} vs {float(axb[i])} (bound {float(bound[i])})")
