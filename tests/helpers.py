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
