"""Generate the golden fixtures in this directory from the reference itself.

Each ``<case>.npz`` holds one seeded CSR matrix (int32 or int64 indices,
fp16 or fp32 values), a dense operand, and the outputs of the reference's own
compiled preprocessing (``oracle/_ref``, built from the reference sources by
``oracle/build_ref.py``): ``csr_to_bcsr``, ``csr_to_ascend_cube``,
``block_level_split`` (a = 222/190 * 0.5, tests/task_mapping/common.py:28),
``preprocess`` and ``preprocess(graph_layout=True)``.  The dense product
``A @ B`` in float64 is computed with SciPy (independent of the C oracle).

The fixtures pin the CPU oracle (tests/test_oracle_golden.py) and the GPU
preprocessing (tests/test_preprocess_gpu.py) on machines where the reference
tree is absent.  Regenerate with ``python tests/golden/make_golden.py`` in an
environment that has the reference tree.
"""

from __future__ import annotations

import contextlib
import io
import os
import sys
from pathlib import Path

import numpy as np
import scipy.sparse as sp
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT / "oracle"))

BLOCK_RATIO = (222.0 / 190.0) * 0.5


def _rows_to_csr(rows):
    crow = np.zeros(len(rows) + 1, np.int64)
    crow[1:] = np.cumsum([len(r) for r in rows])
    col = np.concatenate(rows).astype(np.int64) if rows else np.zeros(0, np.int64)
    return crow, col


def make_case(kind: str, seed: int):
    g = np.random.default_rng(seed)
    if kind == "uniform":
        nrows, ncols = 200, 200
        rows = [np.sort(g.choice(ncols, size=g.binomial(ncols, 0.04), replace=False)) for _ in range(nrows)]
    elif kind == "cluster":
        nrows, ncols = 300, 260
        rows = []
        for r in range(nrows):
            base = set(g.choice(ncols, size=g.integers(0, 6), replace=False).tolist())
            if (r // 16) % 3 == 0:
                c0 = (r // 16) * 7 % (ncols - 24)
                base |= {c for c in range(c0, c0 + 24) if g.random() < 0.7}
            rows.append(np.array(sorted(base), np.int64))
    elif kind == "graph":
        nrows = ncols = 250
        rows = []
        for r in range(nrows):
            s = set(g.choice(ncols, size=g.integers(0, 5), replace=False).tolist())
            if (r // 16) % 2 == 1:
                c0 = (r // 16) * 11 % (ncols - 32)
                s |= {c for c in range(c0, c0 + 32) if g.random() < 0.5}
            rows.append(np.array(sorted(s), np.int64))
    elif kind == "ragged":
        nrows, ncols = 37, 50
        rows = [np.sort(g.choice(ncols, size=int(g.integers(0, 9)), replace=False)) if r % 5 else
                np.zeros(0, np.int64) for r in range(nrows)]
    elif kind == "powerlaw":
        nrows = ncols = 1000
        deg = np.minimum((g.pareto(1.1, nrows) + 1).astype(np.int64), 400)
        w = 1.0 / np.arange(1, ncols + 1) ** 0.9
        w /= w.sum()
        rows = [np.unique(g.choice(ncols, size=int(d), p=w)) for d in deg]
    elif kind == "dense":
        nrows, ncols = 64, 64
        rows = [np.arange(ncols, dtype=np.int64) if (r // 16) % 2 == 0 else
                np.sort(g.choice(ncols, size=3, replace=False)) for r in range(nrows)]
    else:
        raise ValueError(kind)
    crow, col = _rows_to_csr(rows)
    return nrows, ncols, crow, col


CASES = [
    ("uniform_i32_f16", "uniform", 1, torch.int32, torch.float16),
    ("cluster_i64_f32", "cluster", 2, torch.int64, torch.float32),
    ("graph_i32_f16", "graph", 3, torch.int32, torch.float16),
    ("ragged_i32_f32", "ragged", 4, torch.int32, torch.float32),
    ("powerlaw_i64_f16", "powerlaw", 5, torch.int64, torch.float16),
    ("dense_i32_f16", "dense", 6, torch.int32, torch.float16),
]

FUNCS = ("csr_to_bcsr", "csr_to_ascend_cube", "block_level_split", "preprocess", "preprocess_graph")


def case_inputs(kind, seed, idt, vdt):
    nrows, ncols, crow, col = make_case(kind, seed)
    gen = torch.Generator().manual_seed(1000 + seed)
    values = (torch.rand(col.size, generator=gen) * 2 - 1).to(vdt)
    dense = (torch.rand((ncols, 16), generator=gen) * 2 - 1).to(vdt)
    return nrows, ncols, torch.from_numpy(crow).to(idt), torch.from_numpy(col).to(idt), values, dense


def run_funcs(mod, nrows, ncols, crow, col, values) -> dict:
    """Call the five layout functions of ``mod`` (reference or oracle)."""
    out = {}
    with contextlib.redirect_stdout(io.StringIO()):
        out["csr_to_bcsr"] = mod.csr_to_bcsr(crow, col, values, nrows, ncols, 16)
        out["csr_to_ascend_cube"] = mod.csr_to_ascend_cube(crow, col, values, nrows, ncols, 16)
        out["block_level_split"] = mod.block_level_split(crow, col, values, nrows, ncols, BLOCK_RATIO, 16)
        out["preprocess"] = mod.preprocess(crow, col, values, nrows, ncols, 16, False)
        out["preprocess_graph"] = mod.preprocess(crow, col, values, nrows, ncols, 16, True)
    return out


def to_np(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.float16:
        return t.numpy().view(np.float16)
    return t.numpy()


def main():
    import build_ref

    ref = build_ref.load()
    if ref is None:
        raise SystemExit("reference tree not available; cannot regenerate fixtures")
    for name, kind, seed, idt, vdt in CASES:
        nrows, ncols, crow, col, values, dense = case_inputs(kind, seed, idt, vdt)
        arrays = {
            "nrows": np.int64(nrows), "ncols": np.int64(ncols),
            "crow": to_np(crow), "col": to_np(col), "values": to_np(values), "dense": to_np(dense),
        }
        outs = run_funcs(ref, nrows, ncols, crow, col, values)
        for fn, d in outs.items():
            for k, v in d.items():
                arrays[f"{fn}/{k}"] = to_np(v)
        A = sp.csr_matrix((values.double().numpy(), col.numpy(), crow.numpy()), shape=(nrows, ncols))
        arrays["spmm_f64"] = A @ dense.double().numpy()
        np.savez_compressed(HERE / f"{name}.npz", **arrays)
        print(name, nrows, ncols, int(col.numel()), os.path.getsize(HERE / f"{name}.npz"))


if __name__ == "__main__":
    main()
