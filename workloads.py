"""Seeded synthetic inputs for the five BASELINE configurations.

The reference measured on SuiteSparse matrices (tests/data/prepare_data.py),
which are not available offline; these generators stand in with the shapes,
sizes and value distributions BASELINE.json names.  Every matrix is a
coalesced CSR with sorted, distinct columns per row; values are U[-1, 1] in
the config's dtype (tests/task_mapping/common.py:130-136) and the dense
operand B is N(0, 1).  ``scale`` shrinks the row/column count (and nothing
else) so the same generator yields oracle-sized parity cases.

All generators are pure torch and run on the device given, seeded from
``seed`` (default 2027, the reference's base seed,
tests/task_mapping/correctness.py:92).  The same seed on the same device type
gives the same matrix.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch

DEFAULT_SEED = 2027


@dataclass
class Workload:
    name: str
    M: int
    K: int
    N: int
    dtype: torch.dtype
    rowptr: torch.Tensor   # int32 [M + 1]
    col: torch.Tensor      # int32 [nnz]
    val: torch.Tensor      # dtype [nnz]
    B: torch.Tensor        # dtype [K, N]
    params: dict

    @property
    def nnz(self) -> int:
        return int(self.col.numel())

    def flops(self) -> int:
        return 2 * self.nnz * self.N

    def bytes_per_nnz_model(self) -> int:
        """Algorithmic bytes of one SpMM, the per-nnz gather model:
        4(M+1) + nnz(4 + s) + nnz*N*s + M*N*s."""
        s = torch.finfo(self.dtype).bits // 8
        return 4 * (self.M + 1) + self.nnz * (4 + s) + self.nnz * self.N * s + self.M * self.N * s


def _gen(device, seed):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def _csr_from_pairs(rows: torch.Tensor, cols: torch.Tensor, M: int, K: int):
    """Coalesce (row, col) pairs into a sorted, duplicate-free int32 CSR."""
    key = rows.to(torch.int64) * K + cols.to(torch.int64)
    key = torch.unique(key)  # sorted
    r = torch.div(key, K, rounding_mode="floor")
    c = key - r * K
    counts = torch.bincount(r, minlength=M)
    rowptr = torch.zeros(M + 1, dtype=torch.int64, device=key.device)
    rowptr[1:] = torch.cumsum(counts, 0)
    return rowptr.to(torch.int32), c.to(torch.int32)


def _values(nnz, dtype, device, seed):
    g = _gen(device, seed)
    return (torch.rand(nnz, generator=g, device=device) * 2 - 1).to(dtype)


def _dense(K, N, dtype, device, seed):
    g = _gen(device, seed)
    return torch.randn((K, N), generator=g, device=device, dtype=torch.float32).to(dtype)


# --------------------------------------------------------------------------
# degree and column distributions
# --------------------------------------------------------------------------

def _trunc_pareto_floor_mean(xmin: float, alpha: float, xmax: float) -> float:
    """E[floor(X)] for X ~ Pareto(alpha) truncated to [xmin, xmax)."""
    a1 = 1.0 - alpha
    norm = xmin ** a1 - xmax ** a1

    def cdf(x):
        x = np.clip(x, xmin, xmax)
        return (xmin ** a1 - x ** a1) / norm

    k = np.arange(math.floor(xmin), math.ceil(xmax) + 1, dtype=np.float64)
    p = cdf(k + 1) - cdf(k)
    return float((k * p).sum())


def powerlaw_xmin(alpha: float, dmax: int, mean: float) -> float:
    """Bisection for the lower cut-off so that E[floor(X)] == mean, where
    X ~ Pareto(alpha) on [xmin, dmax + 1).  Deterministic (pure arithmetic)."""
    lo, hi = 1.0, float(dmax)
    for _ in range(100):
        mid = 0.5 * (lo + hi)
        if _trunc_pareto_floor_mean(mid, alpha, dmax + 1.0) < mean:
            lo = mid
        else:
            hi = mid
    return 0.5 * (lo + hi)


def powerlaw_degrees(n, alpha, dmax, mean, device, seed):
    xmin = powerlaw_xmin(alpha, dmax, mean)
    u = torch.rand(n, generator=_gen(device, seed), device=device, dtype=torch.float64)
    a1 = 1.0 - alpha
    lo, hi = xmin ** a1, (dmax + 1.0) ** a1
    x = (lo - u * (lo - hi)) ** (1.0 / a1)
    return torch.clamp(torch.floor(x), 1, dmax).to(torch.int64), xmin


def zipf_columns(n, K, s, device, seed):
    """Column ids with P(c) ~ (c + 1)^-s on [0, K) (continuous inverse CDF,
    floored): preferential attachment with hub columns at low ids."""
    u = torch.rand(n, generator=_gen(device, seed), device=device, dtype=torch.float64)
    if abs(s - 1.0) < 1e-12:
        x = torch.exp(u * math.log(K + 1.0)) - 1.0
    else:
        a = 1.0 - s
        x = (1.0 + u * ((K + 1.0) ** a - 1.0)) ** (1.0 / a) - 1.0
    return torch.clamp(torch.floor(x), 0, K - 1).to(torch.int64)


# --------------------------------------------------------------------------
# the five configurations
# --------------------------------------------------------------------------

def config1_uniform(device="cpu", seed=DEFAULT_SEED, scale=1.0, N=128):
    """16384^2, exactly 10 distinct uniform columns per row, fp16, N=128."""
    M = K = max(16, int(16384 * scale))
    per_row = min(10, K)
    g = _gen(device, seed)
    cols = []
    chunk = max(1, (1 << 26) // K)
    for r0 in range(0, M, chunk):
        r1 = min(M, r0 + chunk)
        keys = torch.rand((r1 - r0, K), generator=g, device=device)
        cols.append(torch.topk(keys, per_row, dim=1).indices)
    c = torch.cat(cols).to(torch.int64)
    rows = torch.arange(M, device=device).repeat_interleave(per_row)
    rowptr, col = _csr_from_pairs(rows, c.reshape(-1), M, K)
    val = _values(col.numel(), torch.float16, device, seed + 1)
    B = _dense(K, N, torch.float16, device, seed + 2)
    return Workload("cfg1_uniform", M, K, N, torch.float16, rowptr, col, val, B,
                    {"per_row": per_row, "seed": seed, "scale": scale})


def _powerlaw(name, M, alpha, mean, dmax, N, device, seed, scale):
    deg, xmin = powerlaw_degrees(M, alpha, dmax, mean, device, seed)
    rows = torch.repeat_interleave(torch.arange(M, device=device), deg)
    cols = zipf_columns(rows.numel(), M, 1.0 / (alpha - 1.0), device, seed + 1)
    rowptr, col = _csr_from_pairs(rows, cols, M, M)
    del rows, cols
    val = _values(col.numel(), torch.float16, device, seed + 2)
    B = _dense(M, N, torch.float16, device, seed + 3)
    return Workload(name, M, M, N, torch.float16, rowptr, col, val, B,
                    {"alpha": alpha, "mean_target": mean, "dmax": dmax, "xmin": xmin,
                     "zipf_s": 1.0 / (alpha - 1.0), "nnz_drawn": int(deg.sum()), "seed": seed,
                     "scale": scale})


def config2_powerlaw(device="cpu", seed=DEFAULT_SEED, scale=1.0, N=256):
    """1M^2 power-law graph: degrees Zipf(2.1) on [xmin, 4096] with mean ~16,
    columns by preferential attachment; fp16, N=256."""
    M = max(64, int(1048576 * scale))
    return _powerlaw("cfg2_powerlaw", M, 2.1, 16.0, min(4096, M), N, device, seed, scale)


def config3_fem(device="cpu", seed=DEFAULT_SEED, scale=1.0, N=128):
    """524288^2 FEM-like: per 16-row block row 3-5 dense-ish 16x16 blocks within
    +-2048 columns of the diagonal at fill 0.8, plus 2 off-band nnz per row."""
    M = K = max(256, int(524288 * scale) // 16 * 16)
    nbr = M // 16
    band = min(128, nbr - 1)
    g = _gen(device, seed)
    nb = torch.randint(3, 6, (nbr,), generator=g, device=device)
    # distinct non-zero block offsets in [-band, band]
    keys = torch.rand((nbr, 2 * band), generator=g, device=device)
    idx = torch.topk(keys, 4, dim=1).indices
    off = idx - band
    off = torch.where(off >= 0, off + 1, off)
    bcol = torch.cat([torch.zeros((nbr, 1), dtype=off.dtype, device=device), off], 1)  # diagonal first
    bcol = bcol + torch.arange(nbr, device=device)[:, None]
    keep = (torch.arange(5, device=device)[None, :] < nb[:, None]) & (bcol >= 0) & (bcol < nbr)
    br, slot = torch.nonzero(keep, as_tuple=True)
    bc = bcol[br, slot]
    fill = torch.rand((br.numel(), 16, 16), generator=g, device=device) < 0.8
    b, r, c = torch.nonzero(fill, as_tuple=True)
    rows = br[b] * 16 + r
    cols = bc[b] * 16 + c
    # two uniform off-band entries per row: distance > 2048 (mod K)
    span = max(1, K - 2 * 2049 + 1)
    d = 2049 + torch.randint(0, span, (M, 2), generator=g, device=device)
    orow = torch.arange(M, device=device)[:, None].expand(M, 2)
    ocol = (orow + d) % K
    rowptr, col = _csr_from_pairs(torch.cat([rows, orow.reshape(-1)]), torch.cat([cols, ocol.reshape(-1)]), M, K)
    val = _values(col.numel(), torch.float16, device, seed + 1)
    B = _dense(K, N, torch.float16, device, seed + 2)
    return Workload("cfg3_fem", M, K, N, torch.float16, rowptr, col, val, B,
                    {"block_rows": nbr, "fill": 0.8, "band_blocks": band, "seed": seed, "scale": scale})


def config4_fp32_mixed(device="cpu", seed=DEFAULT_SEED, scale=1.0, N=512):
    """2M^2 fp32: 30% of 16-row windows hold a 64-column cluster at fill 0.6,
    the other rows have Poisson(8) uniform columns; N=512."""
    M = K = max(256, int(2097152 * scale) // 16 * 16)
    nwin = M // 16
    g = _gen(device, seed)
    clustered = torch.rand(nwin, generator=g, device=device) < 0.3
    c0 = torch.randint(0, K - 64, (nwin,), generator=g, device=device)
    cw = torch.nonzero(clustered, as_tuple=True)[0]
    fill = torch.rand((cw.numel(), 16, 64), generator=g, device=device) < 0.6
    w, r, c = torch.nonzero(fill, as_tuple=True)
    rows_c = cw[w] * 16 + r
    cols_c = c0[cw[w]] + c
    row_clustered = clustered.repeat_interleave(16)
    lam = torch.full((M,), 8.0, device=device)
    deg = torch.poisson(lam, generator=g).to(torch.int64)
    deg = torch.where(row_clustered, torch.zeros_like(deg), deg)
    rows_u = torch.repeat_interleave(torch.arange(M, device=device), deg)
    cols_u = torch.randint(0, K, (rows_u.numel(),), generator=g, device=device)
    rowptr, col = _csr_from_pairs(torch.cat([rows_c, rows_u]), torch.cat([cols_c, cols_u]), M, K)
    val = _values(col.numel(), torch.float32, device, seed + 1)
    B = _dense(K, N, torch.float32, device, seed + 2)
    return Workload("cfg4_fp32_mixed", M, K, N, torch.float32, rowptr, col, val, B,
                    {"cluster_fraction": 0.3, "fill": 0.6, "poisson": 8, "seed": seed, "scale": scale})


def config5_large(device="cpu", seed=DEFAULT_SEED, scale=1.0, N=1024):
    """16.7M^2 power law: degrees Zipf(2.0) on [xmin, 4096] with mean ~32;
    fp16, N=1024.  Generate on a GPU at full scale."""
    M = max(64, int(16777216 * scale))
    w = _powerlaw("cfg5_large", M, 2.0, 32.0, min(4096, M), N, device, seed, scale)
    assert w.M + w.nnz < 2 ** 31
    return w


CONFIGS = {
    1: config1_uniform,
    2: config2_powerlaw,
    3: config3_fem,
    4: config4_fp32_mixed,
    5: config5_large,
}


def make(cfg: int, device="cpu", seed=DEFAULT_SEED, scale=1.0, N=None) -> Workload:
    kw = {} if N is None else {"N": N}
    return CONFIGS[cfg](device=device, seed=seed, scale=scale, **kw)


def row_slice(w: Workload, r0: int, r1: int):
    """CSR of rows [r0, r1) (rebased row pointer) - for sampled CPU baselines
    and row-sharded multi-GPU runs."""
    p0, p1 = int(w.rowptr[r0]), int(w.rowptr[r1])
    rp = (w.rowptr[r0:r1 + 1].to(torch.int64) - p0).to(torch.int32)
    return rp, w.col[p0:p1], w.val[p0:p1]
