"""Table-6 task-mapping harness on the GPU.

The reference's paper compares four ways of dividing one CSR matrix between
its matrix engines (the 16-row window layout) and its vector engines (plain
CSR rows), all run through ``spmm_ascend_cube`` (reference harness:
tests/task_mapping/common.py, method list :19-28):

``ours``           the cost-model task mapping, ``preprocess``;
``block-split``    ``block_level_split`` at ratio (222/190) * 0.5;
``naive``          the first nnz/3 nonzeros (in CSR order) to the windows;
``neutronsparse``  entries of dense columns that sit in dense rows to the
                   windows, with NeutronSparseLite's degree threshold.

Design of this module (B200 side):

* ``load_payload`` decodes a ``.pt`` CSR structure file into a ``CsrPayload``
  and validates it against ``PAYLOAD_RULES``, a table of named predicates
  evaluated in order (the first failing one raises ``ValueError``).
  ``save_payload`` / ``convert_matrix`` write the same schema
  (``shape``, ``crow_indices``, ``col_indices``, optional ``name``/``nnz``;
  reference writer: tests/data/prepare_data.py:24-43).
* ``DatasetQuery`` holds the selection filters of a dataset sweep and
  applies them to the sorted ``*.pt`` files of a directory.
* Each method is a function in ``PARTITIONERS`` that turns device tensors
  into a ``Split``: the mapping consumed by ``spmm_ascend_cube`` plus the
  nonzero counts of each side.  The two extra partitioners are expressed
  with per-entry row ids and ``bincount`` reductions on the device; their
  window part becomes a window layout through this engine's GPU
  ``csr_to_bcsr``.
"""

from __future__ import annotations

import hashlib
import math
import struct
from dataclasses import dataclass, field
from pathlib import Path
from typing import Callable, Dict, NamedTuple, Optional, Tuple

import torch

import spmm_npu

AIC_CORES = 20
AIV_CORES = 40
WINDOW_SIZE = 16
METHODS = ("ours", "naive", "neutronsparse", "block-split")
METHOD_LABELS = {
    "ours": "Ascend-SpMM task mapping",
    "naive": "Naive load balancing",
    "neutronsparse": "NeutronSparse load balancing",
    "block-split": "Block-Level split",
}
DEFAULT_BLOCK_RATIO = (222.0 / 190.0) * 0.5
DEFAULT_NAIVE_FRACTION = 1.0 / 3.0
_INT32_MAX = 2**31 - 1
MAPPING_KEYS = ("crow_window_ptr", "unique_col_ids", "value", "vrow_window_ptr", "vcol_indices", "vvalue")


# --------------------------------------------------------------------------
# CSR structure files
# --------------------------------------------------------------------------

class CsrPayload(NamedTuple):
    """A decoded structure file; unpacks as (name, rows, cols, crow, col)."""
    name: str
    rows: int
    cols: int
    crow: torch.Tensor   # int64 [rows + 1]
    col: torch.Tensor    # int64 [nnz]


@dataclass
class _Decoded:
    rows: int
    cols: int
    crow: torch.Tensor
    col: torch.Tensor
    declared_nnz: Optional[int]


def _monotone(t: torch.Tensor) -> bool:
    return t.numel() < 2 or bool((t[1:] >= t[:-1]).all())


# (rule name, predicate that must hold, message when it does not).  Order
# matters: later predicates may assume the earlier ones.
PAYLOAD_RULES: Tuple[Tuple[str, Callable[[_Decoded], bool], Callable[[_Decoded], str]], ...] = (
    ("shape", lambda d: d.rows > 0 and d.cols > 0,
     lambda d: f"matrix shape must be positive, got {d.rows} x {d.cols}"),
    ("pointer length", lambda d: d.crow.dim() == 1 and d.crow.numel() == d.rows + 1,
     lambda d: f"crow_indices needs rows + 1 = {d.rows + 1} entries, got {tuple(d.crow.shape)}"),
    ("pointer span", lambda d: d.col.dim() == 1 and int(d.crow[0]) == 0 and int(d.crow[-1]) == d.col.numel(),
     lambda d: f"crow_indices must run from 0 to the {d.col.numel()} column entries, "
               f"got {int(d.crow[0])}..{int(d.crow[-1])}"),
    ("pointer order", lambda d: _monotone(d.crow),
     lambda d: "crow_indices decreases somewhere (row pointers must be nondecreasing)"),
    ("entries", lambda d: d.col.numel() > 0,
     lambda d: "the matrix has no stored entries"),
    ("column range", lambda d: 0 <= int(d.col.min()) and int(d.col.max()) < d.cols,
     lambda d: f"col_indices must lie in [0, {d.cols}), got {int(d.col.min())}..{int(d.col.max())}"),
    ("32-bit indices", lambda d: max(d.rows, d.cols, d.col.numel()) <= _INT32_MAX,
     lambda d: "the matrix does not fit 32-bit indices (rows, columns and nonzeros must stay below 2^31)"),
    ("declared nnz", lambda d: d.declared_nnz is None or d.declared_nnz == d.col.numel(),
     lambda d: f"the payload declares nnz = {d.declared_nnz} but holds {d.col.numel()} column entries"),
)


def load_payload(path) -> CsrPayload:
    """Read and validate a CSR structure file (the reference's reader:
    tests/task_mapping/common.py:33-63).  Index tensors come back as int64 on
    the CPU; the name defaults to the file stem without a ``_csr`` suffix."""
    path = Path(path)
    try:
        raw = torch.load(path, map_location="cpu", weights_only=True)
    except TypeError:   # torch builds without weights_only
        raw = torch.load(path, map_location="cpu")
    absent = [k for k in ("col_indices", "crow_indices", "shape") if k not in raw]
    if absent:
        raise ValueError(f"payload lacks field(s): {', '.join(absent)}")
    rows, cols = (int(x) for x in raw["shape"])
    d = _Decoded(rows, cols, torch.as_tensor(raw["crow_indices"]).to(torch.int64).contiguous(),
                 torch.as_tensor(raw["col_indices"]).to(torch.int64).contiguous(),
                 int(raw["nnz"]) if "nnz" in raw else None)
    for _name, holds, message in PAYLOAD_RULES:
        if not holds(d):
            raise ValueError(message(d))
    name = raw.get("name") or path.stem.removesuffix("_csr")
    return CsrPayload(str(name), rows, cols, d.crow, d.col)


def save_payload(destination, name: str, rows: int, cols: int, crow, col) -> None:
    """Write a CSR structure file (int64 indices on the CPU)."""
    destination = Path(destination)
    destination.parent.mkdir(parents=True, exist_ok=True)
    as_host = lambda t: t.detach().to("cpu", torch.int64).contiguous()  # noqa: E731
    torch.save({"name": name, "shape": (int(rows), int(cols)), "nnz": int(col.numel()),
                "crow_indices": as_host(crow), "col_indices": as_host(col)}, destination)


def convert_matrix(source, destination):
    """Matrix Market file -> structure file: duplicate entries summed,
    explicit zeros removed, columns sorted within rows.  Returns
    (rows, cols, nnz)."""
    import numpy as np
    from scipy import sparse
    from scipy.io import mmread

    m = mmread(str(source))
    m = sparse.csr_matrix(m if sparse.issparse(m) else np.asarray(m))
    m.sum_duplicates()          # also sorts the column indices
    m.eliminate_zeros()
    m.sort_indices()
    save_payload(destination, Path(source).stem, m.shape[0], m.shape[1],
                 torch.from_numpy(m.indptr.astype(np.int64)), torch.from_numpy(m.indices.astype(np.int64)))
    return m.shape[0], m.shape[1], int(m.nnz)


# --------------------------------------------------------------------------
# dataset selection
# --------------------------------------------------------------------------

@dataclass(frozen=True)
class DatasetQuery:
    """Filters of a dataset sweep, applied in this order to the ``*.pt``
    files under a directory sorted by relative path: ``name`` keeps files
    whose directory is called ``name`` or whose stem contains it; ``index``
    picks exactly one file; otherwise ``[start:stop]`` then the first
    ``limit``.  An empty selection is an error."""
    name: str = ""
    index: Optional[int] = None
    start: int = 0
    stop: Optional[int] = None
    limit: Optional[int] = None

    def check(self) -> None:
        if self.start < 0:
            raise ValueError(f"start must be >= 0, got {self.start}")
        if self.stop is not None and self.stop < self.start:
            raise ValueError(f"stop ({self.stop}) must not be below start ({self.start})")
        if self.limit is not None and self.limit <= 0:
            raise ValueError(f"limit must be positive, got {self.limit}")

    def select(self, root) -> list:
        root = Path(root)
        found = sorted(root.rglob("*.pt"), key=lambda p: p.relative_to(root).as_posix())
        if self.name:
            found = [p for p in found if p.parent.name == self.name or self.name in p.stem]
        if self.index is not None:
            if not 0 <= self.index < len(found):
                raise ValueError(f"index {self.index} is not among the {len(found)} datasets found")
            return [found[self.index]]
        self.check()
        chosen = found[self.start:self.stop][: self.limit]
        if not chosen:
            raise ValueError(f"no .pt datasets selected under {root}")
        return chosen


def discover_datasets(dataset_dir, name: str = "", index: Optional[int] = None, start: int = 0,
                      stop: Optional[int] = None, limit: Optional[int] = None) -> list:
    """``DatasetQuery(name, index, start, stop, limit).select(dataset_dir)``."""
    return DatasetQuery(name, index, start, stop, limit).select(dataset_dir)


# --------------------------------------------------------------------------
# seeded operands
# --------------------------------------------------------------------------

def stable_seed(base_seed: int, relative_path: str) -> int:
    """Seed of one dataset: base_seed plus the first 8 bytes (little endian)
    of the SHA-256 of its relative path, modulo 2^63 - 1."""
    (salt,) = struct.unpack_from("<Q", hashlib.sha256(relative_path.encode()).digest())
    return (base_seed + salt) % (2**63 - 1)


def _uniform_pm1(shape, dtype, seed) -> torch.Tensor:
    gen = torch.Generator().manual_seed(seed)
    return torch.rand(shape, generator=gen).mul_(2).sub_(1).to(dtype).contiguous()


def make_values(nnz: int, dtype: torch.dtype, seed: int) -> torch.Tensor:
    """Nonzero values, U[-1, 1], from a CPU generator seeded with ``seed``."""
    return _uniform_pm1((nnz,), dtype, seed)


def make_dense(cols: int, dim: int, dtype: torch.dtype, seed: int) -> torch.Tensor:
    """Dense operand [cols, dim], U[-1, 1], from a seeded CPU generator."""
    return _uniform_pm1((cols, dim), dtype, seed)


def make_start(pointer: torch.Tensor, cores: int) -> torch.Tensor:
    """First row of each of ``cores`` equal nonzero ranges (the per-core
    start array of the reference's operators).  The engine plans its own
    split and ignores these arrays; they exist for API compatibility."""
    ptr = pointer.to(torch.int64)
    total = int(ptr[-1]) if ptr.numel() else 0
    if total <= 0:
        return torch.zeros(cores, dtype=torch.int32, device=pointer.device)
    per_core = -(-total // cores)
    first_nnz = per_core * torch.arange(cores, dtype=torch.int64, device=ptr.device)
    row = torch.searchsorted(ptr, first_nnz, side="right") - 1
    return row.clamp_(min=0).to(torch.int32)


# --------------------------------------------------------------------------
# partitioners
# --------------------------------------------------------------------------

class Split(NamedTuple):
    """Result of a CSR-level partitioner: the window part and the CSR part as
    (row pointer, columns, values) over the original rows, plus counts."""
    window: Tuple[torch.Tensor, torch.Tensor, torch.Tensor]
    rows: Tuple[torch.Tensor, torch.Tensor, torch.Tensor]
    meta: dict


def compute_neutronsparse_threshold(rows: int, cols: int, nnz: int) -> int:
    """Degree threshold of NeutronSparseLite's SplitStrategy: the mean row
    degree scaled by a factor chosen from the matrix density (the constants
    are that published rule), never below 4; 32 for a matrix without rows."""
    if rows == 0:
        return 32
    density = nnz / (rows * cols) if rows * cols else 0.0
    if density < 0.0002:
        scale = 1.8 if rows > 1_000_000 else 1.0
    elif density > 0.01:
        scale = 0.25
    else:
        scale = 0.55
    return max(4, int((nnz / rows) * scale))


def _pointer(counts: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    return torch.cat([counts.new_zeros(1), counts.cumsum(0)]).to(dtype)


def neutronsparse_parts(crow, col, values, rows: int, cols: int, assume_symmetric: bool = False) -> Split:
    """NeutronSparse partition: a column is dense when its degree exceeds the
    threshold, a row is dense when more than threshold of its entries lie in
    dense columns, and exactly the dense-column entries of dense rows go to
    the window part (reference: tests/task_mapping/common.py:170-229).  With
    ``assume_symmetric`` on a square matrix the row degrees stand in for the
    column degrees.  Both parts keep every row and the CSR entry order."""
    nnz = col.numel()
    dev = col.device
    ptr = crow.to(torch.int64)
    degree = ptr[1:] - ptr[:-1]
    owner = torch.repeat_interleave(torch.arange(rows, device=dev), degree, output_size=nnz)  # row of each entry
    col64 = col.to(torch.int64)
    shortcut = bool(assume_symmetric and rows == cols)
    col_degree = degree if shortcut else torch.bincount(col64, minlength=cols)
    threshold = compute_neutronsparse_threshold(rows, cols, nnz)
    dense_col = col_degree > threshold
    in_dense_col = dense_col[col64]
    dense_hits = torch.bincount(owner[in_dense_col], minlength=rows)
    dense_row = dense_hits > threshold
    to_window = in_dense_col & dense_row[owner]
    win_counts = torch.bincount(owner[to_window], minlength=rows)
    keep = ~to_window
    meta = {"threshold": threshold, "assume_symmetric": bool(assume_symmetric),
            "symmetry_shortcut_used": shortcut, "dense_rows": int(dense_row.sum()),
            "dense_columns": int(dense_col.sum()), "aic_nnz": int(win_counts.sum()),
            "aiv_nnz": nnz - int(win_counts.sum())}
    return Split((_pointer(win_counts, crow.dtype), col[to_window], values[to_window]),
                 (_pointer(degree - win_counts, crow.dtype), col[keep], values[keep]), meta)


def naive_parts(crow, col, values, rows: int, fraction: float) -> Split:
    """Naive split at a nonzero pivot in CSR order: entries before it go to the
    window part.  The pivot is nnz // 3 for the default fraction 1/3 and
    int(nnz * fraction) otherwise (reference: common.py:264-283)."""
    nnz = col.numel()
    pivot = nnz // 3 if math.isclose(fraction, 1.0 / 3.0) else int(nnz * fraction)
    pivot = min(max(pivot, 0), nnz)
    head = torch.minimum(crow, crow.new_tensor(pivot))
    tail = torch.clamp(crow - pivot, min=0)
    meta = {"fraction": fraction, "pivot_nnz": pivot, "aic_nnz": pivot, "aiv_nnz": nnz - pivot}
    return Split((head, col[:pivot], values[:pivot]), (tail, col[pivot:], values[pivot:]), meta)


def _window_layout(part, cols: int) -> Dict[str, torch.Tensor]:
    """Window layout (``csr_to_bcsr``) of a window part.  Rows after its last
    nonempty row are dropped, so the layout covers only the windows in use."""
    ptr, idx, val = part
    nnz = idx.numel()
    if nnz and int(ptr[-1]) != nnz:
        raise ValueError(f"window part: row pointer ends at {int(ptr[-1])} but holds {nnz} entries")
    used = int(torch.searchsorted(ptr.to(torch.int64), ptr.new_tensor([nnz], dtype=torch.int64))[0]) if nnz else 0
    if used == 0:
        return {"crow_window_ptr": ptr.new_zeros(1), "unique_col_ids": idx.new_empty(0), "value": val.new_empty(0)}
    return spmm_npu.csr_to_bcsr(ptr[: used + 1].contiguous(), idx.contiguous(), val.contiguous(), used, cols,
                                WINDOW_SIZE)


def _from_split(split: Split, cols: int, device) -> Tuple[Dict[str, torch.Tensor], dict]:
    layout = _window_layout(split.window, cols)
    vptr, vcol, vval = split.rows
    parts = (layout["crow_window_ptr"], layout["unique_col_ids"], layout["value"], vptr, vcol, vval)
    return {k: t.to(device).contiguous() for k, t in zip(MAPPING_KEYS, parts)}, split.meta


def _layout_counts(mapping, nnz: int) -> dict:
    csr = int(mapping["vcol_indices"].numel())
    return {"aic_nnz": nnz - csr, "aiv_nnz": csr, "aic_blocks": int(mapping["unique_col_ids"].numel())}


def _ours(rows, cols, crow, col, values, opts, device):
    mapping = spmm_npu.preprocess(crow, col, values, rows, cols, WINDOW_SIZE)
    return mapping, _layout_counts(mapping, col.numel())


def _block_split(rows, cols, crow, col, values, opts, device):
    mapping = spmm_npu.block_level_split(crow, col, values, rows, cols, opts.block_ratio, WINDOW_SIZE)
    return mapping, {"ratio": opts.block_ratio, **_layout_counts(mapping, col.numel())}


def _naive(rows, cols, crow, col, values, opts, device):
    return _from_split(naive_parts(crow, col, values, rows, opts.naive_fraction), cols, device)


def _neutron(rows, cols, crow, col, values, opts, device):
    return _from_split(neutronsparse_parts(crow, col, values, rows, cols, opts.assume_symmetric), cols, device)


@dataclass(frozen=True)
class PartitionOptions:
    block_ratio: float = DEFAULT_BLOCK_RATIO
    naive_fraction: float = DEFAULT_NAIVE_FRACTION
    assume_symmetric: bool = False

    def check(self) -> None:
        if not self.block_ratio > 0:
            raise ValueError(f"block_ratio must be positive, got {self.block_ratio}")
        if not 0.0 <= self.naive_fraction <= 1.0:
            raise ValueError(f"naive_fraction must be in [0, 1], got {self.naive_fraction}")


PARTITIONERS = {"ours": _ours, "block-split": _block_split, "naive": _naive, "neutronsparse": _neutron}


def prepare_partition(method: str, rows: int, cols: int, crow: torch.Tensor, col: torch.Tensor,
                      values: torch.Tensor, block_ratio: float = DEFAULT_BLOCK_RATIO,
                      naive_fraction: float = DEFAULT_NAIVE_FRACTION, assume_symmetric: bool = False,
                      device=None) -> Tuple[Dict[str, torch.Tensor], dict]:
    """Run one Table-6 method: returns (mapping for ``spmm_ascend_cube``,
    metadata with the nonzero count of each side).  Inputs may be CPU or CUDA
    tensors; the mapping lives on ``device`` (default: the current CUDA
    device).  ``ours`` returns the full ``preprocess`` dict (packed row
    order; ``inv_permutation`` restores the original rows)."""
    build = PARTITIONERS.get(method)
    if build is None:
        raise ValueError(f"unknown partition method {method!r}; choose one of {', '.join(METHODS)}")
    opts = PartitionOptions(block_ratio, naive_fraction, assume_symmetric)
    opts.check()
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    crow, col, values = (t.to(device) for t in (crow, col, values))
    mapping, meta = build(rows, cols, crow, col, values, opts, device)
    absent = [k for k in MAPPING_KEYS if k not in mapping]
    if absent:
        raise ValueError(f"{method}: mapping lacks {', '.join(absent)}")
    if meta["aic_nnz"] + meta["aiv_nnz"] != col.numel():
        raise ValueError(f"{method}: window ({meta['aic_nnz']}) and CSR ({meta['aiv_nnz']}) nonzeros "
                         f"do not add up to {col.numel()}")
    return mapping, {"method": method, "label": METHOD_LABELS[method], **meta}


# --------------------------------------------------------------------------
# runners
# --------------------------------------------------------------------------

@dataclass
class _Runner:
    """A prepared operator call with every argument already on the device."""
    op: Callable
    args: tuple = field(default_factory=tuple)

    def __call__(self):
        return self.op(*self.args)


def _on(dev, t: torch.Tensor, dtype=None) -> torch.Tensor:
    return t.to(device=dev, dtype=dtype if dtype is not None else t.dtype).contiguous()


def _target(dense: torch.Tensor):
    return dense.device if dense.is_cuda else torch.device("cuda", torch.cuda.current_device())


def build_mixed_invoker(mapping: Dict[str, torch.Tensor], dense: torch.Tensor) -> _Runner:
    """Callable running ``spmm_ascend_cube`` on a mapping with int32 indices."""
    dev, i32 = _target(dense), torch.int32
    idx = [_on(dev, mapping[k], i32) for k in ("crow_window_ptr", "unique_col_ids")]
    vidx = [_on(dev, mapping[k], i32) for k in ("vrow_window_ptr", "vcol_indices")]
    return _Runner(spmm_npu.spmm_ascend_cube,
                   (*idx, _on(dev, mapping["value"]), *vidx, _on(dev, mapping["vvalue"]), _on(dev, dense),
                    make_start(idx[0], AIC_CORES), make_start(vidx[0], AIV_CORES)))


def build_reference_invoker(crow, col, values, dense) -> _Runner:
    """Callable running ``spmm_csr`` (the point every method is compared
    with) on the whole matrix."""
    dev = _target(dense)
    ptr = _on(dev, crow, torch.int32)
    return _Runner(spmm_npu.spmm_csr, (ptr, _on(dev, col, torch.int32), _on(dev, values), _on(dev, dense),
                                       make_start(ptr, AIV_CORES)))


__all__ = [
    "AIC_CORES", "AIV_CORES", "WINDOW_SIZE", "METHODS", "METHOD_LABELS", "DEFAULT_BLOCK_RATIO",
    "DEFAULT_NAIVE_FRACTION", "MAPPING_KEYS", "CsrPayload", "PAYLOAD_RULES", "load_payload", "save_payload",
    "convert_matrix", "DatasetQuery", "discover_datasets", "stable_seed", "make_values", "make_dense",
    "make_start", "Split", "compute_neutronsparse_threshold", "neutronsparse_parts", "naive_parts",
    "PartitionOptions", "PARTITIONERS", "prepare_partition", "build_mixed_invoker", "build_reference_invoker",
]
