"""Persistent graph relabelling for GNN layer loops.

``preprocess(..., graph_layout=True)`` on a square graph returns, besides the
window/CSR mapping, the same mapping with its columns renumbered through the
row permutation P (``renumbered_unique_col_ids``, ``renumbered_vcol_indices``:
the layout of P A P^T) and a fixed-layout mapping of P A^T P^T
(``transpose_*``), both over the same packed row count
(extension/custom_op.cpp:1006-1035; packed_column_reindex.h).  The reference
documents the intended use (spmm_npu.py:1-5): pack node tensors once with P,
run every layer in packed ids, restore original ids only at the end.

``PackedGraph`` is that use, on this engine:

    g = PackedGraph(crow, col, values, n)     # one GPU preprocess
    h = g.pack(x)                             # P x, zero padding rows
    for layer in layers:
        h = act(g.spmm(h) @ w)                # P A P^T h, autograd-aware
    y = g.restore(h)                          # P^T h, original node order

``g.spmm`` is differentiable in its dense argument: the backward pass of
``Y = (P A P^T) H`` is ``dH = (P A^T P^T) dY``, one ``spmm_ascend_cube`` on
the transpose mapping, so forward and backward both stay in packed ids with
no per-layer permutation.
"""

from __future__ import annotations

import torch

import spmm_npu

_FWD_KEYS = ("crow_window_ptr", "renumbered_unique_col_ids", "value", "vrow_window_ptr",
             "renumbered_vcol_indices", "vvalue")
_BWD_KEYS = tuple("transpose_" + k for k in ("crow_window_ptr", "unique_col_ids", "value", "vrow_window_ptr",
                                             "vcol_indices", "vvalue"))


class PackedGraph:
    """A square sparse graph in the packed layout of ``preprocess``."""

    def __init__(self, crow, col, values, num_nodes: int, device=None):
        device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        m = spmm_npu.preprocess(crow.to(device), col.to(device), values.to(device), num_nodes, num_nodes, 16,
                                graph_layout=True)
        if not int(m["packed_layout_supported"].item()):
            raise ValueError("the packed graph layout needs a square matrix")
        self.num_nodes = num_nodes
        self.packed_rows = int(m["packed_rows"].item())
        self.inv_permutation = m["inv_permutation"]
        self.permutation = m["permutation"]
        self.forward_mapping = [m[k].contiguous() for k in _FWD_KEYS]
        self.transpose_mapping = [m[k].contiguous() for k in _BWD_KEYS]
        self.mapping = m
        z = lambda n: torch.zeros(n, dtype=torch.int32, device=device)  # noqa: E731
        self._starts = (z(20), z(40))

    def pack(self, x: torch.Tensor) -> torch.Tensor:
        """P x: rows in packed order, padding rows zero."""
        return spmm_npu.pack_node_tensor(x, self.inv_permutation, self.packed_rows)

    def restore(self, h: torch.Tensor) -> torch.Tensor:
        """P^T h: rows back in original node order."""
        return spmm_npu.restore_node_tensor(h, self.inv_permutation)

    def _run(self, mapping, h: torch.Tensor) -> torch.Tensor:
        y = spmm_npu.spmm_ascend_cube(*mapping, h.contiguous(), *self._starts)
        return y[: self.packed_rows]

    def spmm(self, h: torch.Tensor) -> torch.Tensor:
        """(P A P^T) h for a packed node tensor h, differentiable in h."""
        if h.size(0) != self.packed_rows:
            raise ValueError(f"expected a packed node tensor of {self.packed_rows} rows, got {h.size(0)}")
        return _PackedSpMM.apply(h, self)

    def spmm_transpose(self, h: torch.Tensor) -> torch.Tensor:
        """(P A^T P^T) h for a packed node tensor h."""
        if h.size(0) != self.packed_rows:
            raise ValueError(f"expected a packed node tensor of {self.packed_rows} rows, got {h.size(0)}")
        return self._run(self.transpose_mapping, h)


class _PackedSpMM(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, graph):
        ctx.graph = graph
        return graph._run(graph.forward_mapping, h)

    @staticmethod
    def backward(ctx, grad):
        return ctx.graph._run(ctx.graph.transpose_mapping, grad), None


__all__ = ["PackedGraph"]
