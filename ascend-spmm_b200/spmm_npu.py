"""Public Python API of the B200 SpMM engine (drop-in for the reference's
``spmm_npu`` module, IDMG-Lab/Ascend-SpMM spmm_npu.py:1-78).

Every operator and layout function runs as hand-written CUDA through
``custom_ops_lib`` (the torch-facing module over ``libspmm_b200.so``).  There
is no CPU fallback: importing this module fails if the extension is missing,
and the operators require CUDA tensors, as the reference requires NPU tensors.

For fixed square graphs, ``preprocess(..., graph_layout=True)`` returns
``P A P^T`` mappings; pack node tensors once with ``P`` and restore original
ids only when needed.
"""

import torch

from custom_ops_lib import (  # noqa: F401  (re-exported API)
    device_status,
    spmm_ascend_cube,
    spmm_ascend_cube_aic_without_pipeline,
    spmm_ascend_cube_aiv_mb,
    spmm_ascend_cube_tiles,
    spmm_csr,
    spmm_csr_aiv_mb_batch,
    spmm_cube,
)

from custom_ops_lib import (  # noqa: F401  (GPU layout builders)
    block_level_split,
    csr_to_ascend_cube,
    csr_to_bcsr,
    csr_to_spmm_cube,
    preprocess,
)
from custom_ops_lib import pack_rows as _pack_rows, restore_rows as _restore_rows


def _index(inv_permutation, device):
    return inv_permutation.to(device=device, dtype=torch.long).reshape(-1).contiguous()


# Row scatter / gather on the GPU, differentiable like the reference's
# index_copy_ / index_select (the gradient of one is the other).
class _PackRows(torch.autograd.Function):
    @staticmethod
    def forward(ctx, tensor, index, packed_rows):
        ctx.save_for_backward(index)
        return _pack_rows(tensor.contiguous(), index, packed_rows)

    @staticmethod
    def backward(ctx, grad):
        (index,) = ctx.saved_tensors
        return _restore_rows(grad.contiguous(), index), None, None


class _RestoreRows(torch.autograd.Function):
    @staticmethod
    def forward(ctx, packed, index):
        ctx.save_for_backward(index)
        ctx.rows = packed.size(0)
        return _restore_rows(packed.contiguous(), index)

    @staticmethod
    def backward(ctx, grad):
        (index,) = ctx.saved_tensors
        return _pack_rows(grad.contiguous(), index, ctx.rows), None


def pack_node_tensor(tensor, inv_permutation, packed_rows=None):
    """Apply ``P`` once to a tensor whose leading dimension is original node id.

    Same contract as the reference (spmm_npu.py:22-47): padding rows are
    zero, and errors are raised as ValueError with the reference's messages.
    This helper belongs in graph preprocessing, not in the per-layer loop.
    """
    if tensor.ndim < 1:
        raise ValueError("a node tensor must have at least one dimension")
    index = _index(inv_permutation, tensor.device)
    if tensor.size(0) != index.numel():
        raise ValueError("inv_permutation must contain one entry per original node")
    if index.numel() and bool((index < 0).any().item()):
        raise ValueError("inv_permutation does not map every original node")
    minimum_rows = int(index.max().item()) + 1 if index.numel() else 0
    if packed_rows is None:
        packed_rows = minimum_rows
    elif torch.is_tensor(packed_rows):
        packed_rows = int(packed_rows.item())
    else:
        packed_rows = int(packed_rows)
    if packed_rows < minimum_rows:
        raise ValueError("packed_rows is smaller than the permutation extent")
    return _PackRows.apply(tensor, index, packed_rows)


def restore_node_tensor(packed_tensor, inv_permutation):
    """Apply ``P^T`` once and return rows in original node-id order
    (reference spmm_npu.py:50-61)."""
    if packed_tensor.ndim < 1:
        raise ValueError("a packed node tensor must have at least one dimension")
    index = _index(inv_permutation, packed_tensor.device)
    if index.numel() and (
        bool((index < 0).any().item())
        or int(index.max().item()) >= packed_tensor.size(0)
    ):
        raise ValueError("inv_permutation contains an invalid packed node id")
    return _RestoreRows.apply(packed_tensor, index)


__all__ = [
    "block_level_split",
    "csr_to_ascend_cube",
    "csr_to_bcsr",
    "csr_to_spmm_cube",
    "pack_node_tensor",
    "preprocess",
    "restore_node_tensor",
    "spmm_ascend_cube",
    "spmm_ascend_cube_aic_without_pipeline",
    "spmm_ascend_cube_aiv_mb",
    "spmm_ascend_cube_tiles",
    "spmm_csr",
    "spmm_csr_aiv_mb_batch",
    "spmm_cube",
]
