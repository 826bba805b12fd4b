"""Graph-layout layer loop (ascend-spmm_b200/graph.py): packed forward
P A P^T, autograd backward through the fixed-layout transpose P A^T P^T
(extension/custom_op.cpp:1006-1035), against float64 / dense torch
references."""

import numpy as np
import pytest
import torch

import oracle
from helpers import assert_close, rand_csr

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def graph_mod():
    import build

    build.build()
    import graph

    return graph


def dense_of(crow, col, val, n):
    a = torch.zeros(n, n, dtype=torch.float64)
    rows = torch.repeat_interleave(torch.arange(n), (crow[1:] - crow[:-1]).long())
    a[rows, col.long()] = val.double()
    return a


@pytest.mark.parametrize("dtype,N", [(torch.float16, 128), (torch.float32, 64)])
@pytest.mark.parametrize("idt", [torch.int32, torch.int64])
def test_packed_forward_and_backward(graph_mod, dtype, N, idt):
    n = 700
    crow, col = rand_csr(n, n, 0.02, seed=N, long_rows={5: 300}, empty_every=23, idt=idt)
    g = torch.Generator().manual_seed(3)
    val = (torch.rand(col.numel(), generator=g) * 2 - 1).to(dtype)
    x = torch.randn(n, N, generator=g).to(dtype)
    gy = torch.randn(n, N, generator=g).to(dtype)
    pg = graph_mod.PackedGraph(crow, col, val, n)
    assert pg.packed_rows % 16 == 0 and pg.packed_rows >= n

    xp = pg.pack(x.cuda()).requires_grad_(True)
    yp = pg.spmm(xp)
    assert yp.shape == (pg.packed_rows, N)
    y = pg.restore(yp)
    assert_close(y, oracle.spmm_csr_f64(crow, col, val, x), dtype, "forward")
    # backward: d/dX sum(Y * G) = A^T G, computed in packed ids
    (yp * pg.pack(gy.cuda())).sum().backward()
    gx = pg.restore(xp.grad)
    ref = dense_of(crow, col, val, n).T @ gy.double()
    assert_close(gx, ref.numpy(), dtype, "backward")
    # padding rows stay zero in both directions
    pad = torch.ones(pg.packed_rows, dtype=torch.bool)
    pad[pg.inv_permutation.cpu()] = False
    assert not bool(yp.detach().cpu()[pad].any()) and not bool(xp.grad.cpu()[pad].any())


def test_two_layer_loop_matches_dense(graph_mod):
    """A two-layer GCN-style loop kept in packed ids end to end."""
    n, f, h = 500, 64, 32
    crow, col = rand_csr(n, n, 0.03, seed=8)
    g = torch.Generator().manual_seed(8)
    val = torch.rand(col.numel(), generator=g)
    x = torch.randn(n, f, generator=g)
    w1 = (torch.randn(f, 64, generator=g) * 0.2).cuda().requires_grad_(True)
    w2 = (torch.randn(64, h, generator=g) * 0.2).cuda().requires_grad_(True)
    pg = graph_mod.PackedGraph(crow, col, val, n)
    hp = pg.pack(x.cuda())
    hp = torch.relu(pg.spmm(hp) @ w1)
    hp = pg.spmm(hp) @ w2
    loss = pg.restore(hp).square().sum()
    loss.backward()

    A = dense_of(crow, col, val, n).float().cuda()
    v1 = w1.detach().clone().requires_grad_(True)
    v2 = w2.detach().clone().requires_grad_(True)
    ref = (A @ torch.relu((A @ x.cuda()) @ v1)) @ v2
    ref_loss = ref.square().sum()
    ref_loss.backward()
    assert torch.allclose(loss, ref_loss, rtol=1e-4)
    assert torch.allclose(w1.grad, v1.grad, rtol=1e-3, atol=1e-3)
    assert torch.allclose(w2.grad, v2.grad, rtol=1e-3, atol=1e-3)


def test_unpacked_tensor_rejected(graph_mod):
    n = 40
    crow, col = rand_csr(n, n, 0.1, seed=1)
    pg = graph_mod.PackedGraph(crow, col, torch.ones(col.numel()), n)
    with pytest.raises(ValueError, match="packed node tensor"):
        pg.spmm(torch.ones(n + 1, 16, device="cuda"))


def test_pack_restore_are_differentiable(graph_mod):
    import spmm_npu

    n = 50
    crow, col = rand_csr(n, n, 0.1, seed=2)
    pg = graph_mod.PackedGraph(crow, col, torch.ones(col.numel()), n)
    x = torch.randn(n, 16, device="cuda", requires_grad=True)
    w = torch.randn(pg.packed_rows, 16, device="cuda")
    (spmm_npu.pack_node_tensor(x, pg.inv_permutation, pg.packed_rows) * w).sum().backward()
    assert torch.equal(x.grad, w[pg.inv_permutation.long()])
    p = torch.randn(pg.packed_rows, 16, device="cuda", requires_grad=True)
    v = torch.randn(n, 16, device="cuda")
    (spmm_npu.restore_node_tensor(p, pg.inv_permutation) * v).sum().backward()
    want = torch.zeros_like(p)
    want[pg.inv_permutation.long()] = v
    assert torch.equal(p.grad, want)
