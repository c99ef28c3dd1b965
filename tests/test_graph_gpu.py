"""Message-passing plumbing (ictc_o2_gather_rows, ictc_o2_segment_sum through
ictc_o2_hp_b200.graph) against float64 PyTorch index_select / index_add: values,
gradients, determinism, empty graphs, out-of-range indices, and a full layer
(gather -> RadialUvuTensorProduct -> scatter) against the float64 composition."""

from __future__ import annotations

import pytest
import torch

from oracle import o2_oracle as O

pytestmark = pytest.mark.gpu
TOL = 1e-5


def _graph(nodes, edges, seed, device):
    gen = torch.Generator().manual_seed(seed)
    src = torch.randint(0, nodes, (edges,), generator=gen)
    dst = torch.randint(0, max(nodes // 2, 1), (edges,), generator=gen)  # half the nodes isolated
    if edges > 4:
        src[:3] = dst[:3]        # self loops
        src[3], dst[3] = src[4], dst[4]  # a repeated edge
    return src.to(device), dst.to(device)


def _err(a, b):
    return O.max_error(a.detach().cpu().double().numpy(), b.detach().cpu().double().numpy())


@pytest.mark.parametrize("nodes,edges,width", [(50, 400, 12), (7, 3, 5), (300, 2000, 64)])
def test_gather_scatter_and_gradients(nodes, edges, width, cuda_device):
    from ictc_o2_hp_b200.graph import EdgeIndex, gather, scatter_sum
    src, dst = _graph(nodes, edges, nodes + edges, cuda_device)
    ei = EdgeIndex(src, dst, nodes)
    feats = torch.randn(nodes, width, device=cuda_device, requires_grad=True)
    x = gather(feats, ei)
    out = scatter_sum(x * 2.0, ei)
    g = torch.randn(nodes, width, device=cuda_device)
    (gf,) = torch.autograd.grad(out, (feats,), g)
    fd = feats.detach().cpu().double().requires_grad_(True)
    xd = fd.index_select(0, src.cpu())
    od = torch.zeros(nodes, width, dtype=torch.float64).index_add(0, dst.cpu(), xd * 2.0)
    (gfd,) = torch.autograd.grad(od, (fd,), g.cpu().double())
    assert torch.equal(x.cpu(), feats.detach().cpu().index_select(0, src.cpu()))
    assert _err(out, od) <= TOL and _err(gf, gfd) <= TOL
    # fixed summation order: bit-identical reruns
    again = scatter_sum(gather(feats.detach(), ei) * 2.0, ei)
    assert torch.equal(again, out.detach())


def test_second_derivative_through_the_pair(cuda_device):
    from ictc_o2_hp_b200.graph import EdgeIndex, gather, scatter_sum
    src, dst = _graph(20, 90, 3, cuda_device)
    ei = EdgeIndex(src, dst, 20)
    feats = torch.randn(20, 6, device=cuda_device, requires_grad=True)
    out = scatter_sum(gather(feats, ei) ** 2, ei)
    (gf,) = torch.autograd.grad(out.sum(), (feats,), create_graph=True)
    (gg,) = torch.autograd.grad((gf ** 2).sum(), (feats,))
    fd = feats.detach().cpu().double().requires_grad_(True)
    od = torch.zeros(20, 6, dtype=torch.float64).index_add(0, dst.cpu(),
                                                            fd.index_select(0, src.cpu()) ** 2)
    (gfd,) = torch.autograd.grad(od.sum(), (fd,), create_graph=True)
    (ggd,) = torch.autograd.grad((gfd ** 2).sum(), (fd,))
    assert _err(gf, gfd) <= TOL and _err(gg, ggd) <= TOL


def test_empty_graph_and_bad_index(cuda_device):
    from ictc_o2_hp_b200 import _lib
    from ictc_o2_hp_b200.graph import EdgeIndex, gather, gather_rows, scatter_sum
    none = torch.zeros(0, dtype=torch.int64, device=cuda_device)
    ei = EdgeIndex(none, none, 5)
    feats = torch.randn(5, 3, device=cuda_device)
    assert gather(feats, ei).shape == (0, 3)
    assert torch.count_nonzero(scatter_sum(torch.zeros(0, 3, device=cuda_device), ei)) == 0
    assert _lib.graph_bad_index() == 0
    index = torch.tensor([0, 7, 2], device=cuda_device)  # 7 is out of range for 5 rows
    out = gather_rows(feats, index, index, torch.zeros(6, dtype=torch.int64, device=cuda_device))
    torch.cuda.synchronize()
    assert _lib.graph_bad_index() == 1
    assert torch.count_nonzero(out[1]) == 0 and torch.equal(out[2], feats[2])


def test_message_passing_layer(cuda_device):
    """nodes -> gather by src -> RadialUvuTensorProduct -> scatter to dst, with the
    node-feature, angular, hidden and alpha gradients, against float64 PyTorch."""
    from ictc_o2_hp_b200 import RadialUvuTensorProduct, UvuTensorProduct
    from ictc_o2_hp_b200.graph import EdgeIndex, gather, scatter_sum
    from ictc_o2_hp_b200.ops import torch_uvu_flat
    torch.manual_seed(5)
    n, e, U, H = 40, 300, 16, 12
    tp = UvuTensorProduct(U, 1, 2, parity="full", parity_in2="canonical", shared_weights=False)
    model = RadialUvuTensorProduct(tp, torch.nn.Linear(H, tp.weight_numel, bias=False))
    model = model.to(cuda_device)
    src, dst = _graph(n, e, 11, cuda_device)
    ei = EdgeIndex(src, dst, n)
    base = [torch.randn(n, tp.input1_dimension), torch.randn(e, tp.input2_dimension),
            torch.randn(e, H)]
    g = torch.randn(n, tp.representation_dimension)
    nodes, ang, hid = (t.to(cuda_device).requires_grad_(True) for t in base)
    out = scatter_sum(model(gather(nodes, ei), ang, hid), ei)
    grads = torch.autograd.grad(out, (nodes, ang, hid, model.radial_out.weight), g.to(cuda_device))
    coef = torch.from_numpy(tp._coefficient_values).double()
    nd, ad, hd = (t.double().requires_grad_(True) for t in base)
    alpha = model.radial_out.weight.detach().cpu().double().requires_grad_(True)
    msg = torch_uvu_flat(nd.index_select(0, src.cpu()), ad, hd @ alpha.t(), tp.entries_in1,
                         tp.entries_in2, tp.paths, coef, U, 1, False)
    od = torch.zeros(n, tp.representation_dimension, dtype=torch.float64).index_add(
        0, dst.cpu(), msg)
    want = torch.autograd.grad(od, (nd, ad, hd, alpha), g.double())
    assert _err(out, od) <= TOL
    for name, a, b in zip(("nodes", "angular", "hidden", "alpha"), grads, want):
        assert _err(a, b) <= TOL, name


def test_segment_sum_rejects_non_csr_offsets(cuda_device):
    """Offsets outside [0, value_rows] or decreasing raise the flag and zero the
    segment; valid segments of the same call are summed as usual."""
    from ictc_o2_hp_b200 import _lib
    values = torch.randn(4, 8, device=cuda_device)
    order = torch.arange(4, device=cuda_device)
    out = torch.empty(3, 8, device=cuda_device)
    offsets = torch.tensor([0, 2, 9, 1], device=cuda_device)   # [2, 9) past the end; 9 > 1
    assert _lib.graph_bad_index() == 0
    _lib.segment_sum(values, offsets, order, out)
    torch.cuda.synchronize()
    assert _lib.graph_bad_index() == 1
    assert torch.equal(out[0], values[0] + values[1])
    assert torch.count_nonzero(out[1]) == 0 and torch.count_nonzero(out[2]) == 0


@pytest.mark.parametrize("u,m_max,hidden,bias,nodes,edges", [
    (64, 3, 64, False, 700, 5000),   # config-5 shape
    (16, 2, 8, True, 50, 333),
    (32, 2, 512, True, 40, 150),     # hidden too wide for the edge tile: gathers first
])
def test_radial_messages_match_gather_then_module(u, m_max, hidden, bias, nodes, edges,
                                                  cuda_device):
    """radial_messages (the gather folded into the radial kernels) against
    model(gather(nodes, edges), angular, hidden): messages and every gradient
    (node features, angular, hidden, alpha, bias), bit for bit."""
    from ictc_o2_hp_b200 import RadialUvuTensorProduct, UvuTensorProduct
    from ictc_o2_hp_b200.graph import EdgeIndex, gather, radial_messages
    torch.manual_seed(u + edges)
    tp = UvuTensorProduct(u, 1, m_max, parity="full", parity_in2="canonical",
                          shared_weights=False)
    model = RadialUvuTensorProduct(tp, torch.nn.Linear(hidden, tp.weight_numel, bias=bias))
    model = model.to(cuda_device)
    src = torch.randint(0, nodes, (edges,), device=cuda_device)
    dst = torch.randint(0, nodes, (edges,), device=cuda_device)
    ei = EdgeIndex(src, dst, nodes)
    feats = torch.randn(nodes, tp.input1_dimension, device=cuda_device, requires_grad=True)
    ang = torch.randn(edges, tp.input2_dimension, device=cuda_device, requires_grad=True)
    h = torch.randn(edges, hidden, device=cuda_device, requires_grad=True)
    g = torch.randn(edges, tp.representation_dimension, device=cuda_device)
    params = [model.radial_out.weight] + ([model.radial_out.bias] if bias else [])
    fused = radial_messages(model, feats, ei, ang, h)
    ref = model(gather(feats, ei), ang, h)
    assert torch.equal(fused, ref)
    gf = torch.autograd.grad(fused, (feats, ang, h, *params), g)
    gr = torch.autograd.grad(ref, (feats, ang, h, *params), g)
    for a, b in zip(gf, gr):
        assert torch.equal(a, b)
    # parameter gradients alone (no node or angular role): the unfused kernels run
    only = torch.autograd.grad(radial_messages(model, feats, ei, ang, h), params, g)
    for a, b in zip(only, gr[3:]):
        assert torch.equal(a, b)
    with pytest.raises(NotImplementedError):
        (dx,) = torch.autograd.grad(radial_messages(model, feats, ei, ang, h), (feats,), g,
                                    create_graph=True)
