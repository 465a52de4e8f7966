"""Whole-model parity on the benchmark workloads, and size-independent
properties at sizes the CPU oracle cannot run in seconds.

Tolerance policy as in test_layer_gpu.py: in fp32 mode each tensor within
max(1e-5, 3 x the fp32 reference's own error) of the fp64 oracle; in bf16
mode every tensor within a flat 2e-2 of the fp64 oracle and within 5e-3 of
the rounding-exact bf16 model wherever that model is within 5e-3 of fp64.
The loss uses a deterministic per-graph sum.

The fp64 oracle (and the rounding model) run on the test's CUDA device for
these sizes: the config-5 block has 2.1M edges, whose E x H float64
intermediates the CPU would take minutes over."""
import math

import pytest
import torch

from conftest import check_bf16, check_tensors, graph_sum, rel_err, tolerances
from oracle import egnn_emulation as EM
from oracle import egnn_oracle as O
from pymolecular_b200 import CSR, EGNN
from pymolecular_b200.datasets import CONFIGS, make_workload, point_cloud, proteins, slabs

pytestmark = pytest.mark.gpu


def _model(cfg_id, precision, dev, seed=0):
    mc = CONFIGS[cfg_id]
    torch.manual_seed(seed)
    return EGNN(mc.in_node_nf, mc.hidden_nf, mc.out_node_nf, n_layers=mc.n_layers, device=dev,
                precision=precision)


def _step(model, b, csr, dev):
    h = b.h.to(dev)
    x = b.x.to(dev).clone().requires_grad_(True)
    ho, xo = model(h, x, csr)
    pred = graph_sum(ho[:, 0], b.graph_ptr)
    loss = ((pred - b.target.to(dev)) ** 2).mean()
    loss.backward()
    grads = {k: (v.grad.clone() if v.grad is not None else torch.zeros_like(v))
             for k, v in model.named_parameters()}
    model.zero_grad(set_to_none=True)
    return loss.detach(), ho.detach(), xo.detach(), x.grad, grads


def _as_flat(loss, ho, xo, grads):
    d = {"loss": loss, "h": ho, "x": xo}
    d.update(grads)
    return d


def _batch(cfg_id, size):
    """The workload of a parity case: a graph count for configs 1-4, and for
    config 5 a point cloud of `size` nodes at config 5's point density (2^20
    points in a 200 A box), with its 32 nearest neighbours per node."""
    if cfg_id == 5:
        return point_cloud(n_nodes=size, box=200.0 * (size / float(1 << 20)) ** (1.0 / 3.0), seed=0)
    return make_workload(cfg_id, n_graphs=size)


def _oracle(p, b, dev, fn, *extra, **kw):
    """fp64 oracle / rounding model on `dev`; results back on the CPU."""
    args = (b.h.double().to(dev), b.x.double().to(dev), b.row.to(dev), b.col.to(dev),
            b.graph_index().to(dev), b.target.double().to(dev))
    pd = {k: v.to(dev) for k, v in p.items()}
    loss, h, x, g = fn(pd, *args, *extra, **kw)
    g = {k: (v.cpu() if v is not None else torch.zeros_like(p[k])) for k, v in g.items()}
    return _as_flat(loss.cpu(), h.cpu(), x.cpu(), g)


# (config, precision, graphs or config-5 nodes; None = the whole config)
MODEL_CASES = [
    (1, "fp32", None),
    (2, "bf16", None),
    (2, "fp32", 128),
    (3, "fp32", 1),
    (3, "bf16", 1),
    (4, "bf16", 16),
    (5, "bf16", 1 << 16),
]


@pytest.mark.parametrize("cfg_id,precision,size", MODEL_CASES)
def test_workload_matches_oracle(cfg_id, precision, size, cuda_device):
    dev = cuda_device
    b = _batch(cfg_id, size)
    model = _model(cfg_id, precision, dev)
    csr = CSR.from_edges(b.row, b.col, n_nodes=b.n_nodes, device=dev)
    loss, ho, xo, _, grads = _step(model, b, csr, dev)
    got = _as_flat(loss, ho, xo, grads)
    p = {k: v.detach().double().cpu() for k, v in model.state_dict().items()}
    ref = _oracle(p, b, dev, O.model_grads)
    what = f"config{cfg_id} {precision} ({b.n_nodes} nodes, {b.n_edges} edges)"
    if precision == "fp32":
        p32 = {k: v.float() for k, v in p.items()}
        l32, h32, x32, g32 = O.model_grads(p32, b.h, b.x, b.row, b.col, b.graph_index(), b.target)
        g32 = {k: (g if g is not None else torch.zeros_like(p32[k])) for k, g in g32.items()}
        check_tensors(got, ref, tolerances(ref, _as_flat(l32, h32, x32, g32), 1e-5, 3.0), what)
    else:
        emu = _oracle(p, b, dev, EM.model_fwd_bwd, CONFIGS[cfg_id].n_layers, precision="bf16")
        check_bf16(got, ref, emu, what)


def test_attention_and_edge_attributes_model_bf16(cuda_device):
    """A whole bf16 H = 128 model with the attention gate and 4 edge features
    (tensor-core forward, SIMT backward) on a molecule batch, against the fp64
    oracle and the rounding-exact model."""
    dev = cuda_device
    b = make_workload(2, n_graphs=96)
    g = torch.Generator().manual_seed(3)
    ea = torch.randn(b.n_edges, 4, generator=g)
    torch.manual_seed(0)
    model = EGNN(5, 128, 1, in_edge_nf=4, n_layers=3, attention=True, device=dev, precision="bf16")
    csr = CSR.from_edges(b.row, b.col, n_nodes=b.n_nodes, device=dev)
    h = b.h.to(dev)
    x = b.x.to(dev).clone().requires_grad_(True)
    ho, xo = model(h, x, csr, ea.to(dev))          # edge_attr in the order of the edge list
    pred = graph_sum(ho[:, 0], b.graph_ptr)
    loss = ((pred - b.target.to(dev)) ** 2).mean()
    loss.backward()
    got = _as_flat(loss.detach(), ho.detach(), xo.detach(),
                   {k: v.grad.clone() for k, v in model.named_parameters()})
    p = {k: v.detach().double().cpu() for k, v in model.state_dict().items()}
    ref = _oracle(p, b, dev, O.model_grads, ea.double().to(dev), attention=True)
    emu = _oracle(p, b, dev, EM.model_fwd_bwd, 3, precision="bf16", edge_attr=ea.double().to(dev),
                  attention=True)
    check_bf16(got, ref, emu, f"attention + edge attributes, bf16 ({b.n_nodes} nodes, {b.n_edges} edges)")


def _rotation(seed):
    g = torch.Generator().manual_seed(seed)
    q, _ = torch.linalg.qr(torch.randn(3, 3, generator=g, dtype=torch.float64))
    if torch.det(q) < 0:
        q[:, 0] = -q[:, 0]
    return q.float()


@pytest.mark.parametrize("kind", ["proteins", "slabs", "pointcloud"])
def test_equivariance_at_scale(kind, cuda_device):
    """E(3) equivariance: h_out invariant and x_out = R x_out + t under x -> R x + t."""
    dev = cuda_device
    if kind == "proteins":
        b, cfg = proteins(n_graphs=2, seed=0), 3
    elif kind == "slabs":
        b, cfg = slabs(n_graphs=32, seed=0), 4
    else:
        b, cfg = point_cloud(n_nodes=1 << 16, seed=0, box=80.0), 5
    model = _model(cfg, "fp32", dev)
    csr = CSR.from_edges(b.row, b.col, n_nodes=b.n_nodes, device=dev)
    R = _rotation(7).to(dev)
    t = torch.tensor([1.0, -2.0, 0.5], device=dev)
    h, x = b.h.to(dev), b.x.to(dev)
    with torch.no_grad():
        h1, x1 = model(h, x, csr)
        h2, x2 = model(h, x @ R.T + t, csr)
    assert torch.isfinite(h1).all() and torch.isfinite(x1).all()
    assert rel_err(h2, h1) < 1e-4
    assert rel_err(x2, x1 @ R.T + t) < 1e-4


def test_gradients_finite_and_deterministic_config4(cuda_device):
    dev = cuda_device
    b = make_workload(4, n_graphs=64)
    model = _model(4, "bf16", dev)
    csr = CSR.from_edges(b.row, b.col, n_nodes=b.n_nodes, device=dev)
    a = _step(model, b, csr, dev)
    c = _step(model, b, csr, dev)
    assert math.isfinite(float(a[0]))
    for k in a[4]:
        assert torch.isfinite(a[4][k]).all(), k
        assert torch.equal(a[4][k], c[4][k]), k
