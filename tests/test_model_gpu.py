"""Whole-model parity on the benchmark workloads, and size-independent
properties at sizes the CPU oracle cannot run in seconds."""
import math

import pytest
import torch

from conftest import rel_err
from oracle import egnn_oracle as O
from pymolecular_b200 import CSR, EGNN
from pymolecular_b200.datasets import CONFIGS, make_workload, molecules, point_cloud, proteins, slabs

pytestmark = pytest.mark.gpu

TOL = {"fp32": 1e-5, "bf16": 2e-2}


def _model(cfg_id, precision, dev, seed=0):
    mc = CONFIGS[cfg_id]
    torch.manual_seed(seed)
    return EGNN(mc.in_node_nf, mc.hidden_nf, mc.out_node_nf, n_layers=mc.n_layers, device=dev,
                precision=precision)


def _step(model, b, csr, dev):
    h = b.h.to(dev)
    x = b.x.to(dev).clone().requires_grad_(True)
    ho, xo = model(h, x, csr)
    gi = b.graph_index().to(dev)
    pred = torch.zeros(b.n_graphs, device=dev).index_add_(0, gi, ho[:, 0])
    loss = ((pred - b.target.to(dev)) ** 2).mean()
    loss.backward()
    grads = {k: (v.grad.clone() if v.grad is not None else torch.zeros_like(v))
             for k, v in model.named_parameters()}
    model.zero_grad(set_to_none=True)
    return loss.detach(), ho.detach(), xo.detach(), x.grad, grads


def _oracle_step(model, b):
    p = {k: v.detach().double().cpu() for k, v in model.state_dict().items()}
    loss, ho, xo, grads = O.model_grads(p, b.h.double(), b.x.double(), b.row, b.col, b.graph_index(),
                                        b.target.double())
    return loss, ho, xo, {k: (g if g is not None else torch.zeros_like(p[k])) for k, g in grads.items()}


@pytest.mark.parametrize("cfg_id,precision,n_graphs", [(1, "fp32", None), (2, "bf16", None),
                                                       (2, "fp32", 128)])
def test_molecule_workload_matches_oracle(cfg_id, precision, n_graphs, cuda_device):
    dev = cuda_device
    b = make_workload(cfg_id, n_graphs=n_graphs)
    model = _model(cfg_id, precision, dev)
    csr = CSR.from_edges(b.row, b.col, n_nodes=b.n_nodes, device=dev)
    loss, ho, xo, _, grads = _step(model, b, csr, dev)
    rl, rh, rx, rg = _oracle_step(model, b)
    tol = TOL[precision]
    assert rel_err(loss, rl) < tol
    assert rel_err(ho, rh) < tol
    assert rel_err(xo, rx) < tol
    bad = {k: rel_err(grads[k], rg[k]) for k in rg if not rel_err(grads[k], rg[k]) < tol}
    assert not bad, bad


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
