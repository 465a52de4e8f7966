"""Whole-model parity on the benchmark workloads, and size-independent
properties at sizes the CPU oracle cannot run in seconds.

Tolerance policy as in test_layer_gpu.py: each tensor within
max(1e-5, 3 x the fp32 reference's error) in fp32 mode, and within
max(2e-2, 3 x the error of the rounding-exact bf16 model) in bf16 mode, of
the fp64 oracle.  The loss uses a deterministic per-graph sum."""
import math

import pytest
import torch

from conftest import check_tensors, graph_sum, rel_err, tolerances
from oracle import egnn_emulation as EM
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


@pytest.mark.parametrize("cfg_id,precision,n_graphs", [(1, "fp32", None), (2, "bf16", None),
                                                       (2, "fp32", 128), (4, "bf16", 8)])
def test_molecule_workload_matches_oracle(cfg_id, precision, n_graphs, cuda_device):
    dev = cuda_device
    b = make_workload(cfg_id, n_graphs=n_graphs)
    model = _model(cfg_id, precision, dev)
    csr = CSR.from_edges(b.row, b.col, n_nodes=b.n_nodes, device=dev)
    loss, ho, xo, _, grads = _step(model, b, csr, dev)
    got = _as_flat(loss, ho, xo, grads)
    p = {k: v.detach().double().cpu() for k, v in model.state_dict().items()}
    rl, rh, rx, rg = O.model_grads(p, b.h.double(), b.x.double(), b.row, b.col, b.graph_index(),
                                   b.target.double())
    rg = {k: (g if g is not None else torch.zeros_like(p[k])) for k, g in rg.items()}
    ref = _as_flat(rl, rh, rx, rg)
    if precision == "fp32":
        p32 = {k: v.float() for k, v in p.items()}
        l32, h32, x32, g32 = O.model_grads(p32, b.h, b.x, b.row, b.col, b.graph_index(), b.target)
        g32 = {k: (g if g is not None else torch.zeros_like(p32[k])) for k, g in g32.items()}
        tol = tolerances(ref, _as_flat(l32, h32, x32, g32), 1e-5, 3.0)
    else:
        mc = CONFIGS[cfg_id]
        el, eh, ex, eg = EM.model_fwd_bwd(p, b.h, b.x, b.row, b.col, b.graph_index(), b.target,
                                          mc.n_layers, precision="bf16")
        tol = tolerances(ref, _as_flat(el, eh, ex, eg), 2e-2, 3.0)
    check_tensors(got, ref, tol, f"config{cfg_id} {precision}")


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
