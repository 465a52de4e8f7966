"""A whole training step (forward, loss, backward, SGD update) captured as a
CUDA graph replays the eager step exactly: the kernels are deterministic, so
after the same number of updates the losses and parameters agree bitwise."""
import pytest
import torch

from conftest import graph_sum
from pymolecular_b200 import CSR, EGNN
from pymolecular_b200.datasets import CONFIGS, make_workload
from pymolecular_b200.graphs import GraphedStep

pytestmark = pytest.mark.gpu


def _setup(cfg_id, precision, n_graphs, dev):
    mc = CONFIGS[cfg_id]
    b = make_workload(cfg_id, n_graphs=n_graphs)
    torch.manual_seed(0)
    model = EGNN(mc.in_node_nf, mc.hidden_nf, mc.out_node_nf, n_layers=mc.n_layers, device=dev,
                 precision=precision)
    opt = torch.optim.SGD(model.parameters(), lr=1e-5)
    csr = CSR.from_edges(b.row, b.col, n_nodes=b.n_nodes, device=dev)
    h, x = b.h.to(dev), b.x.to(dev)
    gp, tgt = b.graph_ptr.to(dev), b.target.to(dev)

    def step():
        opt.zero_grad(set_to_none=True)
        ho, _ = model(h, x, csr)
        loss = ((graph_sum(ho[:, 0], gp) - tgt) ** 2).mean()
        loss.backward()
        opt.step()
        return loss.detach()

    return model, step


@pytest.mark.parametrize("cfg_id,precision,n_graphs", [(1, "fp32", 32), (2, "bf16", 64)])
def test_graphed_step_matches_eager(cfg_id, precision, n_graphs, cuda_device):
    warmup, k = 3, 4
    model_e, step_e = _setup(cfg_id, precision, n_graphs, cuda_device)
    for _ in range(warmup):
        step_e()
    eager = [step_e().clone() for _ in range(k)]

    model_g, step_g = _setup(cfg_id, precision, n_graphs, cuda_device)
    graphed = GraphedStep(step_g, warmup=warmup)   # the capture itself runs nothing
    replayed = [graphed.replay().clone() for _ in range(k)]
    torch.cuda.synchronize()
    graphed.release()

    eager, replayed = torch.stack(eager), torch.stack(replayed)
    assert torch.isfinite(eager).all()
    assert not torch.equal(eager[0], eager[-1])   # the updates change the loss
    assert torch.equal(eager, replayed)
    for (name, pe), pg in zip(model_e.named_parameters(), model_g.parameters()):
        assert torch.equal(pe, pg), name
