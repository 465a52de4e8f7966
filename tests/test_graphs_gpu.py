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



def test_graphed_end_to_end_step_reads_new_host_data(cuda_device):
    """A captured public-API step (pinned H2D of inputs and edge list, CSR built
    on the device with deferred validation, forward, backward, loss D2H) picks
    up new data written into the pinned buffers before each replay and matches
    the eager step on that data bitwise."""
    from pymolecular_b200.datasets import molecules
    mc = CONFIGS[1]
    dev = cuda_device
    b0 = molecules(24, seed=1)
    b1 = molecules(24, seed=1)            # same graph sizes and edges ...
    b1.x.mul_(0.5).add_(0.3)              # ... new coordinates and features
    b1.h.copy_(torch.roll(b1.h, 1, 0))
    torch.manual_seed(0)
    model = EGNN(mc.in_node_nf, mc.hidden_nf, mc.out_node_nf, n_layers=mc.n_layers, device=dev)
    host = {k: getattr(b0, k).clone().pin_memory() for k in ("h", "x", "row", "col")}
    gp = b0.graph_ptr.to(dev)
    loss_host = torch.empty(1).pin_memory()
    holder = {}

    def step(check):
        model.zero_grad(set_to_none=False)
        d = {k: v.to(dev, non_blocking=True) for k, v in host.items()}
        csr = CSR.from_edges(d["row"], d["col"], n_nodes=b0.h.shape[0], device=dev, check=check)
        ho, _ = model(d["h"], d["x"], csr)
        loss = (graph_sum(ho[:, 0], gp) ** 2).mean()
        loss.backward()
        loss_host.copy_(loss.detach().reshape(1), non_blocking=True)
        holder["csr"] = csr
        return loss.detach()

    graphed = GraphedStep(lambda: step(False), warmup=2)   # grads exist before the capture
    grads = [v.grad for v in model.parameters()]
    for b in (b0, b1, b0):
        for k in host:
            host[k].copy_(getattr(b, k))
        graphed.replay()
        torch.cuda.synchronize()
        holder["csr"].raise_if_invalid()
        got, got_g = loss_host.clone(), [g.clone() for g in grads]
        step(True)                                          # eager, into the same grad tensors
        torch.cuda.synchronize()
        assert all(v.grad is g for v, g in zip(model.parameters(), grads))
        assert torch.equal(got, loss_host)
        for u, g in zip(got_g, grads):
            assert torch.equal(u, g)
    assert not torch.equal(got_g[0], torch.zeros_like(got_g[0]))
    graphed.release()
