"""The graph-sum MSE loss kernels against a float64 restatement.

pred_g = sum of the graph's node values, loss = mean_g (pred_g - y_g)^2 and
dL/dv_i = 2 (pred_g - y_g) / G: the CUDA forward (chunked segmented scan,
fixed order) and backward must match float64 to float32 rounding (1e-5 of
the largest magnitude) and be bit-identical between reruns, for molecule
batches, one graph much longer than a chunk, empty graphs and graphs that
start or end on a chunk boundary (2048 nodes), and strided values.
"""
import pytest
import torch

from pymolecular_b200 import graph_sum_mse
from pymolecular_b200.datasets import make_workload

pytestmark = pytest.mark.gpu

CHUNK = 2048


def _ref(values, graph_ptr, target):
    v = values.double().cpu()
    gp = graph_ptr.cpu()
    G = target.shape[0]
    pred = torch.stack([v[gp[g]:gp[g + 1]].sum() for g in range(G)]) if G else torch.zeros(0, dtype=torch.float64)
    d = pred - target.double().cpu()
    loss = (d ** 2).mean()
    grad = torch.zeros_like(v)
    for g in range(G):
        grad[gp[g]:gp[g + 1]] = 2 * d[g] / G
    return loss, grad


def _run(values, graph_ptr, target, upstream=1.0):
    v = values.detach().clone().requires_grad_(True)
    loss = graph_sum_mse(v, graph_ptr, target)
    (loss * upstream).backward()
    return loss.detach(), v.grad


def _check(sizes, seed, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    sizes = torch.tensor(sizes, dtype=torch.int64)
    gp = torch.cat([torch.zeros(1, dtype=torch.int64), sizes.cumsum(0)])
    N, G = int(gp[-1]), sizes.numel()
    values = (torch.randn(N, generator=g) * scale).cuda()
    target = (torch.randn(G, generator=g) * scale * 3).cuda()
    gpd = gp.cuda()
    loss, grad = _run(values, gpd, target, upstream=0.75)
    rl, rg = _ref(values, gpd, target)
    assert abs(loss.item() - rl.item()) <= 1e-5 * max(abs(rl.item()), 1e-30), (loss.item(), rl.item())
    rg = rg * 0.75
    assert (grad.double().cpu() - rg).abs().max().item() <= 1e-5 * rg.abs().max().item()
    loss2, grad2 = _run(values, gpd, target, upstream=0.75)
    assert torch.equal(loss, loss2) and torch.equal(grad, grad2)


def test_molecule_batch(cuda_device):
    b = make_workload(2, seed=1, n_graphs=512)
    _check((b.graph_ptr[1:] - b.graph_ptr[:-1]).tolist(), 1)


def test_one_graph_longer_than_many_chunks(cuda_device):
    _check([300_001], 2)


def test_empty_graphs_and_chunk_boundaries(cuda_device):
    sizes = [0, 1, CHUNK - 1, 1, CHUNK, 0, 0, 2 * CHUNK + 1, 3, CHUNK, CHUNK - 3, 0, 5 * CHUNK, 7, 0]
    _check(sizes, 3)


def test_many_small_graphs_and_a_hub_graph(cuda_device):
    g = torch.Generator().manual_seed(4)
    sizes = torch.randint(0, 40, (3000,), generator=g).tolist()
    sizes[1500] = 70_000
    _check(sizes, 4, scale=10.0)


def test_strided_values_and_model_output(cuda_device):
    """values = h_out[:, 0] of an (N, 3) tensor: the loss reads the column in
    place and the gradient lands in column 0 only."""
    g = torch.Generator().manual_seed(5)
    sizes = torch.tensor([5, 9, 0, 4000, 12])
    gp = torch.cat([torch.zeros(1, dtype=torch.int64), sizes.cumsum(0)]).cuda()
    N = int(gp[-1])
    h_out = torch.randn(N, 3, generator=g).cuda().requires_grad_(True)
    target = torch.randn(5, generator=g).cuda()
    loss = graph_sum_mse(h_out[:, 0], gp, target)
    loss.backward()
    rl, rg = _ref(h_out[:, 0].detach(), gp, target)
    assert abs(loss.item() - rl.item()) <= 1e-5 * abs(rl.item())
    assert (h_out.grad[:, 0].double().cpu() - rg).abs().max().item() <= 1e-5 * rg.abs().max().item()
    assert torch.count_nonzero(h_out.grad[:, 1:]) == 0
