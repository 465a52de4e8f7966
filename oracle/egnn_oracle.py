"""CPU oracle for the EGNN layer (TEST INFRASTRUCTURE ONLY).

This file restates, in plain PyTorch on the CPU, the algorithm of the
reference's ``models/EGNN/egnn_clean.py`` (SatxaFortuny/PyMolecular).  It is
the checker the parity tests, ``__graft_entry__.smoke()`` and ``bench.py``'s
CPU-baseline leg compare against.  The product (``pymolecular_b200``) never
imports it; the CUDA path fails loudly instead of falling back here.

Pinning: ``tests/golden/make_golden.py`` imports the reference module itself
(when its sources are available) and stores its fp64 outputs and gradients as
fixtures; ``tests/test_oracle.py`` checks this restatement against them.

Parameters are a dict keyed exactly like the reference ``state_dict``
(``embedding_in.weight``, ``gcl_0.edge_mlp.0.weight``, ...), so weights move
between the reference, this oracle and the CUDA modules unchanged.
Backward is autograd of this forward, as in the reference.
"""
from __future__ import annotations

from typing import Dict, Optional

import torch

Params = Dict[str, torch.Tensor]


def _linear(p: Params, name: str, x: torch.Tensor) -> torch.Tensor:
    """nn.Linear: y = x W^T + b (b absent for coord_mlp.2, egnn_clean.py:33)."""
    y = x @ p[name + ".weight"].t()
    b = p.get(name + ".bias")
    return y + b if b is not None else y


def segment_sum(data: torch.Tensor, seg: torch.Tensor, n: int) -> torch.Tensor:
    """unsorted_segment_sum (egnn_clean.py:149-154): scatter_add over ``seg``."""
    out = data.new_zeros((n, data.shape[1]))
    out.index_add_(0, seg, data)
    return out


def segment_mean(data: torch.Tensor, seg: torch.Tensor, n: int) -> torch.Tensor:
    """unsorted_segment_mean (egnn_clean.py:157-164): sum / max(count, 1)."""
    s = segment_sum(data, seg, n)
    cnt = torch.bincount(seg, minlength=n).to(data.dtype).clamp(min=1)
    return s / cnt[:, None]


def coord2radial(row, col, x, normalize: bool, eps: float = 1e-8):
    """egnn_clean.py:84-93: diff = x[row]-x[col], radial = |diff|^2 (detached norm)."""
    diff = x[row] - x[col]
    radial = (diff ** 2).sum(1, keepdim=True)
    if normalize:
        norm = torch.sqrt(radial).detach() + eps
        diff = diff / norm
    return radial, diff


def e_gcl(p: Params, prefix: str, h, row, col, x, edge_attr=None, *, residual=True,
          attention=False, normalize=False, tanh=False, coords_agg="mean"):
    """E_GCL.forward (egnn_clean.py:95-103) -> (h', x').

    edge_model (:49-58), coord_model (:72-82), node_model (:60-70); the act
    function is SiLU (the reference default, egnn_clean.py:11).
    """
    n = h.shape[0]
    radial, diff = coord2radial(row, col, x, normalize)
    parts = [h[row], h[col], radial]
    if edge_attr is not None:
        parts.append(edge_attr)
    m = torch.cat(parts, dim=1)
    m = torch.nn.functional.silu(_linear(p, prefix + "edge_mlp.0", m))
    m = torch.nn.functional.silu(_linear(p, prefix + "edge_mlp.2", m))
    if attention:
        m = m * torch.sigmoid(_linear(p, prefix + "att_mlp.0", m))
    phi = _linear(p, prefix + "coord_mlp.2",
                  torch.nn.functional.silu(_linear(p, prefix + "coord_mlp.0", m)))
    if tanh:
        phi = torch.tanh(phi)
    trans = diff * phi
    if coords_agg == "sum":
        xa = segment_sum(trans, row, n)
    elif coords_agg == "mean":
        xa = segment_mean(trans, row, n)
    else:
        raise ValueError(f"Wrong coords_agg parameter {coords_agg}")
    x = x + xa
    agg = segment_sum(m, row, n)
    out = _linear(p, prefix + "node_mlp.2",
                  torch.nn.functional.silu(_linear(p, prefix + "node_mlp.0", torch.cat([h, agg], 1))))
    if residual:
        out = h + out
    return out, x


def egnn(p: Params, h, x, row, col, edge_attr=None, n_layers: Optional[int] = None, **flags):
    """EGNN.forward (egnn_clean.py:141-146): embedding_in, L x E_GCL, embedding_out."""
    if n_layers is None:
        n_layers = len({k.split(".")[0] for k in p if k.startswith("gcl_")})
    h = _linear(p, "embedding_in", h)
    for i in range(n_layers):
        h, x = e_gcl(p, f"gcl_{i}.", h, row, col, x, edge_attr, **flags)
    h = _linear(p, "embedding_out", h)
    return h, x


def init_params(in_node_nf: int, hidden_nf: int, out_node_nf: int, n_layers: int,
                in_edge_nf: int = 0, attention: bool = False, seed: int = 0,
                dtype=torch.float32) -> Params:
    """Parameters with the reference's shapes, names and init scheme.

    Shapes follow EGNN.__init__ / E_GCL.__init__ (egnn_clean.py:107-139,
    11-47): nn.Linear default init (kaiming-uniform weights, uniform bias in
    +-1/sqrt(fan_in)), and xavier_uniform(gain=0.001) for the bias-free
    coord_mlp.2 (egnn_clean.py:33-34).  Drawn from a seeded generator in
    module registration order.
    """
    g = torch.Generator().manual_seed(seed)
    p: Params = {}

    def lin(name, fan_in, fan_out, bias=True):
        bound = 1.0 / (fan_in ** 0.5)
        p[name + ".weight"] = (torch.rand(fan_out, fan_in, generator=g, dtype=torch.float64) * 2 - 1) * bound
        if bias:
            p[name + ".bias"] = (torch.rand(fan_out, generator=g, dtype=torch.float64) * 2 - 1) * bound

    H = hidden_nf
    lin("embedding_in", in_node_nf, H)
    lin("embedding_out", H, out_node_nf)
    for i in range(n_layers):
        pre = f"gcl_{i}."
        lin(pre + "edge_mlp.0", 2 * H + 1 + in_edge_nf, H)
        lin(pre + "edge_mlp.2", H, H)
        lin(pre + "node_mlp.0", 2 * H, H)
        lin(pre + "node_mlp.2", H, H)
        lin(pre + "coord_mlp.0", H, H)
        a = 0.001 * (6.0 / (H + 1)) ** 0.5
        p[pre + "coord_mlp.2.weight"] = (torch.rand(1, H, generator=g, dtype=torch.float64) * 2 - 1) * a
        if attention:
            lin(pre + "att_mlp.0", H, 1)
    return {k: v.to(dtype) for k, v in p.items()}


def graph_sum_mse(h_out: torch.Tensor, graph_index: torch.Tensor, target: torch.Tensor):
    """Loss of the benchmark step: mean over graphs of (sum of node outputs - y)^2."""
    pred = segment_sum(h_out, graph_index, target.shape[0])[:, 0]
    return ((pred - target.to(pred.dtype)) ** 2).mean()


def layer_grads(p: Params, prefix: str, h, row, col, x, gh, gx, edge_attr=None, **flags):
    """One E_GCL forward+backward with upstream grads (gh, gx).

    Returns (h', x', dh, dx, {param name: grad}) computed by autograd.
    """
    names = [k for k in p if k.startswith(prefix)]
    leaf = {k: p[k].detach().clone().requires_grad_(True) for k in names}
    hh = h.detach().clone().requires_grad_(True)
    xx = x.detach().clone().requires_grad_(True)
    ho, xo = e_gcl(leaf, prefix, hh, row, col, xx, edge_attr, **flags)
    torch.autograd.backward([ho, xo], [gh, gx])
    return ho.detach(), xo.detach(), hh.grad, xx.grad, {k: v.grad for k, v in leaf.items()}


def model_grads(p: Params, h, x, row, col, graph_index, target, edge_attr=None, **flags):
    """Whole-model forward + graph-sum MSE loss + backward (autograd).

    Returns (loss, h_out, x_out, {param name: grad}).
    """
    leaf = {k: v.detach().clone().requires_grad_(True) for k, v in p.items()}
    ho, xo = egnn(leaf, h, x, row, col, edge_attr, **flags)
    loss = graph_sum_mse(ho, graph_index, target)
    loss.backward()
    return loss.detach(), ho.detach(), xo.detach(), {k: v.grad for k, v in leaf.items()}
