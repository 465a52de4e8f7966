"""Graph-level loss of the training step on the library's kernels.

``graph_sum_mse(values, graph_ptr, target)`` is the objective the EGNN
workloads train with around ``EGNN.forward`` (egnn_clean.py:141-146): the
per-graph sum of one node value (``h_out[:, 0]``) regressed on one target per
graph, ``mean_g (sum_{i in g} values[i] - target[g])^2``.  Graphs are
contiguous node ranges given by ``graph_ptr`` (G + 1 int64 offsets).  Forward
and backward run in ``egnn_graph_mse_fwd`` / ``egnn_graph_mse_bwd``: fixed
summation order (bit-identical reruns), no host synchronisation, so the
whole step stays capturable in a CUDA graph.
"""
from __future__ import annotations

import torch

from . import _native as nat


class _GraphSumMSE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, values, graph_ptr, target):
        N = values.shape[0]
        G = target.shape[0]
        lib = nat.lib()
        pred = torch.empty(max(G, 1), dtype=torch.float32, device=values.device)
        loss = torch.empty((), dtype=torch.float32, device=values.device)
        ws_bytes = lib.egnn_graph_mse_workspace_size(N)
        ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=values.device)
        nat.check(lib.egnn_graph_mse_fwd(N, G, nat.ptr(values), values.stride(0), nat.ptr(graph_ptr),
                                         nat.ptr(target), nat.ptr(pred), nat.ptr(loss), nat.ptr(ws), ws_bytes,
                                         nat.stream_ptr()), "egnn_graph_mse_fwd")
        ctx.save_for_backward(graph_ptr, pred, target)
        ctx.n = N
        return loss

    @staticmethod
    def backward(ctx, gloss):
        graph_ptr, pred, target = ctx.saved_tensors
        N, G = ctx.n, target.shape[0]
        gloss = gloss.contiguous().float()
        grad = torch.empty(N, dtype=torch.float32, device=pred.device)
        nat.check(nat.lib().egnn_graph_mse_bwd(N, G, nat.ptr(graph_ptr), nat.ptr(pred), nat.ptr(target),
                                               nat.ptr(gloss), nat.ptr(grad), 1, nat.stream_ptr()),
                  "egnn_graph_mse_bwd")
        return grad, None, None


def graph_sum_mse(values: torch.Tensor, graph_ptr: torch.Tensor, target: torch.Tensor) -> torch.Tensor:
    """mean over graphs of (sum of the graph's ``values`` - target)^2.

    values: (N,) float32 CUDA (any stride, e.g. ``h_out[:, 0]``);
    graph_ptr: (G + 1,) int64 CUDA node offsets; target: (G,) float32 CUDA.
    """
    if not (values.is_cuda and graph_ptr.is_cuda and target.is_cuda):
        raise ValueError("graph_sum_mse takes CUDA tensors (pymolecular_b200 has no CPU path)")
    if values.dim() != 1 or values.dtype != torch.float32:
        raise TypeError("values must be a 1-D float32 tensor")
    if graph_ptr.dtype != torch.int64 or graph_ptr.dim() != 1 or graph_ptr.shape[0] != target.shape[0] + 1:
        raise ValueError("graph_ptr must be (G + 1,) int64 for a (G,) target")
    target = target.contiguous().float()
    graph_ptr = graph_ptr.contiguous()
    if values.shape[0] > 0 and values.stride(0) < 1:
        values = values.contiguous()
    return _GraphSumMSE.apply(values, graph_ptr, target)


__all__ = ["graph_sum_mse"]
