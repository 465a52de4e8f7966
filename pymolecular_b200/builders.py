"""Graph builders on the device: the step before the layer.

* :func:`get_edges_batch` / :func:`fc_graph` - fully connected intra-graph
  edges, in the order of the reference's ``get_edges`` / ``get_edges_batch``
  (models/EGNN/egnn_clean.py:167-191), for equal or ragged graph sizes.
* :func:`radius_graph` - every neighbour closer than a cutoff, optionally only
  the nearest ``max_num_neighbors`` (the radius graphs of workloads 3 and 4).
* :func:`knn_graph` - the k nearest neighbours (workload 5).
* :func:`morton_order` - Morton codes and the node order they induce
  (workload 5's node partitioning).

Graphs come back as :class:`~pymolecular_b200.csr.CSR` (destination-sorted,
with its transpose), ready for ``EGNN.forward``.  Distances are float32
d2 = (dx*dx + dy*dy) + dz*dz rounded per operation, ties go to the smaller
index: the result is a pure function of the float32 coordinates.  Everything
runs in ``libegnn_b200.so``; there is no CPU path.
"""
from __future__ import annotations

import ctypes as C
from typing import Optional, Sequence, Tuple

import torch

from . import _native as nat
from .csr import CSR, _require_cuda


def _ws(nbytes: int, device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)


def _default_device(t=None):
    if t is not None and torch.is_tensor(t) and t.is_cuda:
        return t.device
    return torch.device("cuda", torch.cuda.current_device())


def fc_graph(graph_ptr, device=None) -> CSR:
    """Fully connected graphs: graph g owns nodes [graph_ptr[g], graph_ptr[g+1]),
    row i holds every other node of its graph in increasing order."""
    device = _require_cuda(device if device is not None else _default_device(graph_ptr))
    gp_host = torch.as_tensor(graph_ptr, dtype=torch.int64).cpu().contiguous()
    if gp_host.dim() != 1 or gp_host.numel() < 2:
        raise ValueError("graph_ptr must be 1-D with at least 2 entries")
    sizes = gp_host[1:] - gp_host[:-1]
    if int(gp_host[0]) != 0 or bool((sizes < 0).any()):
        raise ValueError("graph_ptr must start at 0 and never decrease")
    N, G = int(gp_host[-1]), int(sizes.numel())
    E = int((sizes * (sizes - 1)).clamp(min=0).sum())
    i32 = dict(dtype=torch.int32, device=device)
    row_ptr = torch.empty(N + 1, **i32)
    col_idx = torch.empty(E, **i32)
    row_idx = torch.empty(E, **i32)
    gp = gp_host.to(device)
    lib = nat.lib()
    nbytes = lib.egnn_fc_graph_workspace_size(G)
    ws = _ws(nbytes, device)
    with torch.cuda.device(device):
        nat.check(lib.egnn_fc_graph(N, G, nat.ptr(gp), E, nat.ptr(row_ptr), nat.ptr(col_idx), nat.ptr(row_idx),
                                    nat.ptr(ws), nbytes, nat.stream_ptr()), "egnn_fc_graph")
    return CSR.from_sorted(N, row_ptr, col_idx, row_idx)


def get_edges_batch(n_nodes: int, batch_size: int, device=None):
    """Drop-in for the reference helper (egnn_clean.py:179-191): ``batch_size``
    fully connected graphs of ``n_nodes`` nodes.  Returns ``([rows, cols],
    edge_attr)`` with int64 edges in the reference's order and
    ``edge_attr = ones(E, 1)``, on the device."""
    gp = torch.arange(batch_size + 1, dtype=torch.int64) * int(n_nodes)
    csr = fc_graph(gp, device=device)
    rows, cols = csr.row_idx.long(), csr.col_idx.long()
    return [rows, cols], torch.ones(rows.numel(), 1, device=rows.device)


def _points(x: torch.Tensor) -> torch.Tensor:
    if not torch.is_tensor(x) or not x.is_cuda:
        raise ValueError("x must be a CUDA tensor (pymolecular_b200 has no CPU path)")
    if x.dim() != 2 or x.shape[1] != 3:
        raise ValueError("x must be (N, 3)")
    return x.detach().to(torch.float32).contiguous()


def _graph_ptr(graph_ptr, N: int, device) -> Tuple[Optional[torch.Tensor], int]:
    if graph_ptr is None:
        return None, 1
    gp = torch.as_tensor(graph_ptr).to(device=device, dtype=torch.int64).contiguous()
    if gp.dim() != 1 or gp.numel() < 2:
        raise ValueError("graph_ptr must be 1-D with at least 2 entries")
    return gp, gp.numel() - 1


def _spatial(x, mode: int, k: int, cutoff: float, graph_ptr) -> CSR:
    x = _points(x)
    device = x.device
    N = x.shape[0]
    gp, G = _graph_ptr(graph_ptr, N, device)
    desc = nat.SpatialDesc(N, G, nat.ptr(x), nat.ptr(gp), mode, int(k), float(cutoff))
    lib = nat.lib()
    nbytes = lib.egnn_spatial_workspace_size(N)
    ws = _ws(nbytes, device)
    i32 = dict(dtype=torch.int32, device=device)
    row_ptr = torch.empty(N + 1, **i32)
    with torch.cuda.device(device):
        s = nat.stream_ptr()
        nat.check(lib.egnn_spatial_count(C.byref(desc), nat.ptr(row_ptr), nat.ptr(ws), nbytes, s),
                  "egnn_spatial_count")
        E = int(row_ptr[N].item()) if N else 0
        col_idx = torch.empty(E, **i32)
        row_idx = torch.empty(E, **i32)
        nat.check(lib.egnn_spatial_fill(C.byref(desc), nat.ptr(row_ptr), nat.ptr(col_idx), nat.ptr(row_idx),
                                        nat.ptr(ws), nbytes, s), "egnn_spatial_fill")
    return CSR.from_sorted(N, row_ptr, col_idx, row_idx)


def radius_graph(x: torch.Tensor, cutoff: float, graph_ptr=None,
                 max_num_neighbors: Optional[int] = None) -> CSR:
    """Row i: every j != i of i's graph with d2 < cutoff^2, in increasing j;
    with ``max_num_neighbors`` only that many nearest, nearest first."""
    if not cutoff > 0:
        raise ValueError("cutoff must be > 0")
    cap = int(max_num_neighbors) if max_num_neighbors else 0
    return _spatial(x, nat.GRAPH_RADIUS, cap, cutoff, graph_ptr)


def knn_graph(x: torch.Tensor, k: int, graph_ptr=None, cell: float = 0.0) -> CSR:
    """Row i: the k nearest j != i of i's graph (all of them in smaller
    graphs), nearest first.  ``cell`` is an optional grid-cell hint."""
    return _spatial(x, nat.GRAPH_KNN, int(k), cell, graph_ptr)


def morton_order(x: torch.Tensor, lo: Sequence[float], hi: Sequence[float],
                 bits: int = 21) -> Tuple[torch.Tensor, torch.Tensor]:
    """(codes, perm): int64 Morton codes of the points quantised in [lo, hi)
    (3 x ``bits`` interleaved bits) and the stable sort order of the codes."""
    x = _points(x)
    N = x.shape[0]
    codes = torch.empty(N, dtype=torch.int64, device=x.device)
    perm = torch.empty(N, dtype=torch.int32, device=x.device)
    lib = nat.lib()
    nbytes = lib.egnn_morton_workspace_size(N)
    ws = _ws(nbytes, x.device)
    lo3 = (C.c_double * 3)(*[float(v) for v in lo])
    hi3 = (C.c_double * 3)(*[float(v) for v in hi])
    with torch.cuda.device(x.device):
        nat.check(lib.egnn_morton_order(N, nat.ptr(x), lo3, hi3, int(bits), nat.ptr(codes), nat.ptr(perm),
                                        nat.ptr(ws), nbytes, nat.stream_ptr()), "egnn_morton_order")
    return codes, perm.long()


__all__ = ["fc_graph", "get_edges_batch", "radius_graph", "knn_graph", "morton_order"]
