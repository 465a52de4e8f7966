"""CPU oracle of the device graph builders (TEST INFRASTRUCTURE ONLY).

Plain numpy restatements of the graphs the workloads feed the layer, each in
the exact form the CUDA builders (pymolecular_b200/csrc/graph_build.cu)
promise, so that the device output can be compared bit for bit:

* fully connected intra-graph edges in the order of the reference's
  ``get_edges`` / ``get_edges_batch`` (models/EGNN/egnn_clean.py:167-191):
  row i, then every j != i of its graph in increasing order;
* radius graphs: every j != i of i's graph with d2 < cutoff^2, sources in
  increasing j, or only the ``max_nbrs`` nearest (nearest first) when capped;
* k-nearest-neighbour graphs: the k nearest j != i of i's graph, nearest first.

Distances: d2 = (dx*dx + dy*dy) + dz*dz in float32 with every operation
rounded (dx = x_i - x_j), cutoff^2 = float32(cutoff) * float32(cutoff), ties
in d2 broken by the smaller j.  The survey's workloads describe these graphs
(radius 10 A, radius 6 A capped at 50 nearest, 32 nearest neighbours) and the
dataset generators build them with scipy's cKDTree in float64; the tests pin
this oracle to cKDTree on inputs without near-ties.

Morton order: codes of 3 x ``bits`` interleaved bits of
floor((float64(x) - lo) / (hi - lo) * 2^bits) clipped to [0, 2^bits), bit b
of axis a at position 3b + a (the survey's config-5 ordering), nodes sorted
stably by code.
"""
from __future__ import annotations

import numpy as np


def _graph_ranges(n_nodes, graph_ptr):
    if graph_ptr is None:
        return [(0, n_nodes)]
    gp = np.asarray(graph_ptr, dtype=np.int64)
    return [(int(gp[g]), int(gp[g + 1])) for g in range(len(gp) - 1)]


def fc_graph(graph_ptr):
    """(row, col) int64 of get_edges_batch generalised to ragged graphs."""
    gp = np.asarray(graph_ptr, dtype=np.int64)
    rows, cols = [], []
    for g in range(len(gp) - 1):
        a, b = int(gp[g]), int(gp[g + 1])
        n = b - a
        if n < 2:
            continue
        i = np.repeat(np.arange(a, b), n - 1)
        j = np.tile(np.arange(a, b), n).reshape(n, n)
        j = j[~np.eye(n, dtype=bool)].reshape(-1)
        rows.append(i)
        cols.append(j)
    if not rows:
        return np.zeros(0, np.int64), np.zeros(0, np.int64)
    return np.concatenate(rows), np.concatenate(cols)


def sqdist_f32(xi, xj):
    """d2 of point xi (3,) to the rows of xj (m, 3), float32 and rounded per op."""
    xi = np.asarray(xi, dtype=np.float32)
    xj = np.asarray(xj, dtype=np.float32)
    d = xi[None, :] - xj
    return (d[:, 0] * d[:, 0] + d[:, 1] * d[:, 1]) + d[:, 2] * d[:, 2]


def _rows_to_csr(n_nodes, per_row):
    row_ptr = np.zeros(n_nodes + 1, dtype=np.int64)
    for i, js in enumerate(per_row):
        row_ptr[i + 1] = row_ptr[i] + len(js)
    col = np.concatenate(per_row).astype(np.int64) if per_row and row_ptr[-1] else np.zeros(0, np.int64)
    return row_ptr, col


def radius_graph(x, cutoff, graph_ptr=None, max_nbrs=None):
    """(row_ptr, col_idx) of the radius graph (brute force per graph)."""
    x = np.asarray(x, dtype=np.float32)
    n = x.shape[0]
    c2 = np.float32(cutoff) * np.float32(cutoff)
    per_row = [None] * n
    for a, b in _graph_ranges(n, graph_ptr):
        idx = np.arange(a, b)
        for i in range(a, b):
            d2 = sqdist_f32(x[i], x[a:b])
            sel = (d2 < c2) & (idx != i)
            js, dd = idx[sel], d2[sel]
            if max_nbrs is not None and max_nbrs > 0:
                order = np.lexsort((js, dd))[:max_nbrs]   # by d2, then j
                js = js[order]
            per_row[i] = js
    return _rows_to_csr(n, per_row)


def knn_graph(x, k, graph_ptr=None):
    """(row_ptr, col_idx) of the k-nearest-neighbour graph (brute force per graph)."""
    x = np.asarray(x, dtype=np.float32)
    n = x.shape[0]
    per_row = [None] * n
    for a, b in _graph_ranges(n, graph_ptr):
        idx = np.arange(a, b)
        for i in range(a, b):
            per_row[i] = knn_row(x, i, k, a, b, idx)
    return _rows_to_csr(n, per_row)


def knn_row(x, i, k, a, b, idx=None):
    """The k nearest j != i in [a, b), nearest first, ties by j."""
    if idx is None:
        idx = np.arange(a, b)
    d2 = sqdist_f32(x[i], x[a:b])
    sel = idx != i
    js, dd = idx[sel], d2[sel]
    if k < len(dd):
        # every candidate up to the k-th smallest distance, ties included, so
        # the (d2, j) order below is unaffected by the cut
        kth = np.partition(dd, k - 1)[k - 1] if k > 0 else -np.inf
        keep = dd <= kth
        js, dd = js[keep], dd[keep]
    order = np.lexsort((js, dd))[:k]
    return js[order]


def morton_codes(x, lo, hi, bits=21):
    """uint64 Morton codes of float32 points quantised in float64."""
    p = np.asarray(x, dtype=np.float32).astype(np.float64)
    lo = np.asarray(lo, dtype=np.float64)
    hi = np.asarray(hi, dtype=np.float64)
    q = np.floor((p - lo) / (hi - lo) * float(1 << bits))
    q = np.clip(q, 0, (1 << bits) - 1).astype(np.uint64)
    code = np.zeros(p.shape[0], dtype=np.uint64)
    for bit in range(bits):
        for a in range(3):
            code |= ((q[:, a] >> np.uint64(bit)) & np.uint64(1)) << np.uint64(3 * bit + a)
    return code


def morton_order(x, lo, hi, bits=21):
    code = morton_codes(x, lo, hi, bits)
    return code, np.argsort(code, kind="stable")
