"""CPU oracle for CSR construction (TEST INFRASTRUCTURE ONLY).

Restates, in numpy, the graph layout the reference kernels consume:
``row_ptrs`` (N+1), ``col_indices`` (E) and ``edge_id`` (E)
(forward_kernel.py:18-21, test_mem.py:62-65), with edges ``(row, col)`` =
(destination, source) aggregated over ``row`` (egnn_clean.py:61-62).  The
CSR order is a stable sort by ``row``, i.e. ``torch.sort(row, stable=True)``.
The transpose lists, for every source node, the CSR positions of its
out-edges in increasing position order (stable sort of ``col_idx``).
"""
from __future__ import annotations

import numpy as np


def csr_build(row, col, n_nodes: int):
    """-> (row_ptr int32 (N+1), col_idx, row_idx, edge_id int32 (E))."""
    row = np.asarray(row, dtype=np.int64)
    col = np.asarray(col, dtype=np.int64)
    if row.size and (row.min() < 0 or row.max() >= n_nodes or col.min() < 0 or col.max() >= n_nodes):
        raise IndexError("edge index outside [0, n_nodes)")
    perm = np.argsort(row, kind="stable")
    row_idx = row[perm]
    row_ptr = np.searchsorted(row_idx, np.arange(n_nodes + 1), side="left")
    return (row_ptr.astype(np.int32), col[perm].astype(np.int32), row_idx.astype(np.int32),
            perm.astype(np.int32))


def csr_transpose(col_idx, n_nodes: int):
    """-> (src_ptr int32 (N+1), src_edge int32 (E)) for a CSR's col_idx."""
    col_idx = np.asarray(col_idx, dtype=np.int64)
    src_edge = np.argsort(col_idx, kind="stable")
    src_ptr = np.searchsorted(col_idx[src_edge], np.arange(n_nodes + 1), side="left")
    return src_ptr.astype(np.int32), src_edge.astype(np.int32)


def csr_valid(row_ptr, col_idx, n_nodes: int) -> bool:
    """The checks egnn_graph_check applies to a caller-supplied CSR."""
    row_ptr = np.asarray(row_ptr, dtype=np.int64)
    col_idx = np.asarray(col_idx, dtype=np.int64)
    E = col_idx.size
    if row_ptr.size != n_nodes + 1 or row_ptr[0] != 0 or row_ptr[-1] != E:
        return False
    if np.any(np.diff(row_ptr) < 0):
        return False
    return bool(E == 0 or (col_idx.min() >= 0 and col_idx.max() < n_nodes))
