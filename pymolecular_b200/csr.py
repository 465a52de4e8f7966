"""Destination-sorted CSR graphs on the device.

The reference kernels consume a CSR triple ``row_ptrs`` / ``col_indices`` /
``edge_id`` (forward_kernel.py:18-21) built on the host (test_mem.py:62-65);
``E_GCL``/``EGNN`` take an edge list ``[row, col]`` (egnn_clean.py:61, 141).
``CSR.from_edges`` converts the edge list once on the GPU with a stable sort
by ``row`` (so CSR order == ``torch.sort(row, stable=True)``) and also builds
the transpose CSR the backward needs for its source-side gradients.
"""
from __future__ import annotations

import ctypes as C
from typing import Optional, Sequence

import torch

from . import _native as nat


def _require_cuda(device) -> torch.device:
    device = torch.device(device)
    if device.type != "cuda":
        raise ValueError("pymolecular_b200 runs on CUDA devices only (no CPU fallback); "
                         f"got device {device}")
    return device


class CSR:
    """dst-sorted CSR + transpose, all int32 tensors on one CUDA device.

    row_ptr (N+1), col_idx (E), row_idx (E), edge_id (E): CSR position k holds
    edge ``edge_id[k]`` of the original list, going ``col_idx[k] -> row_idx[k]``.
    src_ptr (N+1), src_edge (E): the CSR positions of each source node's
    out-edges, in increasing position order.
    """

    def __init__(self, n_nodes: int, row_ptr, col_idx, row_idx, edge_id, src_ptr, src_edge):
        self.n_nodes = int(n_nodes)
        self.n_edges = int(col_idx.numel())
        self.row_ptr, self.col_idx, self.row_idx = row_ptr, col_idx, row_idx
        self.edge_id, self.src_ptr, self.src_edge = edge_id, src_ptr, src_edge
        self.device = row_ptr.device
        self.status = None   # deferred validation flag (from_edges(check=False))
        self._struct = None

    # ---- construction --------------------------------------------------------
    @classmethod
    def from_edges(cls, row, col, n_nodes: Optional[int] = None, device=None, check: bool = True) -> "CSR":
        """Build from an edge list (row = destination, col = source).

        ``check=True`` validates the indices and raises on one outside
        [0, n_nodes) (a host synchronisation).  ``check=False`` keeps the call
        asynchronous (capturable in a CUDA graph): the result of the same
        validation stays on the device in ``csr.status`` and
        :meth:`raise_if_invalid` reads it; until then out-of-range sources are
        mapped to node 0, so the layer never indexes out of bounds."""
        if device is None:
            device = row.device if row.is_cuda else torch.device("cuda", torch.cuda.current_device())
        device = _require_cuda(device)
        row = torch.as_tensor(row).to(device=device, dtype=torch.int64).contiguous()
        col = torch.as_tensor(col).to(device=device, dtype=torch.int64).contiguous()
        if row.shape != col.shape or row.dim() != 1:
            raise ValueError("row and col must be 1-D tensors of equal length")
        if n_nodes is None:
            n_nodes = int(torch.maximum(row.max(), col.max()).item()) + 1 if row.numel() else 0
        N, E = int(n_nodes), int(row.numel())
        i32 = dict(dtype=torch.int32, device=device)
        row_ptr = torch.empty(N + 1, **i32)
        col_idx = torch.empty(E, **i32)
        row_idx = torch.empty(E, **i32)
        edge_id = torch.empty(E, **i32)
        src_ptr = torch.empty(N + 1, **i32)
        src_edge = torch.empty(E, **i32)
        lib = nat.lib()
        ws_bytes = lib.egnn_csr_workspace_size(N, E)
        ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=device)
        status = None if check else torch.zeros(1, **i32)
        with torch.cuda.device(device):
            s = nat.stream_ptr()
            if check:
                nat.check(lib.egnn_csr_build(N, E, nat.ptr(row), nat.ptr(col), nat.ptr(row_ptr),
                                             nat.ptr(col_idx), nat.ptr(row_idx), nat.ptr(edge_id),
                                             nat.ptr(ws), ws_bytes, s), "egnn_csr_build")
            else:
                nat.check(lib.egnn_csr_build_async(N, E, nat.ptr(row), nat.ptr(col), nat.ptr(row_ptr),
                                                   nat.ptr(col_idx), nat.ptr(row_idx), nat.ptr(edge_id),
                                                   nat.ptr(status), nat.ptr(ws), ws_bytes, s),
                          "egnn_csr_build_async")
            nat.check(lib.egnn_csr_transpose(N, E, nat.ptr(row_ptr), nat.ptr(col_idx),
                                             nat.ptr(src_ptr), nat.ptr(src_edge), nat.ptr(ws),
                                             ws_bytes, s), "egnn_csr_transpose")
        out = cls(N, row_ptr, col_idx, row_idx, edge_id, src_ptr, src_edge)
        out.status = status
        return out

    def raise_if_invalid(self) -> None:
        """Reads the deferred validation of ``from_edges(check=False)`` (a host
        synchronisation) and raises EgnnError(EGNN_ERR_INDEX) if an edge index
        was outside [0, n_nodes)."""
        if self.status is not None and int(self.status.item()) != 0:
            raise nat.EgnnError(nat.EGNN_ERR_INDEX,
                                f"edge index outside [0, {self.n_nodes}) in the edge list of this CSR")

    @classmethod
    def from_csr(cls, row_ptr, col_idx, edge_id=None, n_nodes: Optional[int] = None,
                 device=None, check: bool = True) -> "CSR":
        """Wrap a caller-built dst CSR (reference layout, forward_kernel.py:18-21).

        The CSR is validated on the device (EgnnError with status
        EGNN_ERR_INDEX when malformed) and its transpose is built.
        """
        device = _require_cuda(device if device is not None else
                               (row_ptr.device if row_ptr.is_cuda else "cuda"))
        i32 = dict(dtype=torch.int32, device=device)
        row_ptr = torch.as_tensor(row_ptr).to(**i32).contiguous()
        col_idx = torch.as_tensor(col_idx).to(**i32).contiguous()
        N = int(n_nodes) if n_nodes is not None else row_ptr.numel() - 1
        E = int(col_idx.numel())
        if row_ptr.numel() != N + 1:
            raise ValueError("row_ptr must have n_nodes + 1 entries")
        if edge_id is None:
            edge_id = torch.arange(E, **i32)
        edge_id = torch.as_tensor(edge_id).to(**i32).contiguous()
        lib = nat.lib()
        ws_bytes = max(lib.egnn_csr_workspace_size(N, E), 256)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=device)
        with torch.cuda.device(device):
            s = nat.stream_ptr()
            g0 = nat.Graph(nat.ptr(row_ptr), nat.ptr(col_idx), None, nat.ptr(edge_id), None, None)
            if check:
                nat.check(lib.egnn_graph_check(N, E, C.byref(g0), nat.ptr(ws), ws_bytes, s),
                          "egnn_graph_check")
            deg = row_ptr[1:] - row_ptr[:-1]
            row_idx = torch.repeat_interleave(torch.arange(N, **i32), deg.long(),
                                              output_size=E).to(torch.int32)
            src_ptr = torch.empty(N + 1, **i32)
            src_edge = torch.empty(E, **i32)
            nat.check(lib.egnn_csr_transpose(N, E, nat.ptr(row_ptr), nat.ptr(col_idx),
                                             nat.ptr(src_ptr), nat.ptr(src_edge), nat.ptr(ws),
                                             ws_bytes, s), "egnn_csr_transpose")
        return cls(N, row_ptr, col_idx, row_idx, edge_id.contiguous(), src_ptr, src_edge)

    @classmethod
    def from_sorted(cls, n_nodes: int, row_ptr, col_idx, row_idx) -> "CSR":
        """Wrap a CSR the device builders produced (rows already in order, edge
        ids = CSR positions) and build its transpose."""
        device = row_ptr.device
        N, E = int(n_nodes), int(col_idx.numel())
        i32 = dict(dtype=torch.int32, device=device)
        edge_id = torch.arange(E, **i32)
        src_ptr = torch.empty(N + 1, **i32)
        src_edge = torch.empty(E, **i32)
        lib = nat.lib()
        ws_bytes = max(lib.egnn_csr_workspace_size(N, E), 256)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=device)
        with torch.cuda.device(device):
            nat.check(lib.egnn_csr_transpose(N, E, nat.ptr(row_ptr), nat.ptr(col_idx), nat.ptr(src_ptr),
                                             nat.ptr(src_edge), nat.ptr(ws), ws_bytes, nat.stream_ptr()),
                      "egnn_csr_transpose")
        return cls(N, row_ptr, col_idx, row_idx, edge_id, src_ptr, src_edge)

    # ---- views -----------------------------------------------------------------
    def struct(self) -> nat.Graph:
        if self._struct is None:
            self._struct = nat.Graph(nat.ptr(self.row_ptr), nat.ptr(self.col_idx),
                                     nat.ptr(self.row_idx), nat.ptr(self.edge_id),
                                     nat.ptr(self.src_ptr), nat.ptr(self.src_edge))
        return self._struct

    def check(self) -> None:
        """Re-validate every index array on the device."""
        lib = nat.lib()
        ws = torch.empty(256, dtype=torch.uint8, device=self.device)
        with torch.cuda.device(self.device):
            nat.check(lib.egnn_graph_check(self.n_nodes, self.n_edges, C.byref(self.struct()),
                                           nat.ptr(ws), 256, nat.stream_ptr()), "egnn_graph_check")

    def degree(self) -> torch.Tensor:
        return (self.row_ptr[1:] - self.row_ptr[:-1]).to(torch.int64)

    def edge_index(self) -> Sequence[torch.Tensor]:
        """(row, col) int64 in CSR order."""
        return self.row_idx.long(), self.col_idx.long()

    def __repr__(self) -> str:
        return f"CSR(n_nodes={self.n_nodes}, n_edges={self.n_edges}, device={self.device})"


def as_csr(edges, n_nodes: int, device) -> CSR:
    """Accept a CSR or a reference-style ``[row, col]`` pair."""
    if isinstance(edges, CSR):
        if edges.n_nodes != n_nodes:
            raise ValueError(f"CSR has {edges.n_nodes} nodes, features have {n_nodes}")
        return edges
    if isinstance(edges, (list, tuple)) and len(edges) == 2:
        return CSR.from_edges(edges[0], edges[1], n_nodes=n_nodes, device=device)
    raise TypeError("edges must be a CSR or a [row, col] pair of index tensors")
