"""Seeded synthetic graph batches for the five EGNN workloads.

The reference ships one generator, ``datasets_loaders.generate_graph_data``
(datasets_loaders.py:3-39), which draws a uniform-degree random CSR on CUDA.
None of the benchmarked workloads uses that graph family, so this module
builds the five workloads the benchmark is quoted on instead.  Everything is
drawn on the CPU from a ``torch.Generator`` / ``numpy.random.Generator`` seeded
explicitly, so the oracle and the GPU path see identical bits.

Edge convention (egnn_clean.py:84-103): an edge is ``(row, col) = (i, j)``,
``row`` is the destination that aggregates, ``col`` the source.  Every
generator returns edges already sorted by ``row`` with a stable order inside a
row, i.e. dst-sorted CSR order, like ``get_edges`` (egnn_clean.py:167-176).

Workloads (hidden size, layers, precision are model settings, see ``CONFIGS``):

1. 96 molecules, n ~ U{9..29}, fully connected, 5-type one-hot, N(0, 1.5^2).
2. as 1 with 512 molecules.
3. 16 protein-like graphs, n ~ U{2000..4000}, self-avoiding-ish 3.8 A walk,
   radius 10 A graph, 20-type uniform one-hot.
4. 256 slab-like graphs, n ~ U{50..200}, uniform in a 12x12x20 A box with
   1.8 A minimum separation, radius 6 A capped at the 50 nearest per row,
   40-type Zipf(1.2) one-hot.
5. one graph of 2^20 nodes uniform in a 200^3 A box, 32 nearest neighbours
   per row (E = 2^25 exactly), Morton-ordered nodes, 16-dim N(0,1) features.
"""
from __future__ import annotations

import dataclasses
import math
from typing import Optional

import numpy as np
import torch


@dataclasses.dataclass
class GraphBatch:
    """A batch of graphs in dst-sorted edge order (host tensors)."""

    h: torch.Tensor            # (N, in_node_nf) float32 node features
    x: torch.Tensor            # (N, 3) float32 coordinates
    row: torch.Tensor          # (E,) int64 destination of each edge, non-decreasing
    col: torch.Tensor          # (E,) int64 source of each edge
    graph_ptr: torch.Tensor    # (G+1,) int64 node offsets of each graph
    target: torch.Tensor       # (G,) float32 regression target per graph
    name: str = ""

    @property
    def n_nodes(self) -> int:
        return int(self.h.shape[0])

    @property
    def n_edges(self) -> int:
        return int(self.row.shape[0])

    @property
    def n_graphs(self) -> int:
        return int(self.graph_ptr.shape[0] - 1)

    def graph_index(self) -> torch.Tensor:
        """(N,) int64 graph id of every node."""
        counts = self.graph_ptr[1:] - self.graph_ptr[:-1]
        return torch.repeat_interleave(torch.arange(self.n_graphs), counts)


@dataclasses.dataclass(frozen=True)
class ModelConfig:
    """Model settings of one workload (EGNN constructor arguments)."""

    in_node_nf: int
    hidden_nf: int
    out_node_nf: int
    n_layers: int
    precision: str          # 'fp32' or 'bf16' (bf16 GEMM inputs, fp32 accumulate)


CONFIGS = {
    1: ModelConfig(in_node_nf=5, hidden_nf=64, out_node_nf=1, n_layers=4, precision="fp32"),
    2: ModelConfig(in_node_nf=5, hidden_nf=128, out_node_nf=1, n_layers=7, precision="bf16"),
    3: ModelConfig(in_node_nf=20, hidden_nf=128, out_node_nf=1, n_layers=4, precision="fp32"),
    4: ModelConfig(in_node_nf=40, hidden_nf=256, out_node_nf=1, n_layers=6, precision="bf16"),
    5: ModelConfig(in_node_nf=16, hidden_nf=128, out_node_nf=1, n_layers=2, precision="bf16"),
}

GRAPHS_PER_BATCH = {1: 96, 2: 512, 3: 16, 4: 256, 5: 1}


# --------------------------------------------------------------------------
# helpers
# --------------------------------------------------------------------------

def fully_connected_edges(sizes, offsets):
    """All ordered pairs (i, j), i != j, inside each graph, row-major.

    Same pair order as ``get_edges``/``get_edges_batch``
    (egnn_clean.py:167-191): for each graph, for i, for j != i.
    """
    rows, cols = [], []
    for n, off in zip(sizes, offsets):
        n = int(n)
        ii = np.repeat(np.arange(n), n)
        jj = np.tile(np.arange(n), n)
        keep = ii != jj
        rows.append(ii[keep] + int(off))
        cols.append(jj[keep] + int(off))
    return np.concatenate(rows), np.concatenate(cols)


def _one_hot(types: np.ndarray, n_types: int) -> torch.Tensor:
    out = np.zeros((types.shape[0], n_types), dtype=np.float32)
    out[np.arange(types.shape[0]), types] = 1.0
    return torch.from_numpy(out)


def _radius_edges(pos: np.ndarray, cutoff: float, max_nbrs: Optional[int] = None):
    """Directed radius-graph edges (i, j), i != j, |x_i - x_j| < cutoff.

    Rows are sorted; inside a row the sources are ordered by distance then
    index when ``max_nbrs`` caps the row (nearest first), else by index.
    """
    from scipy.spatial import cKDTree

    tree = cKDTree(pos)
    n = pos.shape[0]
    rows, cols = [], []
    if max_nbrs is None:
        nbrs = tree.query_ball_point(pos, r=cutoff, return_sorted=True)
        for i, lst in enumerate(nbrs):
            lst = [j for j in lst if j != i]
            rows.append(np.full(len(lst), i, dtype=np.int64))
            cols.append(np.asarray(lst, dtype=np.int64))
    else:
        k = min(max_nbrs + 1, n)
        dist, idx = tree.query(pos, k=k)
        dist = np.atleast_2d(dist)
        idx = np.atleast_2d(idx)
        for i in range(n):
            sel = (idx[i] != i) & (dist[i] < cutoff) & (idx[i] < n)
            js = idx[i][sel][:max_nbrs]
            rows.append(np.full(js.shape[0], i, dtype=np.int64))
            cols.append(js.astype(np.int64))
    return np.concatenate(rows), np.concatenate(cols)


def _assemble(hs, xs, edge_lists, targets, name) -> GraphBatch:
    sizes = [int(x.shape[0]) for x in xs]
    offsets = np.concatenate([[0], np.cumsum(sizes)])
    rows = np.concatenate([r + offsets[g] for g, (r, _) in enumerate(edge_lists)])
    cols = np.concatenate([c + offsets[g] for g, (_, c) in enumerate(edge_lists)])
    return GraphBatch(
        h=torch.cat(hs).float().contiguous(),
        x=torch.from_numpy(np.concatenate(xs).astype(np.float32)),
        row=torch.from_numpy(rows.astype(np.int64)),
        col=torch.from_numpy(cols.astype(np.int64)),
        graph_ptr=torch.from_numpy(offsets.astype(np.int64)),
        target=targets.float(),
        name=name,
    )


# --------------------------------------------------------------------------
# workloads
# --------------------------------------------------------------------------

def molecules(n_graphs: int, seed: int = 0, n_min: int = 9, n_max: int = 29,
              n_types: int = 5, probs=(0.5, 0.3, 0.1, 0.05, 0.05),
              sigma: float = 1.5, name: str = "") -> GraphBatch:
    """Workloads 1-2: fully connected small molecules."""
    g = torch.Generator().manual_seed(seed)
    sizes = torch.randint(n_min, n_max + 1, (n_graphs,), generator=g).tolist()
    p = torch.tensor(probs, dtype=torch.float64)
    hs, xs, edges = [], [], []
    for n in sizes:
        types = torch.multinomial(p, n, replacement=True, generator=g)
        hs.append(torch.nn.functional.one_hot(types, n_types).float())
        x = torch.randn(n, 3, generator=g, dtype=torch.float64) * sigma
        x = x - x.mean(dim=0, keepdim=True)
        xs.append(x.numpy())
        r, c = fully_connected_edges([n], [0])
        edges.append((r, c))
    target = torch.randn(n_graphs, generator=g)
    return _assemble(hs, xs, edges, target, name or f"molecules{n_graphs}")


def _walk(n: int, rng: np.random.Generator, step: float = 3.8, min_sep: float = 3.0,
          tries: int = 10, jitter: float = 0.5) -> np.ndarray:
    """3-D self-avoiding-ish random walk: each step of length ``step`` in a
    uniformly random direction is redrawn up to ``tries`` times while it lands
    closer than ``min_sep`` to an earlier node; the last draw is kept."""
    pos = np.zeros((n, 3))
    for t in range(1, n):
        for _ in range(tries):
            v = rng.normal(size=3)
            v /= np.linalg.norm(v) + 1e-12
            cand = pos[t - 1] + step * v
            d2 = np.sum((pos[:t - 1] - cand) ** 2, axis=1) if t > 1 else np.zeros(0)
            if d2.size == 0 or d2.min() >= min_sep * min_sep:
                break
        pos[t] = cand
    return pos + rng.normal(scale=jitter, size=pos.shape)


def proteins(n_graphs: int = 16, seed: int = 0, n_min: int = 2000, n_max: int = 4000,
             cutoff: float = 10.0, n_types: int = 20, name: str = "") -> GraphBatch:
    """Workload 3: protein-sized walk graphs with a 10 A radius graph."""
    rng = np.random.default_rng(seed)
    sizes = rng.integers(n_min, n_max + 1, size=n_graphs)
    hs, xs, edges = [], [], []
    for n in sizes:
        pos = _walk(int(n), rng)
        types = rng.integers(0, n_types, size=int(n))
        hs.append(_one_hot(types, n_types))
        xs.append(pos)
        edges.append(_radius_edges(pos, cutoff))
    target = torch.from_numpy(rng.normal(size=n_graphs).astype(np.float32))
    return _assemble(hs, xs, edges, target, name or f"proteins{n_graphs}")


def _box_points(n: int, rng: np.random.Generator, box=(12.0, 12.0, 20.0),
                min_sep: float = 1.8, max_tries: int = 100000) -> np.ndarray:
    """Rejection-sample ``n`` points uniform in ``box`` with a minimum separation."""
    from scipy.spatial import cKDTree  # noqa: F401  (kept for symmetry with radius graphs)

    box = np.asarray(box)
    pts = np.empty((n, 3))
    k = 0
    tries = 0
    while k < n:
        cand = rng.uniform(size=3) * box
        tries += 1
        if tries > max_tries:
            raise RuntimeError("rejection sampling did not converge")
        if k == 0 or np.min(np.sum((pts[:k] - cand) ** 2, axis=1)) >= min_sep * min_sep:
            pts[k] = cand
            k += 1
    return pts


def _zipf_types(n: int, n_types: int, s: float, rng: np.random.Generator) -> np.ndarray:
    w = 1.0 / np.arange(1, n_types + 1) ** s
    return rng.choice(n_types, size=n, p=w / w.sum())


def slabs(n_graphs: int = 256, seed: int = 0, n_min: int = 50, n_max: int = 200,
          cutoff: float = 6.0, max_nbrs: int = 50, n_types: int = 40, zipf_s: float = 1.2,
          name: str = "") -> GraphBatch:
    """Workload 4: catalyst-slab-like boxes, radius 6 A capped at 50 nearest."""
    rng = np.random.default_rng(seed)
    sizes = rng.integers(n_min, n_max + 1, size=n_graphs)
    hs, xs, edges = [], [], []
    for n in sizes:
        pos = _box_points(int(n), rng)
        hs.append(_one_hot(_zipf_types(int(n), n_types, zipf_s, rng), n_types))
        xs.append(pos)
        edges.append(_radius_edges(pos, cutoff, max_nbrs=max_nbrs))
    target = torch.from_numpy(rng.normal(size=n_graphs).astype(np.float32))
    return _assemble(hs, xs, edges, target, name or f"slabs{n_graphs}")


def morton_codes(pos: np.ndarray, lo: np.ndarray, hi: np.ndarray, bits: int = 21) -> np.ndarray:
    """Interleaved 3 x ``bits``-bit Morton codes of coordinates quantised in [lo, hi)."""
    q = np.floor((pos - lo) / (hi - lo) * (1 << bits)).astype(np.int64)
    q = np.clip(q, 0, (1 << bits) - 1).astype(np.uint64)
    code = np.zeros(pos.shape[0], dtype=np.uint64)
    for b in range(bits):
        for a in range(3):
            code |= ((q[:, a] >> np.uint64(b)) & np.uint64(1)) << np.uint64(3 * b + a)
    return code


def point_cloud(n_nodes: int = 1 << 20, k: int = 32, seed: int = 0, box: float = 200.0,
                feat: int = 16, name: str = "") -> GraphBatch:
    """Workload 5: one giant kNN graph, Morton-ordered nodes, E = n_nodes * k."""
    from scipy.spatial import cKDTree

    rng = np.random.default_rng(seed)
    pos = rng.uniform(size=(n_nodes, 3)) * box
    order = np.argsort(morton_codes(pos, np.zeros(3), np.full(3, box)), kind="stable")
    pos = pos[order]
    tree = cKDTree(pos)
    _, idx = tree.query(pos, k=k + 1, workers=-1)
    # drop the self match; with continuous coordinates it is the nearest hit.
    nbr = np.empty((n_nodes, k), dtype=np.int64)
    self_first = idx[:, 0] == np.arange(n_nodes)
    nbr[self_first] = idx[self_first, 1:]
    if not self_first.all():
        for i in np.nonzero(~self_first)[0]:
            nbr[i] = [j for j in idx[i] if j != i][:k]
    row = np.repeat(np.arange(n_nodes, dtype=np.int64), k)
    col = nbr.reshape(-1)
    h = torch.from_numpy(rng.normal(size=(n_nodes, feat)).astype(np.float32))
    target = torch.from_numpy(rng.normal(size=1).astype(np.float32))
    return GraphBatch(h=h, x=torch.from_numpy(pos.astype(np.float32)),
                      row=torch.from_numpy(row), col=torch.from_numpy(col),
                      graph_ptr=torch.tensor([0, n_nodes], dtype=torch.int64),
                      target=target, name=name or f"pointcloud{n_nodes}")


def make_workload(cfg: int, seed: int = 0, n_graphs: Optional[int] = None,
                  n_nodes: Optional[int] = None) -> GraphBatch:
    """Batch for workload ``cfg`` (1..5); ``n_graphs``/``n_nodes`` shrink it."""
    if cfg in (1, 2):
        return molecules(n_graphs or GRAPHS_PER_BATCH[cfg], seed=seed, name=f"cfg{cfg}")
    if cfg == 3:
        return proteins(n_graphs or GRAPHS_PER_BATCH[3], seed=seed, name="cfg3")
    if cfg == 4:
        return slabs(n_graphs or GRAPHS_PER_BATCH[4], seed=seed, name="cfg4")
    if cfg == 5:
        return point_cloud(n_nodes or (1 << 20), seed=seed, name="cfg5")
    raise ValueError(f"unknown workload {cfg}")


def graph_loss_terms(batch: GraphBatch):
    """(graph index per node, targets) for the per-graph sum-MSE loss."""
    return batch.graph_index(), batch.target


def describe(batch: GraphBatch) -> dict:
    deg = torch.bincount(batch.row, minlength=batch.n_nodes)
    return {"graphs": batch.n_graphs, "nodes": batch.n_nodes, "edges": batch.n_edges,
            "deg_min": int(deg.min()), "deg_max": int(deg.max()),
            "deg_mean": round(float(deg.float().mean()), 2)}


__all__ = ["GraphBatch", "ModelConfig", "CONFIGS", "GRAPHS_PER_BATCH", "make_workload",
           "molecules", "proteins", "slabs", "point_cloud", "fully_connected_edges",
           "morton_codes", "describe", "graph_loss_terms"]
_ = math
