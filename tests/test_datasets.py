"""Seeded workload generators: shapes, ordering and the graph rules of each config."""
import numpy as np
import torch

from pymolecular_b200.datasets import (CONFIGS, make_workload, molecules, morton_codes, point_cloud,
                                       proteins, slabs)


def _dst_sorted(b):
    return bool(torch.all(b.row[1:] >= b.row[:-1]))


def test_config1_is_the_surveyed_draw():
    b = make_workload(1)
    assert (b.n_graphs, b.n_nodes, b.n_edges) == (96, 1835, 36418)
    assert _dst_sorted(b)
    assert torch.all(b.row != b.col)
    sizes = (b.graph_ptr[1:] - b.graph_ptr[:-1])
    assert int(sizes.min()) >= 9 and int(sizes.max()) <= 29
    assert int((sizes * (sizes - 1)).sum()) == b.n_edges
    # one-hot features, centred coordinates
    assert torch.all(b.h.sum(1) == 1)
    for g in range(b.n_graphs):
        xs = b.x[b.graph_ptr[g]:b.graph_ptr[g + 1]]
        assert xs.mean(0).abs().max() < 1e-5


def test_molecules_are_reproducible_and_seeded():
    a, b, c = molecules(8, seed=3), molecules(8, seed=3), molecules(8, seed=4)
    assert torch.equal(a.x, b.x) and torch.equal(a.row, b.row)
    assert not torch.equal(a.x, c.x)


def test_fully_connected_order_matches_get_edges():
    # get_edges (egnn_clean.py:167-176): for i, for j != i
    b = molecules(1, seed=0, n_min=4, n_max=4)
    expect = [(i, j) for i in range(4) for j in range(4) if i != j]
    assert list(zip(b.row.tolist(), b.col.tolist())) == expect


def test_proteins_radius_graph():
    b = proteins(n_graphs=1, seed=0, n_min=300, n_max=300)
    assert _dst_sorted(b) and torch.all(b.row != b.col)
    d = (b.x[b.row] - b.x[b.col]).norm(dim=1)
    assert float(d.max()) < 10.0
    # symmetric radius graph
    fwd = set(zip(b.row.tolist(), b.col.tolist()))
    assert all((j, i) in fwd for i, j in fwd)
    assert b.h.shape[1] == 20


def test_slabs_capped_knn_radius():
    b = slabs(n_graphs=2, seed=0, n_min=150, n_max=200)
    assert _dst_sorted(b)
    deg = torch.bincount(b.row, minlength=b.n_nodes)
    assert int(deg.max()) <= 50
    d = (b.x[b.row] - b.x[b.col]).norm(dim=1)
    assert float(d.max()) < 6.0
    for g in range(2):
        xs = b.x[b.graph_ptr[g]:b.graph_ptr[g + 1]].double()
        dm = torch.cdist(xs, xs) + torch.eye(xs.shape[0], dtype=torch.float64) * 100
        assert float(dm.min()) >= 1.8 - 1e-4
    assert b.h.shape[1] == 40


def test_point_cloud_knn_and_morton_order():
    b = point_cloud(n_nodes=4096, k=32, seed=0, box=50.0)
    assert b.n_edges == 4096 * 32
    assert _dst_sorted(b) and torch.all(b.row != b.col)
    codes = morton_codes(b.x.double().numpy(), np.zeros(3), np.full(3, 50.0))
    assert np.all(np.diff(codes.astype(np.int64)) >= 0) or np.mean(np.diff(codes.astype(np.float64)) >= 0) > 0.99


def test_config_table():
    assert CONFIGS[2].hidden_nf == 128 and CONFIGS[2].n_layers == 7 and CONFIGS[2].precision == "bf16"
    assert CONFIGS[4].hidden_nf == 256 and CONFIGS[5].n_layers == 2
