"""The CPU oracle of the graph builders, pinned to the reference's own
get_edges_batch (golden fixture) and to scipy's cKDTree, which the workload
generators use."""
import numpy as np
import pytest
import torch

from conftest import GOLDEN
from oracle import graph_oracle as GO
from pymolecular_b200 import datasets


def test_fc_graph_matches_reference_get_edges_batch():
    fx = torch.load(GOLDEN / "graphs" / "get_edges_batch.pt", weights_only=False)
    assert fx["cases"]
    for (n, b), (rows, cols, attr) in fx["cases"].items():
        r, c = GO.fc_graph(np.arange(b + 1) * n)
        assert np.array_equal(r, rows.numpy()), (n, b)
        assert np.array_equal(c, cols.numpy()), (n, b)
        assert attr.shape == (rows.numel(), 1)


def test_fc_graph_ragged():
    r, c = GO.fc_graph([0, 3, 3, 4, 7])
    # graph sizes 3, 0, 1, 3: rows 0-2 and 4-6 fully connected, node 3 isolated
    exp = [(i, j) for g in ([0, 1, 2], [4, 5, 6]) for i in g for j in g if i != j]
    assert list(zip(r.tolist(), c.tolist())) == exp


def _ragged_points(seed, sizes, box=12.0):
    g = np.random.default_rng(seed)
    xs = [g.uniform(0, box, size=(n, 3)).astype(np.float32) for n in sizes]
    gp = np.concatenate([[0], np.cumsum(sizes)])
    return np.concatenate(xs), gp


def _kdtree_rows(x, gp, fn):
    rows = []
    for g in range(len(gp) - 1):
        a, b = int(gp[g]), int(gp[g + 1])
        r, c = fn(x[a:b].astype(np.float64))
        for i in range(b - a):
            rows.append(c[r == i] + a)
    return rows


def _csr_rows(row_ptr, col):
    return [col[row_ptr[i]:row_ptr[i + 1]] for i in range(len(row_ptr) - 1)]


@pytest.mark.parametrize("cap", [None, 12])
def test_radius_oracle_matches_kdtree(cap):
    x, gp = _ragged_points(1, [150, 1, 90, 200], box=10.0)
    rp, col = GO.radius_graph(x, 3.0, gp, max_nbrs=cap)
    got = _csr_rows(rp, col)
    ref = _kdtree_rows(x, gp, lambda p: datasets._radius_edges(p, 3.0, max_nbrs=cap))
    assert len(got) == len(ref)
    for i, (a, b) in enumerate(zip(got, ref)):
        assert np.array_equal(a, b), i


def test_knn_oracle_matches_kdtree():
    from scipy.spatial import cKDTree
    x, gp = _ragged_points(2, [300, 5, 120], box=20.0)
    k = 8
    rp, col = GO.knn_graph(x, k, gp)
    got = _csr_rows(rp, col)
    for g in range(len(gp) - 1):
        a, b = int(gp[g]), int(gp[g + 1])
        kk = min(k + 1, b - a)
        _, idx = cKDTree(x[a:b].astype(np.float64)).query(x[a:b].astype(np.float64), k=kk)
        idx = np.atleast_2d(idx).reshape(b - a, -1)
        for i in range(b - a):
            exp = [j + a for j in idx[i] if j != i][:k]
            assert np.array_equal(got[a + i], exp), (g, i)


def test_morton_oracle_matches_dataset_codes():
    g = np.random.default_rng(3)
    x = (g.uniform(size=(5000, 3)) * 200.0).astype(np.float32)
    code, perm = GO.morton_order(x, [0, 0, 0], [200, 200, 200])
    ref = datasets.morton_codes(x.astype(np.float64), np.zeros(3), np.full(3, 200.0))
    assert np.array_equal(code, ref)
    assert np.array_equal(perm, np.argsort(ref, kind="stable"))


def test_distance_spec_is_per_operation_float32():
    a = np.array([1.1, -2.3, 7.7], dtype=np.float32)
    b = np.array([[0.3, 4.4, -1.9]], dtype=np.float32)
    d = a - b[0]
    exp = np.float32(np.float32(np.float32(d[0] * d[0]) + np.float32(d[1] * d[1])) + np.float32(d[2] * d[2]))
    assert GO.sqdist_f32(a, b)[0] == exp
