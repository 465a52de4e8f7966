"""Device graph builders against the CPU oracle (oracle/graph_oracle.py),
bit for bit: fully connected batches (and the reference's get_edges_batch),
radius graphs (uncapped and capped), k-nearest-neighbour graphs and Morton
order, on ragged batches, ties, duplicate points, dense clusters that need
several output passes, sparse outliers that force the exact fallback, and a
config-5-sized cloud checked on sampled rows plus whole-graph properties."""
import numpy as np
import pytest
import torch

from conftest import GOLDEN
from oracle import graph_oracle as GO
from pymolecular_b200 import builders
from pymolecular_b200 import _native as nat

pytestmark = pytest.mark.gpu


def _rows(csr):
    return csr.row_ptr.cpu().numpy().astype(np.int64), csr.col_idx.cpu().numpy().astype(np.int64)


def _check_csr(csr, rp, col):
    grp, gcol = _rows(csr)
    assert np.array_equal(grp, rp)
    assert np.array_equal(gcol, col)
    # row_idx, edge ids and the transpose are consistent with the rows
    N = len(rp) - 1
    assert np.array_equal(csr.row_idx.cpu().numpy(), np.repeat(np.arange(N), np.diff(rp)))
    assert np.array_equal(csr.edge_id.cpu().numpy(), np.arange(len(col)))
    csr.check()


def _ragged(seed, sizes, box):
    g = np.random.default_rng(seed)
    x = np.concatenate([g.uniform(0, box, size=(n, 3)) for n in sizes]).astype(np.float32)
    return x, np.concatenate([[0], np.cumsum(sizes)]).astype(np.int64)


def test_get_edges_batch_matches_reference(cuda_device):
    fx = torch.load(GOLDEN / "graphs" / "get_edges_batch.pt", weights_only=False)
    for (n, b), (rows, cols, attr) in fx["cases"].items():
        (r, c), a = builders.get_edges_batch(n, b, device=cuda_device)
        assert torch.equal(r.cpu(), rows) and torch.equal(c.cpu(), cols), (n, b)
        assert torch.equal(a.cpu(), attr)


@pytest.mark.parametrize("sizes", [[3, 0, 1, 3], [29] * 40, [1], [2, 2, 2], list(range(0, 30))])
def test_fc_graph_matches_oracle(sizes, cuda_device):
    gp = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int64)
    csr = builders.fc_graph(torch.from_numpy(gp), device=cuda_device)
    r, c = GO.fc_graph(gp)
    rp = np.concatenate([[0], np.cumsum(np.bincount(r, minlength=int(gp[-1])))]) if len(r) else np.zeros(int(gp[-1]) + 1, np.int64)
    _check_csr(csr, rp, c)


RADIUS_CASES = [
    # (name, sizes, box, cutoff, cap)
    ("one graph", [2000], 40.0, 5.0, None),
    ("ragged batch", [300, 1, 0, 150, 700], 15.0, 4.0, None),
    ("capped", [400, 250], 12.0, 6.0, 50),
    ("capped small", [60, 3], 8.0, 6.0, 5),
]


@pytest.mark.parametrize("name,sizes,box,cutoff,cap", RADIUS_CASES)
def test_radius_graph_matches_oracle(name, sizes, box, cutoff, cap, cuda_device):
    x, gp = _ragged(len(name), sizes, box)
    csr = builders.radius_graph(torch.from_numpy(x).to(cuda_device), cutoff, graph_ptr=torch.from_numpy(gp),
                                max_num_neighbors=cap)
    rp, col = GO.radius_graph(x, cutoff, gp, max_nbrs=cap)
    _check_csr(csr, rp, col)


def test_radius_graph_ties_duplicates_and_long_rows(cuda_device):
    # a lattice (many equal distances, pairs exactly at the cutoff), duplicated
    # points (d2 = 0), and a dense ball whose rows exceed one output pass
    lat = np.stack(np.meshgrid(*[np.arange(6)] * 3, indexing="ij"), -1).reshape(-1, 3).astype(np.float32) * 1.5
    dup = lat[:20].copy()
    g = np.random.default_rng(7)
    ball = (g.normal(size=(700, 3)) * 0.3 + 20.0).astype(np.float32)
    x = np.concatenate([lat, dup, ball])
    for cutoff, cap in [(1.5, None), (3.0, None), (3.0, 7), (2.5, 300), (50.0, None)]:
        csr = builders.radius_graph(torch.from_numpy(x).to(cuda_device), cutoff, max_num_neighbors=cap)
        rp, col = GO.radius_graph(x, cutoff, None, max_nbrs=cap)
        _check_csr(csr, rp, col)


@pytest.mark.parametrize("k,sizes,box", [(32, [3000], 30.0), (8, [200, 5, 1, 0, 90], 10.0), (16, [17, 16, 40], 3.0),
                                         (1, [50], 5.0), (256, [600], 8.0)])
def test_knn_graph_matches_oracle(k, sizes, box, cuda_device):
    x, gp = _ragged(k + len(sizes), sizes, box)
    csr = builders.knn_graph(torch.from_numpy(x).to(cuda_device), k, graph_ptr=torch.from_numpy(gp))
    rp, col = GO.knn_graph(x, k, gp)
    _check_csr(csr, rp, col)


def test_knn_graph_clusters_outliers_and_ties(cuda_device):
    # dense clusters, far outliers (need a larger cube or the whole-graph
    # fallback), a lattice (equal distances) and duplicates
    g = np.random.default_rng(11)
    clusters = np.concatenate([g.normal(size=(400, 3)) * 0.2 + c for c in ([0, 0, 0], [30, 0, 0], [0, 40, 5])])
    outliers = g.uniform(-300, 300, size=(12, 3))
    lat = np.stack(np.meshgrid(*[np.arange(5)] * 3, indexing="ij"), -1).reshape(-1, 3) * 2.0 + 100.0
    x = np.concatenate([clusters, outliers, lat, lat[:10]]).astype(np.float32)
    for k in (6, 24):
        csr = builders.knn_graph(torch.from_numpy(x).to(cuda_device), k)
        rp, col = GO.knn_graph(x, k)
        _check_csr(csr, rp, col)
    assert nat.lib().egnn_device_status(nat.stream_ptr()) == nat.EGNN_OK


def test_knn_config5_scale_sampled_rows(cuda_device):
    """1M uniform points, k = 32 (workload 5): every row has 32 distinct
    non-self sources in non-decreasing distance; 1000 sampled rows equal the
    brute-force oracle exactly."""
    n, k = 1 << 20, 32
    g = np.random.default_rng(0)
    x = (g.uniform(size=(n, 3)) * 200.0).astype(np.float32)
    xd = torch.from_numpy(x).to(cuda_device)
    csr = builders.knn_graph(xd, k)
    rp, col = _rows(csr)
    assert np.array_equal(rp, np.arange(n + 1) * k)
    nb = col.reshape(n, k)
    assert not (nb == np.arange(n)[:, None]).any()
    srt = np.sort(nb, axis=1)
    assert not (srt[:, 1:] == srt[:, :-1]).any()
    d = ((x[nb] - x[:, None, :]) ** 2).sum(-1)
    assert (np.diff(d, axis=1) >= -1e-5).all()
    for i in g.choice(n, size=1000, replace=False):
        assert np.array_equal(nb[i], GO.knn_row(x, i, k, 0, n)), i


def test_morton_order_matches_oracle(cuda_device):
    g = np.random.default_rng(5)
    x = (g.uniform(-5, 205, size=(200_000, 3))).astype(np.float32)   # some outside [lo, hi): clipped
    x[:100] = x[100:200]                                             # equal codes: stable order
    codes, perm = builders.morton_order(torch.from_numpy(x).to(cuda_device), [0, 0, 0], [200, 200, 200])
    rc, rperm = GO.morton_order(x, [0, 0, 0], [200, 200, 200])
    assert np.array_equal(codes.cpu().numpy().astype(np.uint64), rc)
    assert np.array_equal(perm.cpu().numpy(), rperm)


def test_builder_guards(cuda_device):
    x = torch.zeros(10, 3, device=cuda_device)
    with pytest.raises(nat.EgnnError):
        builders.knn_graph(x, 300)                 # k above the built maximum
    with pytest.raises(nat.EgnnError) as ei:
        builders.radius_graph(x, 1.0, graph_ptr=torch.tensor([0, 6, 4, 10]))
    assert ei.value.status == nat.EGNN_ERR_INDEX
    with pytest.raises(ValueError):
        builders.radius_graph(x, 0.0)
    with pytest.raises(ValueError):
        builders.fc_graph(torch.tensor([0, 5, 3]), device=cuda_device)
    with pytest.raises(ValueError):
        builders.knn_graph(torch.zeros(10, 3), 4)  # CPU tensors are rejected
    # empty inputs
    e = builders.radius_graph(torch.zeros(0, 3, device=cuda_device), 1.0)
    assert e.n_nodes == 0 and e.n_edges == 0



def _same_up_to_float32_boundary(csr, b, cutoff, capped):
    """Per-row neighbour sets of a device CSR against a generator batch: any
    difference must sit on the cutoff (uncapped) or on the cap's k-th distance
    (capped) to float32 precision.  Returns the number of rows that differ."""
    rp, col = _rows(csr)
    hrp = np.concatenate([[0], np.cumsum(np.bincount(b.row.numpy(), minlength=b.n_nodes))])
    hcol = b.col.numpy()
    x = b.x.numpy()
    c2 = np.float32(cutoff) * np.float32(cutoff)
    differ = 0
    for i in range(b.n_nodes):
        a, h = col[rp[i]:rp[i + 1]], hcol[hrp[i]:hrp[i + 1]]
        if np.array_equal(a, h):
            continue
        sa, sh = set(a.tolist()), set(h.tolist())
        d = GO.sqdist_f32(x[i], x[sorted(sa ^ sh)]) if sa != sh else np.zeros(0, np.float32)
        if capped:
            ref = np.sort(GO.sqdist_f32(x[i], x[a]))[-1] if len(a) else c2
            assert np.allclose(d, ref, rtol=1e-5), i
            # nearest first in both: position by position the distances agree, so
            # only neighbours at equal float32 distances can trade places
            if len(a) == len(h):
                assert np.allclose(GO.sqdist_f32(x[i], x[a]), GO.sqdist_f32(x[i], x[h]), rtol=1e-5), i
        else:
            assert sa != sh and np.allclose(d, c2, rtol=1e-5), i
        differ += 1
    return differ


def test_builders_reproduce_the_workload_graphs(cuda_device):
    """The device builders give the graphs of the workload generators (scipy
    cKDTree in float64) up to float32 ties at the cutoff or the cap: protein
    walks with a 10 A radius graph (workload 3), slabs with a 6 A radius graph
    capped at 50 nearest (workload 4), and the fully connected molecule batch
    (workloads 1-2) edge for edge."""
    from pymolecular_b200 import datasets
    b3 = datasets.proteins(2, seed=3)
    csr3 = builders.radius_graph(b3.x.to(cuda_device), 10.0, graph_ptr=b3.graph_ptr)
    assert _same_up_to_float32_boundary(csr3, b3, 10.0, False) <= b3.n_nodes // 1000
    b4 = datasets.slabs(16, seed=4)
    csr4 = builders.radius_graph(b4.x.to(cuda_device), 6.0, graph_ptr=b4.graph_ptr, max_num_neighbors=50)
    assert _same_up_to_float32_boundary(csr4, b4, 6.0, True) <= b4.n_nodes // 100
    b2 = datasets.molecules(64, seed=2)
    csr2 = builders.fc_graph(b2.graph_ptr, device=cuda_device)
    assert torch.equal(csr2.row_idx.cpu().long(), b2.row) and torch.equal(csr2.col_idx.cpu().long(), b2.col)
