"""The CPU oracle against the golden fixtures made by the reference itself."""
import os
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from conftest import golden_cases, load_golden, rel_err
from oracle import egnn_oracle as O
from oracle import csr_oracle as CO

# The reference's models/EGNN directory (EGNN_REFERENCE_DIR); the checks that
# import the reference module itself are skipped when it is not given.
REF = Path(os.environ["EGNN_REFERENCE_DIR"]) if os.environ.get("EGNN_REFERENCE_DIR") else None


def _flags(case):
    f = dict(case.get("flags", {}))
    return f


@pytest.mark.parametrize("name", golden_cases())
def test_oracle_matches_golden(name):
    c = load_golden(name)
    p = {k: v.double() for k, v in c["state_dict"].items()}
    if c["kind"] in ("model", "demo"):
        h = c["h"].clone().requires_grad_(True)
        x = c["x"].clone().requires_grad_(True)
        leaf = {k: v.clone().requires_grad_(True) for k, v in p.items()}
        ho, xo = O.egnn(leaf, h, x, c["row"], c["col"], c.get("edge_attr"), **_flags(c))
        if c["kind"] == "model":
            gi = torch.repeat_interleave(torch.arange(len(c["graph_ptr"]) - 1),
                                         c["graph_ptr"][1:] - c["graph_ptr"][:-1])
            loss = O.graph_sum_mse(ho, gi, c["target"])
        else:
            loss = (ho ** 2).sum() + (xo * torch.linspace(-1, 1, 96, dtype=torch.float64).view(32, 3)).sum()
        loss.backward()
        assert rel_err(loss, c["loss"]) < 1e-12
        grads = {k: (v.grad if v.grad is not None else torch.zeros_like(v)) for k, v in leaf.items()}
        gh, gx = h.grad, x.grad
    else:
        ho, xo, gh, gx, grads = O.layer_grads(p, "", c["h"], c["row"], c["col"], c["x"], c["gh"], c["gx"],
                                              c.get("edge_attr"), **_flags(c))
        grads = {k: (v if v is not None else torch.zeros_like(p[k])) for k, v in grads.items()}
    assert rel_err(ho, c["h_out"]) < 1e-12
    assert rel_err(xo, c["x_out"]) < 1e-12
    assert rel_err(gh, c["grad_h"]) < 1e-12
    assert rel_err(gx, c["grad_x"]) < 1e-12
    assert set(grads) == set(c["grads"])
    for k in grads:
        assert rel_err(grads[k], c["grads"][k]) < 1e-12, k


@pytest.mark.skipif(REF is None or not REF.exists(), reason="EGNN_REFERENCE_DIR not set")
def test_oracle_matches_live_reference():
    sys.path.insert(0, str(REF))
    import egnn_clean
    from pymolecular_b200.datasets import molecules
    b = molecules(7, seed=11)
    torch.manual_seed(5)
    ref = egnn_clean.EGNN(5, 32, 1, n_layers=3, normalize=True, tanh=True).double()
    p = {k: v.detach() for k, v in ref.state_dict().items()}
    h1, x1 = ref(b.h.double(), b.x.double(), [b.row, b.col], None)
    h2, x2 = O.egnn(p, b.h.double(), b.x.double(), b.row, b.col, normalize=True, tanh=True)
    assert rel_err(h2, h1) < 1e-13 and rel_err(x2, x1) < 1e-13


def test_init_params_shapes_match_golden():
    c = load_golden("model_molecules")
    p = O.init_params(5, 32, 1, 2)
    assert {k: tuple(v.shape) for k, v in p.items()} == {k: tuple(v.shape) for k, v in c["state_dict"].items()}


def test_csr_oracle_matches_stable_sort():
    g = torch.Generator().manual_seed(0)
    N, E = 97, 1000
    row = torch.randint(0, N, (E,), generator=g)
    col = torch.randint(0, N, (E,), generator=g)
    row_ptr, col_idx, row_idx, edge_id = CO.csr_build(row.numpy(), col.numpy(), N)
    srt, perm = torch.sort(row, stable=True)
    assert np.array_equal(edge_id, perm.numpy())
    assert np.array_equal(row_idx, srt.numpy())
    assert np.array_equal(col_idx, col[perm].numpy())
    assert np.array_equal(row_ptr[1:] - row_ptr[:-1], torch.bincount(row, minlength=N).numpy())
    src_ptr, src_edge = CO.csr_transpose(col_idx, N)
    # every CSR position appears once, grouped by source, increasing within a group
    assert np.array_equal(np.sort(src_edge), np.arange(E))
    for j in range(N):
        seg = src_edge[src_ptr[j]:src_ptr[j + 1]]
        assert np.all(col_idx[seg] == j) and np.all(np.diff(seg) > 0)
    assert CO.csr_valid(row_ptr, col_idx, N)
    bad = row_ptr.copy()
    bad[5], bad[6] = bad[6], bad[5] - 1
    assert not CO.csr_valid(bad, col_idx, N)


def test_csr_oracle_rejects_out_of_range():
    with pytest.raises(IndexError):
        CO.csr_build([0, 1, 5], [1, 2, 0], 5)


def test_fp32_oracle_within_layer_tolerance():
    """The 1e-5 fp32 bar is reachable: the fp32 oracle itself sits well inside it."""
    c = load_golden("layer_default_h64")
    p64 = {k: v.double() for k, v in c["state_dict"].items()}
    p32 = {k: v.float() for k, v in p64.items()}
    r64 = O.layer_grads(p64, "", c["h"], c["row"], c["col"], c["x"], c["gh"], c["gx"])
    r32 = O.layer_grads(p32, "", c["h"].float(), c["row"], c["col"], c["x"].float(), c["gh"].float(),
                        c["gx"].float())
    for a, b in zip(r32[:4], r64[:4]):
        assert rel_err(a, b) < 1e-5
    for k in r64[4]:
        assert rel_err(r32[4][k], r64[4][k]) < 1e-5, k


@pytest.mark.parametrize("name", ["layer_default_h64", "layer_flags_h32", "layer_noresidual_h32",
                                  "layer_attention_h64", "layer_attention_flags_h32"])
def test_emulation_backward_matches_autograd(name):
    """The rounding-exact model's hand-derived backward (the same algebra as the
    kernels, attention gate included) equals the reference's autograd when
    nothing is rounded."""
    from oracle import egnn_emulation as EM
    c = load_golden(name)
    p = {k: v.double() for k, v in c["state_dict"].items()}
    got = EM.layer_fwd_bwd(p, c["h"], c["row"], c["col"], c["x"], c["gh"], c["gx"], c.get("edge_attr"),
                           precision="fp32", **_flags(c))
    for a, b in zip(got[:4], (c["h_out"], c["x_out"], c["grad_h"], c["grad_x"])):
        assert rel_err(a, b) < 1e-12
    assert set(got[4]) == set(c["grads"])
    for k, v in got[4].items():
        assert rel_err(v, c["grads"][k]) < 1e-12, k
