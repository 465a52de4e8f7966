"""Generates the golden fixtures in this directory from the REFERENCE itself.

    python tests/golden/make_golden.py /path/to/PyMolecular [case ...]

Imports ``models/EGNN/egnn_clean.py`` from the reference checkout, runs its
``EGNN`` / ``E_GCL`` in float64 on seeded inputs, backpropagates a seeded
loss and stores inputs, weights (state_dict), outputs and every gradient as
``<case>.pt``.  The reference is not needed afterwards: the tests compare the
in-repo oracle (oracle/egnn_oracle.py) and the CUDA path against these files.
"""
from __future__ import annotations

import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from pymolecular_b200.datasets import molecules  # noqa: E402


def load_reference(root: Path):
    sys.path.insert(0, str(root / "models" / "EGNN"))
    import egnn_clean  # noqa: E402
    return egnn_clean


def _grads(module):
    return {k: (v.grad.detach().clone() if v.grad is not None else torch.zeros_like(v))
            for k, v in module.named_parameters()}


def case_model(ref, name, seed, n_graphs, n_min, n_max, hidden, layers, **flags):
    """Whole EGNN: embedding_in, L x E_GCL, embedding_out; graph-sum MSE loss."""
    b = molecules(n_graphs, seed=seed, n_min=n_min, n_max=n_max)
    torch.manual_seed(seed)
    model = ref.EGNN(in_node_nf=5, hidden_nf=hidden, out_node_nf=1, n_layers=layers, **flags).double()
    h0, x0 = b.h.double(), b.x.double().requires_grad_(True)
    h0.requires_grad_(True)
    ho, xo = model(h0, x0, [b.row, b.col], None)
    gi = b.graph_index()
    pred = torch.zeros(b.n_graphs, dtype=torch.float64).index_add_(0, gi, ho[:, 0])
    loss = ((pred - b.target.double()) ** 2).mean()
    loss.backward()
    return dict(kind="model", hidden=hidden, n_layers=layers, in_node_nf=5, out_node_nf=1, flags=flags,
                h=b.h.double(), x=b.x.double(), row=b.row, col=b.col, graph_ptr=b.graph_ptr,
                target=b.target.double(), state_dict={k: v.clone() for k, v in model.state_dict().items()},
                h_out=ho.detach(), x_out=xo.detach(), loss=loss.detach(), grads=_grads(model),
                grad_h=h0.grad.clone(), grad_x=x0.grad.clone())


def _random_graph(g, n, n_edges, hub=None, isolated=(), self_loop=True, duplicate=True):
    row = torch.randint(0, n, (n_edges,), generator=g)
    col = torch.randint(0, n, (n_edges,), generator=g)
    if hub is not None:   # a high in-degree row
        k = n_edges // 4
        row[:k] = hub
    for v in isolated:    # rows/cols that never appear
        keep = (row != v) & (col != v)
        row, col = row[keep], col[keep]
    if self_loop:
        row = torch.cat([row, torch.tensor([1])])
        col = torch.cat([col, torch.tensor([1])])
    if duplicate:
        row = torch.cat([row, row[2:3], row[2:3]])
        col = torch.cat([col, col[2:3], col[2:3]])
    return row.long(), col.long()


def case_layer(ref, name, seed, n, n_edges, hidden, edges_in_d=0, input_nf=None, output_nf=None, **flags):
    """One E_GCL with random upstream gradients on an unsorted, ragged graph
    (input_nf / output_nf default to hidden, as inside EGNN)."""
    input_nf = hidden if input_nf is None else input_nf
    output_nf = hidden if output_nf is None else output_nf
    g = torch.Generator().manual_seed(seed)
    row, col = _random_graph(g, n, n_edges, hub=3, isolated=(n - 1, n - 2))
    E = row.numel()
    torch.manual_seed(seed)
    layer = ref.E_GCL(input_nf, output_nf, hidden, edges_in_d=edges_in_d, **flags).double()
    h = torch.randn(n, input_nf, generator=g, dtype=torch.float64).requires_grad_(True)
    x = (torch.randn(n, 3, generator=g, dtype=torch.float64) * 1.5).requires_grad_(True)
    ea = torch.randn(E, edges_in_d, generator=g, dtype=torch.float64) if edges_in_d else None
    gh = torch.randn(n, output_nf, generator=g, dtype=torch.float64)
    gx = torch.randn(n, 3, generator=g, dtype=torch.float64)
    ho, xo, _ = layer(h, [row, col], x, edge_attr=ea)
    torch.autograd.backward([ho, xo], [gh, gx])
    return dict(kind="layer", hidden=hidden, input_nf=input_nf, output_nf=output_nf,
                edges_in_d=edges_in_d, flags=flags,
                h=h.detach(), x=x.detach(), row=row, col=col, edge_attr=ea, gh=gh, gx=gx,
                state_dict={k: v.clone() for k, v in layer.state_dict().items()},
                h_out=ho.detach(), x_out=xo.detach(), grads=_grads(layer),
                grad_h=h.grad.clone(), grad_x=x.grad.clone())


def case_reference_demo(ref):
    """The reference's own __main__ (egnn_clean.py:194-210): 8 x 4 nodes, in_edge_nf=1."""
    torch.manual_seed(0)
    edges, edge_attr = ref.get_edges_batch(4, 8)
    h = torch.ones(32, 1, dtype=torch.float64).requires_grad_(True)
    x = torch.ones(32, 3, dtype=torch.float64)
    x = (x + 0.1 * torch.randn(32, 3, dtype=torch.float64)).requires_grad_(True)
    model = ref.EGNN(in_node_nf=1, hidden_nf=32, out_node_nf=1, in_edge_nf=1).double()
    ho, xo = model(h, x, edges, edge_attr.double())
    loss = (ho ** 2).sum() + (xo * torch.linspace(-1, 1, 96, dtype=torch.float64).view(32, 3)).sum()
    loss.backward()
    return dict(kind="demo", hidden=32, n_layers=4, in_node_nf=1, out_node_nf=1, in_edge_nf=1,
                h=h.detach(), x=x.detach(), row=edges[0], col=edges[1], edge_attr=edge_attr.double(),
                state_dict={k: v.clone() for k, v in model.state_dict().items()},
                h_out=ho.detach(), x_out=xo.detach(), loss=loss.detach(), grads=_grads(model),
                grad_h=h.grad.clone(), grad_x=x.grad.clone())


CASES = {
    "model_molecules": lambda r: case_model(r, "model_molecules", 1, 5, 3, 7, 32, 2),
    "layer_default_h64": lambda r: case_layer(r, "layer_default_h64", 2, 48, 200, 64),
    "layer_flags_h32": lambda r: case_layer(r, "layer_flags_h32", 3, 40, 150, 32, edges_in_d=2,
                                            normalize=True, tanh=True, coords_agg="sum"),
    "layer_noresidual_h32": lambda r: case_layer(r, "layer_noresidual_h32", 4, 30, 90, 32,
                                                 residual=False),
    "reference_demo": case_reference_demo,
    "layer_attention_h64": lambda r: case_layer(r, "layer_attention_h64", 5, 48, 200, 64, attention=True),
    "layer_attention_flags_h32": lambda r: case_layer(r, "layer_attention_flags_h32", 6, 40, 150, 32,
                                                      edges_in_d=3, attention=True, normalize=True,
                                                      tanh=True, coords_agg="sum"),
    "model_attention_molecules": lambda r: case_model(r, "model_attention_molecules", 7, 5, 3, 7, 32, 2,
                                                      attention=True),
    # E_GCL with input_nf / output_nf other than hidden_nf (egnn_clean.py:11-31)
    "layer_dims_i16_o8_h32": lambda r: case_layer(r, "layer_dims_i16_o8_h32", 8, 40, 160, 32, edges_in_d=2,
                                                  input_nf=16, output_nf=8, residual=False),
    "layer_dims_i12_h64": lambda r: case_layer(r, "layer_dims_i12_h64", 9, 48, 200, 64, input_nf=12,
                                               output_nf=12, attention=True),
}


def case_get_edges_batch(ref):
    """The reference's fully connected batch edges (egnn_clean.py:167-191)."""
    out = {}
    for n, b in [(4, 8), (5, 3), (9, 1), (1, 3), (2, 5), (29, 4)]:
        edges, attr = ref.get_edges_batch(n, b)
        out[(n, b)] = (edges[0].clone(), edges[1].clone(), attr.clone())
    return dict(kind="graphs", cases=out)


# graph-construction fixtures live in golden/graphs/ (not layer or model cases)
GRAPH_CASES = {"get_edges_batch": case_get_edges_batch}


def main():
    root = Path(sys.argv[1]) if len(sys.argv) > 1 else None
    if root is None or not (root / "models" / "EGNN" / "egnn_clean.py").exists():
        raise SystemExit("usage: make_golden.py <reference checkout>")
    ref = load_reference(root)
    names = sys.argv[2:] or list(CASES) + list(GRAPH_CASES)   # optionally only the named cases
    for name in names:
        if name in GRAPH_CASES:
            (HERE / "graphs").mkdir(exist_ok=True)
            torch.save(GRAPH_CASES[name](ref), HERE / "graphs" / f"{name}.pt")
            print(name)
            continue
        fn = CASES[name]
        data = fn(ref)
        data["name"] = name
        torch.save(data, HERE / f"{name}.pt")
        print(name, {k: tuple(v.shape) for k, v in data.items() if torch.is_tensor(v)})


if __name__ == "__main__":
    main()
