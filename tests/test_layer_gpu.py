"""Parity of the CUDA layer (through the C ABI) with the CPU oracle.

Error = max |y - y_ref| / max |y_ref| per tensor, against the fp64 oracle,
on h, x, dL/dh, dL/dx and every parameter gradient.
  fp32 mode: <= max(1e-5, 3 x the error of the reference algorithm run in
    fp32 on the same inputs).  Where the reference's own fp32 result is
    further than 1e-5 from fp64 (ill-conditioned gradients), no fp32
    implementation can promise 1e-5.
  bf16-GEMM mode: <= 2e-2 (flat), and within 5e-3 of the rounding-exact
    bf16 model (oracle/egnn_emulation.py) on every tensor that model computes
    to better than 5e-3 itself.
CSR construction is compared bit for bit.
"""
import numpy as np
import pytest
import torch

from conftest import as_dict, check_bf16, check_tensors, golden_cases, load_golden, rel_err, tolerances
from oracle import csr_oracle as CO
from oracle import egnn_emulation as EM
from oracle import egnn_oracle as O
from pymolecular_b200 import CSR, EGNN, E_GCL
from pymolecular_b200 import _native as nat

pytestmark = pytest.mark.gpu

TOL = {"fp32": 1e-5, "bf16": 2e-2}


def _layer_from_state(sd, hidden, precision, dev, edges_in_d=0, input_nf=None, output_nf=None, **flags):
    layer = E_GCL(input_nf or hidden, output_nf or hidden, hidden, edges_in_d=edges_in_d, precision=precision,
                  **flags).to(dev)
    layer.load_state_dict({k: v.float() for k, v in sd.items()})
    return layer


def _run_layer(layer, h, x, csr, gh, gx, edge_attr=None):
    h = h.clone().requires_grad_(True)
    x = x.clone().requires_grad_(True)
    ho, xo, _ = layer(h, csr, x, edge_attr=edge_attr)
    torch.autograd.backward([ho, xo], [gh, gx])
    grads = {k: v.grad.clone() for k, v in layer.named_parameters()}
    for v in layer.parameters():
        v.grad = None
    return ho.detach(), xo.detach(), h.grad, x.grad, grads


def _fp32_tol(p, h, row, col, x, gh, gx, ea, ref, flags):
    """Per-tensor fp32 bar: max(1e-5, 3 x the fp32 reference's own error)."""
    p32 = {k: v.float() for k, v in p.items()}
    r32 = O.layer_grads(p32, "", h.float(), row, col, x.float(), gh.float(), gx.float(),
                        ea.float() if ea is not None else None, **flags)
    return tolerances(as_dict(ref), as_dict(r32), 1e-5, 3.0)


# ---------------------------------------------------------------------------
# golden fixtures (reference outputs, fp64)
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("name", golden_cases())
def test_golden_fixture_fp32(name, cuda_device):
    c = load_golden(name)
    dev = cuda_device
    if c["kind"] == "layer":
        flags = dict(c.get("flags", {}))
        layer = _layer_from_state(c["state_dict"], c["hidden"], "fp32", dev, c["edges_in_d"],
                                  c.get("input_nf"), c.get("output_nf"), **flags)
        csr = CSR.from_edges(c["row"], c["col"], n_nodes=c["h"].shape[0], device=dev)
        ea = c["edge_attr"].float().to(dev) if c["edge_attr"] is not None else None
        res = _run_layer(layer, c["h"].float().to(dev), c["x"].float().to(dev), csr,
                         c["gh"].float().to(dev), c["gx"].float().to(dev), ea)
        ref = (c["h_out"], c["x_out"], c["grad_h"], c["grad_x"], c["grads"])
        tol = _fp32_tol(c["state_dict"], c["h"], c["row"], c["col"], c["x"], c["gh"], c["gx"],
                        c["edge_attr"], ref, flags)
        check_tensors(as_dict(res), as_dict(ref), tol, name)
        return
    flags = dict(c.get("flags", {}))
    model = EGNN(c["in_node_nf"], c["hidden"], c["out_node_nf"], in_edge_nf=c.get("in_edge_nf", 0),
                 n_layers=c["n_layers"], device=dev, **flags)
    model.load_state_dict({k: v.float() for k, v in c["state_dict"].items()})
    h = c["h"].float().to(dev).requires_grad_(True)
    x = c["x"].float().to(dev).requires_grad_(True)
    ea = c["edge_attr"].float().to(dev) if c.get("edge_attr") is not None else None
    ho, xo = model(h, x, [c["row"].to(dev), c["col"].to(dev)], ea)
    loss = _golden_loss(c, ho, xo)
    loss.backward()
    got = {"loss": loss, "h": ho, "x": xo, "dh": h.grad, "dx": x.grad}
    got.update({k: (v.grad if v.grad is not None else torch.zeros_like(v)) for k, v in model.named_parameters()})
    ref = {"loss": c["loss"], "h": c["h_out"], "x": c["x_out"], "dh": c["grad_h"], "dx": c["grad_x"]}
    ref.update(c["grads"])
    # the reference algorithm in fp32 on the same inputs sets the achievable bar
    p32 = {k: v.float().clone().requires_grad_(True) for k, v in c["state_dict"].items()}
    h32 = c["h"].float().clone().requires_grad_(True)
    x32 = c["x"].float().clone().requires_grad_(True)
    ho32, xo32 = O.egnn(p32, h32, x32, c["row"], c["col"],
                        c["edge_attr"].float() if c.get("edge_attr") is not None else None, **flags)
    l32 = _golden_loss(c, ho32, xo32)
    l32.backward()
    r32 = {"loss": l32, "h": ho32, "x": xo32, "dh": h32.grad, "dx": x32.grad}
    r32.update({k: (v.grad if v.grad is not None else torch.zeros_like(v)) for k, v in p32.items()})
    check_tensors(got, ref, tolerances(ref, r32, 1e-5, 3.0), name)


def _golden_loss(c, ho, xo):
    if c["kind"] == "model":
        from conftest import graph_sum
        pred = graph_sum(ho[:, 0], c["graph_ptr"])
        return ((pred - c["target"].to(pred.dtype).to(pred.device)) ** 2).mean()
    w = torch.linspace(-1, 1, 96, dtype=xo.dtype, device=xo.device).view(32, 3)
    return (ho ** 2).sum() + (xo * w).sum()


# ---------------------------------------------------------------------------
# seeded layer sweep against the fp64 oracle
# ---------------------------------------------------------------------------

def _seeded_layer_case(seed, N, E, H, edges_in_d=0, hub=True, attention=False):
    g = torch.Generator().manual_seed(seed)
    row = torch.randint(0, N, (E,), generator=g)
    col = torch.randint(0, N, (E,), generator=g)
    if hub:
        row[: E // 3] = 0           # one row much longer than an edge range
    p = O.init_params(H, H, 1, 1, in_edge_nf=edges_in_d, attention=attention, seed=seed, dtype=torch.float64)
    p = {k[len("gcl_0."):]: v for k, v in p.items() if k.startswith("gcl_0.")}
    # larger coord weights than the 0.001 xavier gain so the x path is exercised
    p["coord_mlp.2.weight"] = p["coord_mlp.2.weight"] * 300.0
    h = torch.randn(N, H, generator=g, dtype=torch.float64)
    x = torch.randn(N, 3, generator=g, dtype=torch.float64) * 1.5
    ea = torch.randn(E, edges_in_d, generator=g, dtype=torch.float64) if edges_in_d else None
    gh = torch.randn(N, H, generator=g, dtype=torch.float64)
    gx = torch.randn(N, 3, generator=g, dtype=torch.float64)
    return row, col, p, h, x, ea, gh, gx


LAYER_CASES = [
    # (H, precision, N, E, edges_in_d, flags)
    (32, "fp32", 300, 4000, 0, {}),
    (64, "fp32", 500, 12000, 0, {}),
    (128, "fp32", 700, 20000, 0, {}),
    (256, "fp32", 400, 9000, 0, {}),
    (64, "fp32", 300, 5000, 3, {"normalize": True, "tanh": True}),
    (128, "fp32", 300, 5000, 0, {"coords_agg": "sum", "residual": False}),
    (64, "bf16", 500, 12000, 0, {}),
    (128, "bf16", 700, 20000, 0, {}),
    (256, "bf16", 400, 9000, 0, {}),
    (128, "bf16", 300, 5000, 2, {"normalize": True}),            # tensor-core forward, SIMT backward
    (128, "bf16", 2000, 40000, 16, {"attention": True, "tanh": True}),
    # attention gate (SIMT path for every H and precision)
    (32, "fp32", 300, 4000, 2, {"attention": True, "tanh": True}),
    (128, "fp32", 700, 20000, 0, {"attention": True}),
    (256, "fp32", 400, 9000, 0, {"attention": True, "normalize": True}),
    (64, "bf16", 500, 12000, 0, {"attention": True, "coords_agg": "sum"}),
    (128, "bf16", 2000, 60000, 0, {"attention": True}),       # tensor-core forward, SIMT backward
    (128, "bf16", 3000, 100000, 0, {"attention": True, "normalize": True, "tanh": True, "coords_agg": "sum",
                                    "residual": False}),
    (256, "bf16", 400, 9000, 0, {"attention": True}),
    # tensor-core paths (bf16, no edge attributes): fused edge kernels at H = 128,
    # edge-row GEMMs at H = 256 (fewer edges than one tile; several tiles per CTA)
    (256, "bf16", 100, 90, 0, {}),
    (256, "bf16", 300, 128, 0, {}),                      # exactly one tile
    (256, "bf16", 1000, 128 * 148 + 1, 0, {"tanh": True}),   # 149 tiles: a second, one-row tile
    (256, "bf16", 2000, 60000, 0, {"normalize": True, "tanh": True, "coords_agg": "sum"}),
    (256, "bf16", 3000, 100000, 0, {"residual": False}),
    (128, "bf16", 100, 90, 0, {}),
    (128, "bf16", 2000, 60000, 0, {"normalize": True, "tanh": True, "coords_agg": "sum"}),
    (128, "bf16", 3000, 100000, 0, {"residual": False}),
]


@pytest.mark.parametrize("H,precision,N,E,d,flags", LAYER_CASES)
def test_layer_matches_oracle(H, precision, N, E, d, flags, cuda_device):
    dev = cuda_device
    row, col, p, h, x, ea, gh, gx = _seeded_layer_case(H * 7 + E, N, E, H, d, hub=True,
                                                       attention=flags.get("attention", False))
    ref = O.layer_grads(p, "", h, row, col, x, gh, gx, ea, **flags)
    layer = _layer_from_state(p, H, precision, dev, d, **flags)
    csr = CSR.from_edges(row, col, n_nodes=N, device=dev)
    res = _run_layer(layer, h.float().to(dev), x.float().to(dev), csr, gh.float().to(dev),
                     gx.float().to(dev), ea.float().to(dev) if ea is not None else None)
    got, refd = as_dict(res), as_dict(ref)
    what = f"H={H} {precision} d={d} {flags}"
    if precision == "fp32":
        check_tensors(got, refd, _fp32_tol(p, h, row, col, x, gh, gx, ea, ref, flags), what)
        return
    emu = as_dict(EM.layer_fwd_bwd(p, h, row, col, x, gh, gx, ea, precision="bf16", **flags))
    check_bf16(got, refd, emu, what)


# E_GCL(input_nf, output_nf, hidden_nf) with input_nf / output_nf other than
# hidden_nf (egnn_clean.py:11-31; EGNN itself always builds them equal)
DIM_CASES = [
    # (input_nf, output_nf, H, precision, N, E, edges_in_d, flags)
    (16, 16, 128, "bf16", 1500, 30000, 0, {}),                          # fused tensor-core edge kernels
    (40, 7, 256, "bf16", 600, 12000, 0, {"residual": False}),           # edge-row GEMMs
    (5, 1, 64, "fp32", 500, 8000, 0, {"residual": False}),
    (128, 32, 128, "fp32", 400, 6000, 2, {"residual": False, "attention": True}),
    (20, 20, 32, "bf16", 300, 4000, 0, {"normalize": True}),
    (3, 3, 128, "fp32", 700, 9000, 0, {"coords_agg": "sum"}),
]


@pytest.mark.parametrize("nin,nout,H,precision,N,E,d,flags", DIM_CASES)
def test_layer_with_other_input_output_widths(nin, nout, H, precision, N, E, d, flags, cuda_device):
    dev = cuda_device
    seed = nin * 31 + nout * 7 + H
    g = torch.Generator().manual_seed(seed)
    row = torch.randint(0, N, (E,), generator=g)
    col = torch.randint(0, N, (E,), generator=g)
    row[: E // 3] = 0
    torch.manual_seed(seed)
    cpu_layer = E_GCL(nin, nout, H, edges_in_d=d, **flags)      # the reference's shapes and init order
    p = {k: v.detach().double() for k, v in cpu_layer.state_dict().items()}
    p["coord_mlp.2.weight"] = p["coord_mlp.2.weight"] * 300.0
    h = torch.randn(N, nin, generator=g, dtype=torch.float64)
    x = torch.randn(N, 3, generator=g, dtype=torch.float64) * 1.5
    ea = torch.randn(E, d, generator=g, dtype=torch.float64) if d else None
    gh = torch.randn(N, nout, generator=g, dtype=torch.float64)
    gx = torch.randn(N, 3, generator=g, dtype=torch.float64)
    ref = O.layer_grads(p, "", h, row, col, x, gh, gx, ea, **flags)
    layer = _layer_from_state(p, H, precision, dev, d, nin, nout, **flags)
    csr = CSR.from_edges(row, col, n_nodes=N, device=dev)
    res = _run_layer(layer, h.float().to(dev), x.float().to(dev), csr, gh.float().to(dev),
                     gx.float().to(dev), ea.float().to(dev) if ea is not None else None)
    assert res[0].shape == (N, nout) and res[2].shape == (N, nin)
    got, refd = as_dict(res), as_dict(ref)
    what = f"in={nin} out={nout} H={H} {precision} d={d} {flags}"
    if precision == "fp32":
        check_tensors(got, refd, _fp32_tol(p, h, row, col, x, gh, gx, ea, ref, flags), what)
        return
    emu = as_dict(EM.layer_fwd_bwd(p, h, row, col, x, gh, gx, ea, precision="bf16", **flags))
    check_bf16(got, refd, emu, what)


@pytest.mark.parametrize("H,precision", [(64, "fp32"), (256, "bf16")])
def test_layer_without_edges(H, precision, cuda_device):
    """E = 0: agg = 0, x' = x, only the node MLP acts (the edge-row path at
    H = 256 still writes zero edge-weight gradients)."""
    dev = cuda_device
    N = 20
    row = torch.zeros(0, dtype=torch.int64)
    col = torch.zeros(0, dtype=torch.int64)
    _, _, p, h, x, _, gh, gx = _seeded_layer_case(1, N, 10, H)
    ref = O.layer_grads(p, "", h, row, col, x, gh, gx)
    layer = _layer_from_state(p, H, precision, dev)
    csr = CSR.from_edges(row, col, n_nodes=N, device=dev)
    res = _run_layer(layer, h.float().to(dev), x.float().to(dev), csr, gh.float().to(dev), gx.float().to(dev))
    if precision == "fp32":
        tol = _fp32_tol(p, h, row, col, x, gh, gx, None, ref, {})
        check_tensors(as_dict(res), as_dict(ref), tol, f"no edges H={H} {precision}")
    else:
        emu = as_dict(EM.layer_fwd_bwd(p, h, row, col, x, gh, gx, None, precision="bf16"))
        check_bf16(as_dict(res), as_dict(ref), emu, f"no edges H={H} {precision}")


def test_single_edge_and_isolated_nodes(cuda_device):
    dev = cuda_device
    N, H = 9, 32
    row = torch.tensor([4])
    col = torch.tensor([7])
    _, _, p, h, x, _, gh, gx = _seeded_layer_case(2, N, 10, H)
    ref = O.layer_grads(p, "", h, row, col, x, gh, gx)
    layer = _layer_from_state(p, H, "fp32", dev)
    csr = CSR.from_edges(row, col, n_nodes=N, device=dev)
    res = _run_layer(layer, h.float().to(dev), x.float().to(dev), csr, gh.float().to(dev), gx.float().to(dev))
    check_tensors(as_dict(res), as_dict(ref), _fp32_tol(p, h, row, col, x, gh, gx, None, ref, {}), "single edge")


@pytest.mark.parametrize("precision,H", [("fp32", 128), ("bf16", 128), ("bf16", 256)])
def test_backward_is_deterministic(precision, H, cuda_device):
    dev = cuda_device
    N, E = 2000, 60000
    row, col, p, h, x, _, gh, gx = _seeded_layer_case(9, N, E, H)
    layer = _layer_from_state(p, H, precision, dev)
    csr = CSR.from_edges(row, col, n_nodes=N, device=dev)
    args = (h.float().to(dev), x.float().to(dev), csr, gh.float().to(dev), gx.float().to(dev))
    a = _run_layer(layer, *args)
    b = _run_layer(layer, *args)
    for u, v in zip(a[:4], b[:4]):
        assert torch.equal(u, v)
    for k in a[4]:
        assert torch.equal(a[4][k], b[4][k]), k
    assert nat.lib().egnn_device_status(nat.stream_ptr()) == nat.EGNN_OK, nat.last_error()


# ---------------------------------------------------------------------------
# CSR construction and guards
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("N,E", [(1, 0), (10, 1), (97, 1000), (5000, 200000)])
def test_csr_build_bit_exact(N, E, cuda_device):
    g = torch.Generator().manual_seed(N + E)
    row = torch.randint(0, N, (E,), generator=g)
    col = torch.randint(0, N, (E,), generator=g)
    csr = CSR.from_edges(row, col, n_nodes=N, device=cuda_device)
    rp, ci, ri, eid = CO.csr_build(row.numpy(), col.numpy(), N)
    assert np.array_equal(csr.row_ptr.cpu().numpy(), rp)
    assert np.array_equal(csr.col_idx.cpu().numpy(), ci)
    assert np.array_equal(csr.row_idx.cpu().numpy(), ri)
    assert np.array_equal(csr.edge_id.cpu().numpy(), eid)
    sp, se = CO.csr_transpose(ci, N)
    assert np.array_equal(csr.src_ptr.cpu().numpy(), sp)
    assert np.array_equal(csr.src_edge.cpu().numpy(), se)
    srt, perm = torch.sort(row, stable=True)
    assert torch.equal(csr.edge_id.cpu().long(), perm)


def test_csr_deferred_validation(cuda_device):
    """from_edges(check=False) builds the same CSR without a host read-back and
    leaves the validation result on the device; a bad index is flagged (and the
    CSR stays in range) instead of raising at build time."""
    g = torch.Generator().manual_seed(4)
    N, E = 300, 5000
    row = torch.randint(0, N, (E,), generator=g)
    col = torch.randint(0, N, (E,), generator=g)
    a = CSR.from_edges(row, col, n_nodes=N, device=cuda_device)
    b = CSR.from_edges(row, col, n_nodes=N, device=cuda_device, check=False)
    for f in ("row_ptr", "col_idx", "row_idx", "edge_id", "src_ptr", "src_edge"):
        assert torch.equal(getattr(a, f), getattr(b, f)), f
    b.raise_if_invalid()
    bad_col = col.clone()
    bad_col[17] = N + 4
    c = CSR.from_edges(row, bad_col, n_nodes=N, device=cuda_device, check=False)
    assert int(c.col_idx.min()) >= 0 and int(c.col_idx.max()) < N
    with pytest.raises(nat.EgnnError) as ei:
        c.raise_if_invalid()
    assert ei.value.status == nat.EGNN_ERR_INDEX


def test_csr_from_reference_triple(cuda_device):
    g = torch.Generator().manual_seed(3)
    N, E = 200, 3000
    row = torch.randint(0, N, (E,), generator=g)
    col = torch.randint(0, N, (E,), generator=g)
    rp, ci, ri, eid = CO.csr_build(row.numpy(), col.numpy(), N)
    csr = CSR.from_csr(torch.from_numpy(rp), torch.from_numpy(ci), torch.from_numpy(eid), device=cuda_device)
    assert np.array_equal(csr.row_idx.cpu().numpy(), ri)


def test_guards_return_errors_not_faults(cuda_device):
    dev = cuda_device
    with pytest.raises(nat.EgnnError) as ei:
        CSR.from_edges(torch.tensor([0, 1, 2]), torch.tensor([1, 9, 0]), n_nodes=5, device=dev)
    assert ei.value.status == nat.EGNN_ERR_INDEX
    with pytest.raises(nat.EgnnError) as ei:
        CSR.from_edges(torch.tensor([0, -1]), torch.tensor([1, 0]), n_nodes=5, device=dev)
    assert ei.value.status == nat.EGNN_ERR_INDEX
    # non-monotone row_ptr
    with pytest.raises(nat.EgnnError) as ei:
        CSR.from_csr(torch.tensor([0, 3, 1, 4]), torch.tensor([0, 1, 2, 0]), n_nodes=3, device=dev)
    assert ei.value.status == nat.EGNN_ERR_INDEX
    # column out of range in a caller CSR
    with pytest.raises(nat.EgnnError):
        CSR.from_csr(torch.tensor([0, 1, 2, 2]), torch.tensor([0, 7]), n_nodes=3, device=dev)
    # wrong dtype / device
    layer = E_GCL(32, 32, 32).to(dev)
    csr = CSR.from_edges(torch.tensor([0, 1]), torch.tensor([1, 0]), n_nodes=2, device=dev)
    with pytest.raises(TypeError):
        layer(torch.zeros(2, 32, device=dev, dtype=torch.float64), csr, torch.zeros(2, 3, device=dev))
    with pytest.raises(ValueError):
        layer(torch.zeros(2, 32), csr, torch.zeros(2, 3))


def test_legacy_edge_list_equals_csr(cuda_device):
    dev = cuda_device
    c = load_golden("layer_default_h64")
    layer = _layer_from_state(c["state_dict"], 64, "fp32", dev)
    h, x = c["h"].float().to(dev), c["x"].float().to(dev)
    a = layer(h, [c["row"].to(dev), c["col"].to(dev)], x)
    csr = CSR.from_edges(c["row"], c["col"], n_nodes=h.shape[0], device=dev)
    b = layer(h, csr, x)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
