"""Host-side checks that need no GPU: the C ABI library loads and exports every
declared symbol, size queries behave, and the module API mirrors the reference."""
import ctypes as C
import re
from pathlib import Path

import pytest
import torch
from torch import nn

from conftest import ROOT, load_golden
from pymolecular_b200 import _native as nat
from pymolecular_b200 import EGNN, E_GCL


def declared_symbols():
    text = (ROOT / "include" / "egnn_b200.h").read_text()
    return sorted(set(re.findall(r"EGNN_API\s+[\w\s\*]+?\b(egnn_\w+)\s*\(", text)))


def test_header_declares_the_abi():
    syms = declared_symbols()
    for name in ["egnn_csr_build", "egnn_csr_transpose", "egnn_layer_fwd", "egnn_layer_bwd",
                 "egnn_workspace_size", "egnn_last_error"]:
        assert name in syms


def test_library_exports_every_declared_symbol():
    lib = nat.lib()
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert set(declared_symbols()) == set(nat.EXPORTED)


def test_version_and_error_plumbing():
    lib = nat.lib()
    assert lib.egnn_version().startswith(b"egnn_b200")
    assert isinstance(nat.last_error(), str)


def test_workspace_sizes_are_host_only_and_monotone():
    lib = nat.lib()
    small = nat.LayerDesc(1000, 20000, 128, 0, nat.FLAG_RESIDUAL, nat.PREC_FP32)
    big = nat.LayerDesc(4000, 80000, 128, 0, nat.FLAG_RESIDUAL, nat.PREC_FP32)
    for which in (nat.WS_FWD, nat.WS_BWD):
        a = lib.egnn_workspace_size(C.byref(small), which, 148)
        b = lib.egnn_workspace_size(C.byref(big), which, 148)
        assert 0 < a < b
    # backward keeps one H-vector per edge: at least E*H*4 bytes
    assert lib.egnn_workspace_size(C.byref(big), nat.WS_BWD, 148) >= 80000 * 128 * 4
    # per node: agg (H), P and Q (2H), node-MLP pre-activation and activation (2H)
    assert lib.egnn_saved_size(C.byref(small)) == 1000 * 5 * 128 * 4
    assert lib.egnn_csr_workspace_size(1000, 20000) >= 4 * 20000 * 4


def test_workspace_size_rejects_unsupported_shapes():
    lib = nat.lib()
    for d in [nat.LayerDesc(10, 10, 48, 0, 1, 0),          # hidden not built
              nat.LayerDesc(10, 10, 64, 17, 1, 0),         # too many edge features
              nat.LayerDesc(10, 10, 64, 0, 1, 7),          # unknown precision
              nat.LayerDesc(10, 10, 64, 0, 64, 0)]:        # unknown flag bit
        assert lib.egnn_workspace_size(C.byref(d), nat.WS_FWD, 148) == 0


def test_attention_workspace_holds_gate_scratch():
    """attention=True is built: its backward workspace adds the per-CTA scratch
    of the gate (ungated messages of a chunk and the gate-gradient sums)."""
    lib = nat.lib()
    plain = nat.LayerDesc(1000, 50000, 128, 0, 1, 0)
    att = nat.LayerDesc(1000, 50000, 128, 0, 1 | nat.FLAG_ATTENTION, 0)
    assert lib.egnn_workspace_size(C.byref(att), nat.WS_FWD, 148) == \
        lib.egnn_workspace_size(C.byref(plain), nat.WS_FWD, 148)
    extra = lib.egnn_workspace_size(C.byref(att), nat.WS_BWD, 148) - \
        lib.egnn_workspace_size(C.byref(plain), nat.WS_BWD, 148)
    # at most 148 x 8 CTAs, each with 64 x 128 + 16 x 129 floats
    assert 0 < extra <= 148 * 8 * (64 * 128 + 16 * 129) * 4 + 256


def test_edge_row_path_workspace_holds_the_per_edge_operands():
    """bf16 mode at H = 256 runs the edge-row tensor-core GEMMs, whose workspace
    carries the per-edge operands between kernels; the fused paths keep only
    per-edge gradients (backward) and nothing per edge in the forward."""
    lib = nat.lib()

    def per_edge(which, prec, H):
        E0, E1 = 100_000, 1_100_000
        d0 = nat.LayerDesc(30000, E0, H, 0, nat.FLAG_RESIDUAL, prec)
        d1 = nat.LayerDesc(30000, E1, H, 0, nat.FLAG_RESIDUAL, prec)
        return (lib.egnn_workspace_size(C.byref(d1), which, 148) -
                lib.egnn_workspace_size(C.byref(d0), which, 148)) / (E1 - E0)

    # forward: u1 and m tiles (2 x 512 B), fp32 m (1 KB), phi, geometry (16 B)
    assert 2048 + 16 <= per_edge(nat.WS_FWD, nat.PREC_BF16, 256) < 2048 + 64
    # backward: four bf16 tiles and two fp16 row sets (6 x 512 B), dL/da1 rows
    # (1 KB slot), coordinate gradients, factors, geometry, phi
    assert 3072 + 1024 + 48 <= per_edge(nat.WS_BWD, nat.PREC_BF16, 256) < 3072 + 1024 + 128
    # fp32 mode (SIMT kernels) and the fused H = 128 tensor-core path
    assert per_edge(nat.WS_FWD, nat.PREC_FP32, 256) == 0
    assert per_edge(nat.WS_BWD, nat.PREC_FP32, 256) == 256 * 4 + 16
    assert per_edge(nat.WS_FWD, nat.PREC_BF16, 128) == 0
    assert per_edge(nat.WS_BWD, nat.PREC_BF16, 128) == 128 * 4 + 16


def test_attention_state_dict_matches_reference():
    c = load_golden("model_attention_molecules")
    torch.manual_seed(7)
    m = EGNN(in_node_nf=5, hidden_nf=32, out_node_nf=1, n_layers=2, attention=True)
    sd = m.state_dict()
    assert list(sd) == list(c["state_dict"])
    for k, v in sd.items():
        assert torch.equal(v.double(), c["state_dict"][k]), k


def test_state_dict_names_and_seeded_init_match_reference():
    c = load_golden("model_molecules")
    torch.manual_seed(1)
    m = EGNN(in_node_nf=5, hidden_nf=32, out_node_nf=1, n_layers=2)
    sd = m.state_dict()
    assert list(sd) == list(c["state_dict"])
    for k, v in sd.items():
        assert torch.equal(v.double(), c["state_dict"][k]), k
    # and it loads reference checkpoints as they are
    m.load_state_dict({k: v.float() for k, v in c["state_dict"].items()})


@pytest.mark.parametrize("name", ["layer_dims_i16_o8_h32", "layer_dims_i12_h64"])
def test_other_input_output_widths_match_reference_shapes_and_init(name):
    """E_GCL(input_nf, output_nf, hidden_nf) with widths other than hidden_nf:
    the same parameter names, shapes and seeded initial values as the
    reference module the fixture was made from."""
    c = load_golden(name)
    torch.manual_seed(int(c["name"] == "layer_dims_i12_h64") + 8)   # the fixtures' seeds: 8, 9
    layer = E_GCL(c["input_nf"], c["output_nf"], c["hidden"], edges_in_d=c["edges_in_d"], **c["flags"])
    sd = layer.state_dict()
    assert list(sd) == list(c["state_dict"])
    for k, v in sd.items():
        assert torch.equal(v.double(), c["state_dict"][k]), k


def test_widths_in_the_layer_descriptor():
    lib = nat.lib()
    same = nat.LayerDesc(1000, 20000, 64, 0, 0, nat.PREC_FP32)
    wide = nat.LayerDesc(1000, 20000, 64, 0, 0, nat.PREC_FP32, 200, 300)
    assert lib.egnn_workspace_size(C.byref(wide), nat.WS_BWD, 148) > lib.egnn_workspace_size(
        C.byref(same), nat.WS_BWD, 148)
    # the residual needs input_nf == output_nf; widths above 1024 are not built
    for d in [nat.LayerDesc(10, 10, 64, 0, nat.FLAG_RESIDUAL, 0, 16, 8),
              nat.LayerDesc(10, 10, 64, 0, 0, 0, 2000, 8)]:
        assert lib.egnn_workspace_size(C.byref(d), nat.WS_FWD, 148) == 0
    layer = E_GCL(16, 8, 32)       # residual=True by default, as in the reference
    with pytest.raises(NotImplementedError, match="input_nf == output_nf"):
        layer(torch.zeros(4, 16), [torch.tensor([0]), torch.tensor([1])], torch.zeros(4, 3))


def test_e_gcl_signature_guards():
    with pytest.raises(NotImplementedError):
        E_GCL(32, 32, 32, act_fn=nn.ReLU())
    with pytest.raises(Exception):
        E_GCL(32, 32, 32, coords_agg="max")
    with pytest.raises(ValueError):
        E_GCL(32, 32, 32, precision="fp8")


def test_cpu_tensors_are_rejected_not_computed():
    m = EGNN(in_node_nf=5, hidden_nf=32, out_node_nf=1, n_layers=1)
    h = torch.zeros(4, 5)
    x = torch.zeros(4, 3)
    with pytest.raises(ValueError, match="CUDA"):
        m(h, x, [torch.tensor([0, 1]), torch.tensor([1, 0])], None)


def test_precision_switch():
    m = EGNN(in_node_nf=5, hidden_nf=32, out_node_nf=1, n_layers=2, precision="bf16")
    assert m.precision == "bf16"
    m.precision = "fp32"
    assert all(m._modules[f"gcl_{i}"].precision == "fp32" for i in range(2))


def test_flag_bits_match_header():
    text = (ROOT / "include" / "egnn_b200.h").read_text()
    for name, val in [("EGNN_FLAG_RESIDUAL", nat.FLAG_RESIDUAL), ("EGNN_FLAG_ATTENTION", nat.FLAG_ATTENTION),
                      ("EGNN_FLAG_NORMALIZE", nat.FLAG_NORMALIZE), ("EGNN_FLAG_TANH", nat.FLAG_TANH),
                      ("EGNN_FLAG_COORDS_SUM", nat.FLAG_COORDS_SUM)]:
        assert re.search(rf"{name}\s*=\s*{val}\b", text), name
    assert len(nat.LayerDesc._fields_) == 8 and C.sizeof(nat.LayerDesc) == 40
    assert C.sizeof(nat.Graph) == 6 * 8
    assert C.sizeof(nat.LayerParams) == 13 * 8


def test_no_oracle_import_in_product():
    """The product path never imports the CPU oracle (it must fail loudly instead)."""
    pat = re.compile(r"^\s*(from\s+oracle|import\s+oracle)", re.M)
    for p in (ROOT / "pymolecular_b200").rglob("*.py"):
        assert not pat.search(p.read_text()), p


def test_graph_mse_entry_points_validate_before_any_launch():
    """The loss entry points reject bad shapes and null pointers with an
    error status (no GPU needed: nothing is launched)."""
    lib = nat.lib()
    assert lib.egnn_graph_mse_workspace_size(0) > 0
    assert lib.egnn_graph_mse_workspace_size(10_000_000) >= 2 * 4 * (10_000_000 // 2048)
    # nodes without graphs, negative sizes, null pointers
    assert lib.egnn_graph_mse_fwd(10, 0, 1, 1, 1, 1, 1, 1, 1, 1 << 20, None) == nat.EGNN_ERR_INVALID_ARG
    assert lib.egnn_graph_mse_fwd(-1, 1, 1, 1, 1, 1, 1, 1, 1, 1 << 20, None) == nat.EGNN_ERR_INVALID_ARG
    assert lib.egnn_graph_mse_fwd(10, 2, None, 1, 1, 1, 1, 1, 1, 1 << 20, None) == nat.EGNN_ERR_INVALID_ARG
    assert lib.egnn_graph_mse_fwd(10, 2, 1, 1, 1, 1, 1, 1, 1, 0, None) == nat.EGNN_ERR_WORKSPACE
    assert lib.egnn_graph_mse_bwd(10, 0, 1, 1, 1, 1, 1, 1, None) == nat.EGNN_ERR_INVALID_ARG
    assert lib.egnn_graph_mse_bwd(10, 2, 1, None, 1, 1, 1, 1, None) == nat.EGNN_ERR_INVALID_ARG
    assert lib.egnn_graph_mse_bwd(0, 0, None, None, None, None, None, 1, None) == nat.EGNN_OK
    with pytest.raises(ValueError, match="CUDA"):
        from pymolecular_b200 import graph_sum_mse
        graph_sum_mse(torch.zeros(4), torch.tensor([0, 4]), torch.zeros(1))


def test_bf16_workspaces_hold_the_split_weight_images():
    """bf16 mode: the layer's prep writes split bf16 tile images of the node
    GEMMs' weights into the workspace (hi and lo parts, 64 x 64 blocks in
    64-row chunks, column blocks padded to a multiple of 4)."""
    lib = nat.lib()

    def image_bytes(K, N):
        nkc = (K + 63) // 64
        nb = ((N + 63) // 64 + 3) // 4 * 4
        return 2 * nkc * nb * 8192

    H, N, E = 64, 5000, 60000
    fp = nat.LayerDesc(N, E, H, 0, 0, nat.PREC_FP32)   # H = 64: the SIMT edge kernels in both precisions
    bf = nat.LayerDesc(N, E, H, 0, 0, nat.PREC_BF16)
    fwd = image_bytes(H, 2 * H) + image_bytes(2 * H, H) + image_bytes(H, H)
    bwd = image_bytes(H, H) + image_bytes(H, 2 * H) + image_bytes(2 * H, H)
    assert lib.egnn_workspace_size(C.byref(bf), nat.WS_FWD, 148) >= lib.egnn_workspace_size(
        C.byref(fp), nat.WS_FWD, 148) + fwd
    assert lib.egnn_workspace_size(C.byref(bf), nat.WS_BWD, 148) >= lib.egnn_workspace_size(
        C.byref(fp), nat.WS_BWD, 148) + bwd
