"""Node-side GEMMs (embedding layers and the node MLP GEMMs of the layer) at
fp32 accuracy: egnn_linear_fwd / egnn_linear_bwd against float64 torch,
covering both operand layouts, ragged M and K tails, split-K weight
gradients and the fused bias-gradient sum."""
import pytest
import torch

from conftest import rel_err
from pymolecular_b200 import _native as nat

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("m,k,o", [(1000, 64, 128), (777, 96, 256), (10000, 128, 32), (9939, 5, 128),
                                   (4097, 128, 1), (130, 256, 128), (33, 40, 64), (300, 1, 7), (5000, 8, 1),
                                   (65, 3, 300),
                                   # weight gradients with one narrow side at many stages of rows: the
                                   # embeddings of configs 3-5 (narrow groups of 9, 16-byte and 4-byte
                                   # staging of the wide side)
                                   (200000, 16, 128), (300000, 128, 1), (50000, 40, 256), (20000, 20, 128),
                                   (7000, 44, 100), (7000, 44, 99)])
def test_linear_fwd_bwd_fp32_accuracy(m, k, o, cuda_device):
    g = torch.Generator(device=cuda_device).manual_seed(m + k + o)
    x = torch.randn(m, k, device=cuda_device, generator=g)
    w = torch.randn(o, k, device=cuda_device, generator=g) / k ** 0.5
    b = torch.randn(o, device=cuda_device, generator=g)
    dy = torch.randn(m, o, device=cuda_device, generator=g)
    lib = nat.lib()
    y = torch.empty(m, o, device=cuda_device)
    nat.check(lib.egnn_linear_fwd(m, k, o, nat.ptr(x), nat.ptr(w), nat.ptr(b), nat.ptr(y), nat.stream_ptr()))
    dx, dw, db = torch.empty_like(x), torch.empty_like(w), torch.empty_like(b)
    ws_bytes = lib.egnn_linear_workspace_size(m, k, o)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=cuda_device)
    nat.check(lib.egnn_linear_bwd(m, k, o, nat.ptr(x), nat.ptr(w), nat.ptr(dy), nat.ptr(dx), nat.ptr(dw),
                                  nat.ptr(db), nat.ptr(ws), ws_bytes, nat.stream_ptr()))
    assert lib.egnn_device_status(nat.stream_ptr()) == nat.EGNN_OK, nat.last_error()
    xd, wd, bd, dyd = x.double(), w.double(), b.double(), dy.double()
    assert rel_err(y, xd @ wd.t() + bd) < 1e-5
    assert rel_err(dx, dyd @ wd) < 1e-5
    assert rel_err(dw, dyd.t() @ xd) < 1e-5
    assert rel_err(db, dyd.sum(0)) < 1e-5
