"""The bounded waits of the tensor-core edge kernels give up cleanly.

Every mbarrier wait in the fused tcgen05 edge kernels has a poll limit.  A
kernel whose wait runs out counts the event, waits (with the built-in limit)
for the MMAs it already issued, frees its tensor memory and returns, so the
context stays usable; egnn_device_status then reports the event.  The
debugging setting EGNN_DEBUG_WAIT_POLLS=0 makes the first MMA-completion wait
of every such kernel give up at once (nothing is made to hang: the MMAs do
complete, and the drain wait sees them complete).  The test checks that the
status reports it and that the next calls, with the setting removed, give the
same results as before.
"""
import os

import pytest
import torch

from pymolecular_b200 import CSR, E_GCL
from pymolecular_b200 import _native as nat

pytestmark = pytest.mark.gpu


def _layer_step(layer, h, x, csr, gh, gx):
    h = h.clone().requires_grad_(True)
    x = x.clone().requires_grad_(True)
    ho, xo, _ = layer(h, csr, x)
    torch.autograd.backward([ho, xo], [gh, gx])
    out = [ho.detach(), xo.detach(), h.grad, x.grad] + [p.grad.clone() for p in layer.parameters()]
    for p in layer.parameters():
        p.grad = None
    return out


def test_wait_give_up_is_reported_and_the_context_stays_usable(cuda_device, monkeypatch):
    dev = cuda_device
    N, E, H = 1500, 30000, 128
    g = torch.Generator().manual_seed(5)
    row = torch.randint(0, N, (E,), generator=g)
    col = torch.randint(0, N, (E,), generator=g)
    torch.manual_seed(5)
    layer = E_GCL(H, H, H, precision="bf16").to(dev)   # bf16, H = 128: the fused tcgen05 edge kernels
    csr = CSR.from_edges(row, col, n_nodes=N, device=dev)
    h = torch.randn(N, H, device=dev)
    x = torch.randn(N, 3, device=dev)
    gh = torch.randn(N, H, device=dev)
    gx = torch.randn(N, 3, device=dev)
    lib = nat.lib()
    monkeypatch.delenv("EGNN_DEBUG_WAIT_POLLS", raising=False)
    ref = _layer_step(layer, h, x, csr, gh, gx)
    assert lib.egnn_device_status(nat.stream_ptr()) == nat.EGNN_OK, nat.last_error()

    monkeypatch.setenv("EGNN_DEBUG_WAIT_POLLS", "0")
    _layer_step(layer, h, x, csr, gh, gx)          # every tensor-core edge kernel gives up
    status = lib.egnn_device_status(nat.stream_ptr())
    assert status == nat.EGNN_ERR_CUDA
    assert "timed out" in nat.last_error()
    # the counter was reset by the status call
    assert lib.egnn_device_status(nat.stream_ptr()) == nat.EGNN_OK

    monkeypatch.delenv("EGNN_DEBUG_WAIT_POLLS")
    again = _layer_step(layer, h, x, csr, gh, gx)
    assert lib.egnn_device_status(nat.stream_ptr()) == nat.EGNN_OK, nat.last_error()
    for k, (a, b) in enumerate(zip(again, ref)):
        assert torch.equal(a, b), k
    assert "EGNN_DEBUG_WAIT_POLLS" not in os.environ
