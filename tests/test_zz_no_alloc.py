"""egnn_linear_bwd_static: the allocation-free embedding backward.

Callers that cannot call cudaMalloc (a plugin whose host framework owns all
device memory and offers it no workspace) use this entry point; its
scratch is a fixed array inside the library.  It must give the same result
as egnn_linear_bwd with a caller workspace, call after call, and refuse
shapes whose scratch would not fit.  This file is collected last on purpose.
"""
import pytest
import torch

from conftest import rel_err
from pymolecular_b200 import _native as nat

pytestmark = pytest.mark.gpu

TOL = 1e-5   # the fp32 bar of the parity tests; the two paths normally agree bit for bit


def _with_workspace(lib, m, k, o, x, w, dy):
    dx, dw, db = torch.empty_like(x), torch.empty_like(w), torch.empty(o, device=x.device)
    ws_bytes = lib.egnn_linear_workspace_size(m, k, o)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=x.device)
    nat.check(lib.egnn_linear_bwd(m, k, o, nat.ptr(x), nat.ptr(w), nat.ptr(dy), nat.ptr(dx), nat.ptr(dw),
                                  nat.ptr(db), nat.ptr(ws), ws_bytes, nat.stream_ptr()), "egnn_linear_bwd")
    return dx, dw, db


def _static(lib, m, k, o, x, w, dy):
    dx, dw, db = torch.empty_like(x), torch.empty_like(w), torch.empty(o, device=x.device)
    nat.check(lib.egnn_linear_bwd_static(m, k, o, nat.ptr(x), nat.ptr(w), nat.ptr(dy), nat.ptr(dx),
                                         nat.ptr(dw), nat.ptr(db), nat.stream_ptr()),
              "egnn_linear_bwd_static")
    return dx, dw, db


@pytest.mark.parametrize("m,k,o", [(9939, 5, 128), (8192, 40, 256), (9939, 128, 1)])
def test_static_scratch_matches_workspace_path(m, k, o, cuda_device):
    lib = nat.lib()
    assert lib.egnn_linear_workspace_size(m, k, o) <= nat.LINEAR_BWD_STATIC_SCRATCH_BYTES
    g = torch.Generator(device=cuda_device).manual_seed(m + k + o)
    for call in range(2):   # two calls in a row: the array keeps the previous call's contents
        x = torch.randn(m, k, device=cuda_device, generator=g)
        w = torch.randn(o, k, device=cuda_device, generator=g)
        dy = torch.randn(m, o, device=cuda_device, generator=g)
        ref = _with_workspace(lib, m, k, o, x, w, dy)
        got = _static(lib, m, k, o, x, w, dy)
        torch.cuda.synchronize()
        for name, a, b in zip(("dx", "dw", "db"), got, ref):
            assert rel_err(a, b) <= TOL, (call, name, rel_err(a, b))


def test_static_scratch_rejects_oversized_shapes(cuda_device):
    lib = nat.lib()
    m, k, o = 1 << 20, 512, 512
    assert lib.egnn_linear_workspace_size(m, k, o) > nat.LINEAR_BWD_STATIC_SCRATCH_BYTES
    status = lib.egnn_linear_bwd_static(m, k, o, None, None, None, None, None, None, nat.stream_ptr())
    assert status == nat.EGNN_ERR_WORKSPACE
    assert "static array" in nat.last_error()
