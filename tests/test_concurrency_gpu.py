"""The C ABI is safe across host threads on distinct streams.

egnn_layer_bwd forks its parameter-gradient work onto side streams and joins
them with events.  Two host threads that each run backwards on their own
stream must not record or wait on each other's events: if they did, one
call's side work could start before that call's producers finished and read
stale workspace contents.  Each call here gets different upstream gradients,
so any such mix-up changes its outputs; every output must equal, bit for bit,
the same call made alone.  ctypes releases the GIL during the foreign call,
so the two threads enqueue their work truly concurrently.
"""
import ctypes as C
import threading

import pytest
import torch

from pymolecular_b200 import CSR, E_GCL
from pymolecular_b200 import _native as nat
from pymolecular_b200.egnn import _PRECISIONS, _ptrs

pytestmark = pytest.mark.gpu


class _Call:
    """The buffers of one egnn_layer_bwd call (inputs shared, outputs own)."""

    def __init__(self, layer, h, x, csr, saved, gh, gx):
        self.layer, self.h, self.x, self.csr, self.saved, self.gh, self.gx = layer, h, x, csr, saved, gh, gx
        N, H = h.shape
        self.desc = nat.LayerDesc(N, csr.n_edges, H, 0, layer._flags(), _PRECISIONS[layer.precision])
        self.params = [t.detach() for t in layer._params()]
        self.grad_h = torch.empty_like(h)
        self.grad_x = torch.empty_like(x)
        self.grads = [torch.empty_like(t) for t in self.params]

    def outputs(self):
        return [self.grad_h, self.grad_x] + self.grads

    def run(self, ws, stream_handle):
        lib = nat.lib()
        p = nat.LayerParams(*_ptrs(self.params))
        gp = nat.LayerGrads(*_ptrs(self.grads))
        return lib.egnn_layer_bwd(C.byref(self.desc), C.byref(self.csr.struct()), C.byref(p), nat.ptr(self.h),
                                  nat.ptr(self.x), None, nat.ptr(self.saved), nat.ptr(self.gh), nat.ptr(self.gx),
                                  nat.ptr(self.grad_h), nat.ptr(self.grad_x), C.byref(gp), nat.ptr(ws),
                                  ws.numel(), stream_handle)


@pytest.mark.parametrize("H,precision", [(128, "bf16"), (256, "bf16"), (64, "fp32")])
def test_concurrent_backwards_on_two_streams_match_serial_calls(H, precision, cuda_device):
    dev = cuda_device
    N, E, iters = 2000, 40000, 6
    g = torch.Generator().manual_seed(H)
    row = torch.randint(0, N, (E,), generator=g)
    col = torch.randint(0, N, (E,), generator=g)
    torch.manual_seed(H)
    layer = E_GCL(H, H, H, precision=precision).to(dev)
    with torch.no_grad():
        layer.coord_mlp[2].weight.mul_(300.0)   # exercise the coordinate path
    csr = CSR.from_edges(row, col, n_nodes=N, device=dev)
    h = torch.randn(N, H, device=dev)
    x = torch.randn(N, 3, device=dev) * 1.5
    lib = nat.lib()
    desc = nat.LayerDesc(N, E, H, 0, layer._flags(), _PRECISIONS[precision])
    saved = torch.empty(lib.egnn_saved_size(C.byref(desc)) // 4, device=dev)
    h_out, x_out = torch.empty_like(h), torch.empty_like(x)
    ws_f = torch.empty(lib.egnn_workspace_size(C.byref(desc), nat.WS_FWD, 0), dtype=torch.uint8, device=dev)
    p = nat.LayerParams(*_ptrs([t.detach() for t in layer._params()]))
    nat.check(lib.egnn_layer_fwd(C.byref(desc), C.byref(csr.struct()), C.byref(p), nat.ptr(h), nat.ptr(x), None,
                                 nat.ptr(h_out), nat.ptr(x_out), nat.ptr(saved), nat.ptr(ws_f), ws_f.numel(),
                                 nat.stream_ptr()), "egnn_layer_fwd")
    ws_bytes = lib.egnn_workspace_size(C.byref(desc), nat.WS_BWD, 0)

    # thread t, iteration i: its own upstream gradients and outputs
    calls = [[_Call(layer, h, x, csr, saved, torch.randn(N, H, device=dev) * (1 + i + 7 * t),
                    torch.randn(N, 3, device=dev) * (1 + i - 3 * t)) for i in range(iters)] for t in range(2)]

    # each call alone, synchronised, on the current stream
    ref = []
    ws0 = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    for t in range(2):
        for c in calls[t]:
            nat.check(c.run(ws0, nat.stream_ptr()), "egnn_layer_bwd (serial)")
            torch.cuda.synchronize()
            ref.append([o.clone() for o in c.outputs()])

    # the same calls from two threads, each on its own stream with its own workspace
    streams = [torch.cuda.Stream(device=dev) for _ in range(2)]
    wss = [torch.empty(ws_bytes, dtype=torch.uint8, device=dev) for _ in range(2)]
    for s in streams:
        s.wait_stream(torch.cuda.current_stream())
    for t in range(2):
        for c in calls[t]:
            for o in c.outputs():
                o.fill_(float("nan"))
    torch.cuda.synchronize()
    status = [[None] * iters for _ in range(2)]
    start = threading.Barrier(2)

    def worker(t):
        torch.cuda.set_device(dev)
        start.wait()
        for i, c in enumerate(calls[t]):
            status[t][i] = c.run(wss[t], streams[t].cuda_stream)

    threads = [threading.Thread(target=worker, args=(t,)) for t in range(2)]
    for th in threads:
        th.start()
    for th in threads:
        th.join()
    torch.cuda.synchronize()
    assert all(s == nat.EGNN_OK for row_ in status for s in row_), (status, nat.last_error())
    k = 0
    for t in range(2):
        for i, c in enumerate(calls[t]):
            for j, (a, b) in enumerate(zip(c.outputs(), ref[k])):
                assert torch.equal(a, b), f"thread {t} call {i} output {j} differs from the serial call"
            k += 1
    assert lib.egnn_device_status(nat.stream_ptr()) == nat.EGNN_OK, nat.last_error()
