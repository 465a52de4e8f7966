"""Drop-in ``E_GCL`` and ``EGNN`` modules backed by the sm_100a kernels.

Same constructor arguments, submodule names, parameter shapes and forward
signatures as the reference ``models/EGNN/egnn_clean.py``:

* ``E_GCL(input_nf, output_nf, hidden_nf, edges_in_d=0, act_fn=nn.SiLU(),
  residual=True, attention=False, normalize=False, coords_agg='mean',
  tanh=False)`` (egnn_clean.py:11) with
  ``forward(h, edge_index, coord, edge_attr=None, node_attr=None) ->
  (h, coord, edge_attr)`` (egnn_clean.py:95-103).
* ``EGNN(in_node_nf, hidden_nf, out_node_nf, in_edge_nf=0, device='cpu',
  act_fn=nn.SiLU(), n_layers=4, residual=True, attention=False,
  normalize=False, tanh=False)`` (egnn_clean.py:107) with
  ``forward(h, x, edges, edge_attr) -> (h, x)`` (egnn_clean.py:141-146).

``edges`` / ``edge_index`` may be a :class:`~pymolecular_b200.csr.CSR` or the
reference's ``[row, col]`` pair (converted once, on the GPU, by a stable sort).
Parameters keep the reference ``state_dict`` names, so checkpoints move both
ways.  One extra keyword, ``precision='fp32' | 'bf16'``, selects fp32 GEMMs
(default) or bf16 GEMM inputs with fp32 accumulation.

``E_GCL`` takes any ``input_nf`` / ``output_nf`` next to ``hidden_nf`` (as
the reference constructor does; ``EGNN`` builds every layer with all three
equal, egnn_clean.py:136).

Differences that raise instead of silently diverging:
``act_fn`` other than SiLU, ``residual=True`` with ``input_nf != output_nf``
(the reference's ``h + out`` fails on the shapes, or broadcasts when one of
them is 1; here it always raises, NotImplementedError being a RuntimeError),
``node_attr`` (the reference node_mlp width ignores it, egnn_clean.py:29 vs
:63-64), CPU tensors.
"""
from __future__ import annotations

import ctypes as C

import torch
from torch import nn

from . import _native as nat
from .csr import CSR, as_csr

_PARAM_ORDER = ["edge_mlp.0.weight", "edge_mlp.0.bias", "edge_mlp.2.weight", "edge_mlp.2.bias",
                "node_mlp.0.weight", "node_mlp.0.bias", "node_mlp.2.weight", "node_mlp.2.bias",
                "coord_mlp.0.weight", "coord_mlp.0.bias", "coord_mlp.2.weight"]
_ATT_ORDER = ["att_mlp.0.weight", "att_mlp.0.bias"]   # appended when attention=True

_PRECISIONS = {"fp32": nat.PREC_FP32, "bf16": nat.PREC_BF16}


def _check_tensor(t: torch.Tensor, name: str) -> torch.Tensor:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (pymolecular_b200 has no CPU path)")
    if t.dtype != torch.float32:
        raise TypeError(f"{name} must be float32, got {t.dtype}")
    return t.contiguous()


def _ptrs(tensors):
    """Device pointers in egnn_layer_params field order; the att_* fields stay
    NULL when the layer has no attention gate."""
    ptrs = [nat.ptr(t) for t in tensors]
    return ptrs + [None] * (len(_PARAM_ORDER) + len(_ATT_ORDER) - len(ptrs))


class _LayerFn(torch.autograd.Function):
    """One E_GCL forward/backward through egnn_layer_fwd / egnn_layer_bwd."""

    @staticmethod
    def forward(ctx, h, x, edge_attr, csr: CSR, cfg, *params):
        flags, precision, d, H, O = cfg
        N, I = h.shape
        desc = nat.LayerDesc(N, csr.n_edges, H, d, flags, precision, I, O)
        lib = nat.lib()
        h_out = torch.empty(N, O, dtype=torch.float32, device=h.device)
        x_out = torch.empty_like(x)
        saved = torch.empty(max(lib.egnn_saved_size(C.byref(desc)) // 4, 1), dtype=torch.float32,
                            device=h.device)
        ws_bytes = lib.egnn_workspace_size(C.byref(desc), nat.WS_FWD, 0)
        ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=h.device)
        p = nat.LayerParams(*_ptrs(params))
        nat.check(lib.egnn_layer_fwd(C.byref(desc), C.byref(csr.struct()), C.byref(p), nat.ptr(h),
                                     nat.ptr(x), nat.ptr(edge_attr), nat.ptr(h_out), nat.ptr(x_out),
                                     nat.ptr(saved), nat.ptr(ws), ws_bytes, nat.stream_ptr()),
                  "egnn_layer_fwd")
        ctx.csr = csr
        ctx.cfg = cfg
        ctx.has_attr = edge_attr is not None
        ctx.save_for_backward(h, x, edge_attr if edge_attr is not None else h.new_empty(0), saved,
                              *params)
        return h_out, x_out

    @staticmethod
    def backward(ctx, gh, gx):
        h, x, edge_attr, saved, *params = ctx.saved_tensors
        if not ctx.has_attr:
            edge_attr = None
        flags, precision, d, H, O = ctx.cfg
        csr = ctx.csr
        N, I = h.shape
        gh = h.new_zeros(N, O) if gh is None else gh.contiguous().float()
        gx = torch.zeros_like(x) if gx is None else gx.contiguous().float()
        desc = nat.LayerDesc(N, csr.n_edges, H, d, flags, precision, I, O)
        lib = nat.lib()
        grad_h = torch.empty_like(h)
        grad_x = torch.empty_like(x)
        grads = [torch.empty_like(t) for t in params]
        ws_bytes = lib.egnn_workspace_size(C.byref(desc), nat.WS_BWD, 0)
        ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=h.device)
        p = nat.LayerParams(*_ptrs(params))
        gp = nat.LayerGrads(*_ptrs(grads))
        nat.check(lib.egnn_layer_bwd(C.byref(desc), C.byref(csr.struct()), C.byref(p), nat.ptr(h),
                                     nat.ptr(x), nat.ptr(edge_attr), nat.ptr(saved), nat.ptr(gh),
                                     nat.ptr(gx), nat.ptr(grad_h), nat.ptr(grad_x), C.byref(gp),
                                     nat.ptr(ws), ws_bytes, nat.stream_ptr()), "egnn_layer_bwd")
        return (grad_h, grad_x, None, None, None, *grads)


class _LinearFn(torch.autograd.Function):
    """y = x W^T + b through egnn_linear_fwd / egnn_linear_bwd."""

    @staticmethod
    def forward(ctx, x, w, b):
        M, K = x.shape
        O = w.shape[0]
        y = torch.empty(M, O, dtype=torch.float32, device=x.device)
        nat.check(nat.lib().egnn_linear_fwd(M, K, O, nat.ptr(x), nat.ptr(w), nat.ptr(b), nat.ptr(y),
                                            nat.stream_ptr()), "egnn_linear_fwd")
        ctx.save_for_backward(x, w)
        ctx.has_bias = b is not None
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w = ctx.saved_tensors
        M, K = x.shape
        O = w.shape[0]
        dy = dy.contiguous().float()
        dx = torch.empty_like(x) if ctx.needs_input_grad[0] else None
        dw = torch.empty_like(w)
        db = torch.empty(O, dtype=torch.float32, device=x.device) if ctx.has_bias else None
        lib = nat.lib()
        ws_bytes = lib.egnn_linear_workspace_size(M, K, O)
        ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=x.device)
        nat.check(lib.egnn_linear_bwd(M, K, O, nat.ptr(x), nat.ptr(w), nat.ptr(dy), nat.ptr(dx),
                                      nat.ptr(dw), nat.ptr(db), nat.ptr(ws), ws_bytes,
                                      nat.stream_ptr()), "egnn_linear_bwd")
        return dx, dw, db


def linear(x: torch.Tensor, layer: nn.Linear) -> torch.Tensor:
    """nn.Linear forward on the library's node GEMM."""
    x = _check_tensor(x, "input")
    return _LinearFn.apply(x, layer.weight, layer.bias)


class E_GCL(nn.Module):
    """E(n)-equivariant graph convolution layer (egnn_clean.py:5-103)."""

    def __init__(self, input_nf, output_nf, hidden_nf, edges_in_d=0, act_fn=nn.SiLU(), residual=True,
                 attention=False, normalize=False, coords_agg='mean', tanh=False,
                 precision: str = "fp32"):
        super().__init__()
        if not isinstance(act_fn, nn.SiLU):
            raise NotImplementedError("only act_fn=nn.SiLU() is built (the reference default)")
        if coords_agg not in ("mean", "sum"):
            raise Exception('Wrong coords_agg parameter %s' % coords_agg)
        if precision not in _PRECISIONS:
            raise ValueError(f"precision must be one of {sorted(_PRECISIONS)}")
        input_edge = input_nf * 2
        self.input_nf, self.output_nf, self.hidden_nf = input_nf, output_nf, hidden_nf
        self.residual = residual
        self.attention = attention
        self.normalize = normalize
        self.coords_agg = coords_agg
        self.tanh = tanh
        self.epsilon = 1e-8
        self.precision = precision
        self.edges_in_d = edges_in_d
        edge_coords_nf = 1
        # Same submodules, created in the same order as the reference, so a
        # seeded construction draws the same initial weights.
        self.edge_mlp = nn.Sequential(
            nn.Linear(input_edge + edge_coords_nf + edges_in_d, hidden_nf), act_fn,
            nn.Linear(hidden_nf, hidden_nf), act_fn)
        self.node_mlp = nn.Sequential(
            nn.Linear(hidden_nf + input_nf, hidden_nf), act_fn,
            nn.Linear(hidden_nf, output_nf))
        layer = nn.Linear(hidden_nf, 1, bias=False)
        torch.nn.init.xavier_uniform_(layer.weight, gain=0.001)
        coord_mlp = [nn.Linear(hidden_nf, hidden_nf), act_fn, layer]
        if self.tanh:
            coord_mlp.append(nn.Tanh())
        self.coord_mlp = nn.Sequential(*coord_mlp)
        if self.attention:
            self.att_mlp = nn.Sequential(nn.Linear(hidden_nf, 1), nn.Sigmoid())

    def _flags(self) -> int:
        f = 0
        if self.residual:
            f |= nat.FLAG_RESIDUAL
        if self.attention:
            f |= nat.FLAG_ATTENTION
        if self.normalize:
            f |= nat.FLAG_NORMALIZE
        if self.tanh:
            f |= nat.FLAG_TANH
        if self.coords_agg == "sum":
            f |= nat.FLAG_COORDS_SUM
        return f

    def _params(self):
        sd = dict(self.named_parameters())
        return [sd[k] for k in _PARAM_ORDER + (_ATT_ORDER if self.attention else [])]

    def forward(self, h, edge_index, coord, edge_attr=None, node_attr=None):
        if node_attr is not None:
            raise NotImplementedError("node_attr is not supported (the reference node_mlp input "
                                      "width does not include it, egnn_clean.py:29, 63-64)")
        if self.residual and self.input_nf != self.output_nf:
            raise NotImplementedError(f"residual=True needs input_nf == output_nf (got {self.input_nf}, "
                                      f"{self.output_nf}): the residual adds h to the node MLP output "
                                      "(egnn_clean.py:68-69)")
        h = _check_tensor(h, "h")
        coord = _check_tensor(coord, "coord")
        if coord.dim() != 2 or coord.shape[1] != 3:
            raise ValueError("coord must be (N, 3)")
        if h.dim() != 2 or h.shape[1] != self.input_nf:
            raise ValueError(f"h must be (N, {self.input_nf})")
        csr = as_csr(edge_index, h.shape[0], h.device)
        d = self.edges_in_d
        if d == 0 and edge_attr is not None:
            raise ValueError("edge_attr given but the layer was built with edges_in_d=0")
        if d > 0:
            if edge_attr is None:
                raise ValueError(f"layer expects edge_attr with {d} features")
            edge_attr = _check_tensor(edge_attr, "edge_attr")
            if edge_attr.shape != (csr.n_edges, d):
                raise ValueError(f"edge_attr must be ({csr.n_edges}, {d})")
        cfg = (self._flags(), _PRECISIONS[self.precision], d, self.hidden_nf, self.output_nf)
        h_out, x_out = _LayerFn.apply(h, coord, edge_attr, csr, cfg, *self._params())
        return h_out, x_out, edge_attr


class EGNN(nn.Module):
    """EGNN model (egnn_clean.py:106-146): embedding_in, n_layers E_GCL, embedding_out."""

    def __init__(self, in_node_nf, hidden_nf, out_node_nf, in_edge_nf=0, device='cpu',
                 act_fn=nn.SiLU(), n_layers=4, residual=True, attention=False, normalize=False,
                 tanh=False, precision: str = "fp32"):
        super().__init__()
        self.hidden_nf = hidden_nf
        self.device = device
        self.n_layers = n_layers
        self.embedding_in = nn.Linear(in_node_nf, self.hidden_nf)
        self.embedding_out = nn.Linear(self.hidden_nf, out_node_nf)
        for i in range(0, n_layers):
            self.add_module("gcl_%d" % i, E_GCL(self.hidden_nf, self.hidden_nf, self.hidden_nf,
                                                edges_in_d=in_edge_nf, act_fn=act_fn,
                                                residual=residual, attention=attention,
                                                normalize=normalize, tanh=tanh,
                                                precision=precision))
        self.to(self.device)

    @property
    def precision(self) -> str:
        return self._modules["gcl_0"].precision if self.n_layers else "fp32"

    @precision.setter
    def precision(self, value: str) -> None:
        for i in range(self.n_layers):
            self._modules["gcl_%d" % i].precision = value

    def forward(self, h, x, edges, edge_attr=None):
        h = _check_tensor(h, "h")
        csr = as_csr(edges, h.shape[0], h.device)
        h = linear(h, self.embedding_in)
        for i in range(0, self.n_layers):
            h, x, _ = self._modules["gcl_%d" % i](h, csr, x, edge_attr=edge_attr)
        h = linear(h, self.embedding_out)
        return h, x


__all__ = ["E_GCL", "EGNN", "CSR", "linear"]
