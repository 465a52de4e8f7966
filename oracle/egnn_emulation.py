"""Rounding-exact CPU model of the CUDA layer (TEST INFRASTRUCTURE ONLY).

The reference oracle (egnn_oracle.py) says what E_GCL computes; this module
says how the CUDA kernels round while computing it, so that a bf16-GEMM
result can be checked much tighter than against fp64 alone.  It follows the
same factored algorithm as the kernels (egnn_clean.py:49-103 restated with
W1 [h_i, h_j, r] = P_i + Q_j + w_r r) and rounds to bf16 exactly the GEMM
operands the kernels round in bf16 mode (edge_mlp.2.weight as a hi + lo
pair of bf16 values); accumulation is float64.  With
precision='fp32' nothing is rounded and it is a second fp64 restatement of
the layer's forward and hand-derived backward.
"""
from __future__ import annotations

import torch

from .egnn_oracle import segment_sum


def _bf(t, on):
    """Round to the bf16 grid (when `on`), keeping the dtype."""
    return t.to(torch.bfloat16).to(t.dtype) if on else t


def _split(t, on):
    """hi + lo with hi = bf16(t), lo = bf16(t - hi): the value a pair of bf16
    MMAs (x W_hi + x W_lo) multiplies by, about 16 significant bits."""
    if not on:
        return t
    hi = _bf(t, True)
    return hi + _bf(t - hi, True)


def _silu(a):
    s = torch.sigmoid(a)
    return a * s, s * (1 + a * (1 - s))


def layer_fwd_bwd(p, h, row, col, x, gh, gx, edge_attr=None, precision="bf16", residual=True,
                  attention=False, normalize=False, tanh=False, coords_agg="mean", backward=True):
    """(h', x', dL/dh, dL/dx, {param: grad}) with the kernels' rounding points
    (with backward=False: (h', x', None, None, {}))."""
    on = precision == "bf16"
    d = torch.float64
    h, x, gh, gx = h.to(d), x.to(d), gh.to(d), gx.to(d)
    p = {k: v.to(d) for k, v in p.items()}
    N, I = h.shape                      # I = input_nf
    W1 = p["edge_mlp.0.weight"]
    H = W1.shape[0]                     # hidden_nf
    Wa, Wb, wr = W1[:, :I], W1[:, I:2 * I], W1[:, 2 * I]
    We = W1[:, 2 * I + 1:]
    b1, W2, b2 = p["edge_mlp.0.bias"], p["edge_mlp.2.weight"], p["edge_mlp.2.bias"]
    Wn1, bn1, Wn2, bn2 = p["node_mlp.0.weight"], p["node_mlp.0.bias"], p["node_mlp.2.weight"], p["node_mlp.2.bias"]
    Wc1, bc1, wc2 = p["coord_mlp.0.weight"], p["coord_mlp.0.bias"], p["coord_mlp.2.weight"][0]
    deg = torch.bincount(row, minlength=N).to(d)
    scale = torch.ones(N, dtype=d, device=h.device) if coords_agg == "sum" else 1.0 / deg.clamp(min=1)

    # ---- forward
    P = h @ Wa.t() + b1
    Q = h @ Wb.t()
    dlt = x[row] - x[col]
    r = (dlt ** 2).sum(1)
    inv = 1.0 / (torch.sqrt(r) + 1e-8) if normalize else torch.ones_like(r)
    a1 = P[row] + Q[col] + wr * r[:, None]
    if edge_attr is not None and edge_attr.shape[1]:
        a1 = a1 + edge_attr.to(d) @ We.t()
    u1, s1 = _silu(a1)
    u1 = _bf(u1, on)
    # W2 enters every product as hi + lo (two bf16 MMAs): a plain bf16 W2 is
    # the same rounding on every edge, and that systematic error is what the
    # coordinate-MLP weight gradients (sums with heavy cancellation) amplify
    W2s = _split(W2, on)
    a2 = u1 @ W2s.t() + b2
    m, d2 = _silu(a2)
    if attention:
        # gate in full precision on the ungated message (egnn_clean.py:55-57)
        n = m
        wa, ba = p["att_mlp.0.weight"][0], p["att_mlp.0.bias"]
        at = torch.sigmoid(n @ wa + ba)
        m = n * at[:, None]
    mb = _bf(m, on)
    c1 = mb @ _bf(Wc1, on).t() + bc1
    v, dv = _silu(c1)
    phi = v @ wc2
    if tanh:
        phi = torch.tanh(phi)
    agg = segment_sum(m, row, N)
    x_out = x + segment_sum(dlt * inv[:, None] * phi[:, None], row, N) * scale[:, None]
    cat = torch.cat([h, agg], 1)
    n1pre = cat @ Wn1.t() + bn1
    n1, dn1 = _silu(n1pre)
    h_out = n1 @ Wn2.t() + bn2
    if residual:
        h_out = h_out + h
    if not backward:
        return h_out, x_out, None, None, {}

    # ---- backward
    g = {}
    g["node_mlp.2.weight"] = gh.t() @ n1
    g["node_mlp.2.bias"] = gh.sum(0)
    g_n1pre = (gh @ Wn2) * dn1
    g["node_mlp.0.weight"] = g_n1pre.t() @ cat
    g["node_mlp.0.bias"] = g_n1pre.sum(0)
    gh_acc = g_n1pre @ Wn1[:, :I] + (gh if residual else 0.0)
    g_agg = g_n1pre @ Wn1[:, I:]

    g_trans = gx[row] * scale[row][:, None]
    gphi = (g_trans * dlt).sum(1) * inv
    if tanh:
        gphi = gphi * (1 - phi ** 2)
    g_c1 = gphi[:, None] * wc2 * dv
    g["coord_mlp.2.weight"] = (gphi[:, None] * v).sum(0)[None, :]
    g["coord_mlp.0.bias"] = g_c1.sum(0)
    gc1b = _bf(g_c1, on)
    g["coord_mlp.0.weight"] = gc1b.t() @ mb
    g_m = gc1b @ _bf(Wc1, on) + g_agg[row]
    if attention:
        gs = (g_m * n).sum(1) * at * (1 - at)
        g["att_mlp.0.weight"] = (gs[:, None] * n).sum(0)[None, :]
        g["att_mlp.0.bias"] = gs.sum(0, keepdim=True)
        g_m = g_m * at[:, None] + gs[:, None] * wa
    g_a2 = g_m * d2
    g["edge_mlp.2.bias"] = g_a2.sum(0)
    ga2b = _bf(g_a2, on)
    g["edge_mlp.2.weight"] = ga2b.t() @ u1
    g_a1 = (ga2b @ W2s) * s1
    gr = g_a1 @ wr
    self_loop = (row == col).to(d)
    gdl = g_trans * (phi * inv * (1 - self_loop))[:, None] + 2 * gr[:, None] * dlt
    # the tensor-core paths (bf16, H = 128 fused edge kernels, H = 256 edge-row
    # GEMMs; no edge attributes, no attention) store g_a1 in bf16 for the
    # dst / src row sums (edge_tc.cu, edge_rows.cu); fp32 elsewhere
    tc_path = on and H in (128, 256) and (edge_attr is None or edge_attr.shape[1] == 0) and not attention
    g_a1s = _bf(g_a1, tc_path)
    S_dst = segment_sum(g_a1s, row, N)
    S_src = segment_sum(g_a1s, col, N)
    grad_x = gx + segment_sum(gdl, row, N) - segment_sum(gdl, col, N)
    grad_h = gh_acc + S_dst @ Wa + S_src @ Wb
    gW1 = torch.zeros_like(W1)
    gW1[:, :I] = S_dst.t() @ h
    gW1[:, I:2 * I] = S_src.t() @ h
    gW1[:, 2 * I] = (g_a1 * r[:, None]).sum(0)
    if edge_attr is not None and edge_attr.shape[1]:
        gW1[:, 2 * I + 1:] = g_a1.t() @ edge_attr.to(d)
    g["edge_mlp.0.weight"] = gW1
    g["edge_mlp.0.bias"] = S_dst.sum(0)
    return h_out, x_out, grad_h, grad_x, g


def model_fwd_bwd(p, h0, x0, row, col, graph_index, target, n_layers, precision="bf16", edge_attr=None,
                  **flags):
    """Whole EGNN step (embedding_in, L layers, embedding_out, graph-sum MSE)
    with the kernels' rounding points; the embeddings are fp32 node GEMMs.
    edge_attr: (E, d) per edge in the order of row / col, or None.

    Returns (loss, h_out, x_out, {param: grad}).
    """
    d = torch.float64
    p = {k: v.to(d) for k, v in p.items()}
    h = h0.to(d) @ p["embedding_in.weight"].t() + p["embedding_in.bias"]
    x = x0.to(d)
    ins = []
    for i in range(n_layers):
        pre = f"gcl_{i}."
        lp = {k[len(pre):]: v for k, v in p.items() if k.startswith(pre)}
        ins.append((h, x, lp))
        h, x, _, _, _ = layer_fwd_bwd(lp, h, row, col, x, h, x, edge_attr, precision=precision, backward=False,
                                      **flags)
    h_last = h
    out = h_last @ p["embedding_out.weight"].t() + p["embedding_out.bias"]
    G = target.shape[0]
    pred = segment_sum(out, graph_index, G)[:, 0]
    diff = pred - target.to(d)
    loss = (diff ** 2).mean()
    g_out = (2.0 * diff / G)[graph_index][:, None]
    grads = {"embedding_out.weight": g_out.t() @ h_last, "embedding_out.bias": g_out.sum(0)}
    gh = g_out @ p["embedding_out.weight"]
    gx = torch.zeros_like(x)
    for i in reversed(range(n_layers)):
        hi, xi, lp = ins[i]
        _, _, gh, gx, lg = layer_fwd_bwd(lp, hi, row, col, xi, gh, gx, edge_attr, precision=precision, **flags)
        grads.update({f"gcl_{i}.{k}": v for k, v in lg.items()})
    grads["embedding_in.weight"] = gh.t() @ h0.to(d)
    grads["embedding_in.bias"] = gh.sum(0)
    return loss, out, x, grads
