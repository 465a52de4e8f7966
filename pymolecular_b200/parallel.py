"""Multi-GPU training for the EGNN layer: one process per GPU.

Two decompositions:

* Graph-batch data parallelism (batches of independent graphs): every rank
  steps its own graphs; gradients are summed with one all-reduce of a flat
  fp32 buffer (NCCL over NVLink on GPUs, gloo in the CPU tests).
  ``partition_graphs`` balances graphs over ranks by edges + nodes
  (longest-processing-time greedy) when a fixed global batch is split.

* Node-range partitioning of one giant graph: nodes are ordered along a
  Morton curve and each rank owns a contiguous range and the CSR rows of its
  nodes.  Before every layer the rank fetches the rows of h and x of its
  "halo" (source nodes of its edges owned by other ranks); in the backward
  the gradients of those halo rows are returned to their owners and added
  there in fixed rank order (deterministic).  ``HaloPlan`` builds the
  exchange lists once; ``halo_exchange`` is the autograd-aware exchange.

The reference (models/EGNN/egnn_clean.py) is single-process; this module is
the multi-GPU layer the benchmark configurations ask for.
"""
from __future__ import annotations

import dataclasses
from typing import List, Sequence

import torch
import torch.distributed as dist


# ---------------------------------------------------------------------------
# data parallel
# ---------------------------------------------------------------------------

def partition_graphs(n_nodes: Sequence[int], n_edges: Sequence[int], world: int) -> List[List[int]]:
    """Assign graphs to ranks, balancing sum(E + N) (greedy LPT).

    Deterministic: graphs are taken by decreasing cost (ties by index) and
    each goes to the least-loaded rank (ties by rank).  Each rank's list is
    returned in increasing graph order.
    """
    cost = [int(e) + int(n) for n, e in zip(n_nodes, n_edges)]
    order = sorted(range(len(cost)), key=lambda g: (-cost[g], g))
    load = [0] * world
    parts: List[List[int]] = [[] for _ in range(world)]
    for g in order:
        r = min(range(world), key=lambda k: (load[k], k))
        parts[r].append(g)
        load[r] += cost[g]
    return [sorted(p) for p in parts]


def layer_buckets(names: Sequence[str]) -> List[List[int]]:
    """Group parameter indices into all-reduce buckets, one per module of
    the layer stack (the prefix before the first '.': ``embedding_in``,
    ``gcl_0`` ... ``gcl_{L-1}``, ``embedding_out``), ordered as the backward
    produces them: the last module first (egnn_clean.py:142-145 run in
    reverse)."""
    groups: dict = {}
    order: List[str] = []
    for i, n in enumerate(names):
        key = n.split(".")[0]
        if key not in groups:
            groups[key] = []
            order.append(key)
        groups[key].append(i)
    return [groups[k] for k in reversed(order)]


class GradAllReduce:
    """Sum (or average) the gradients of `params` over the process group.

    Gradients are reduced in buckets (``buckets``: lists of parameter
    indices; default one bucket for everything).  With ``overlap=True`` each
    parameter gets a post-accumulate-grad hook, and a bucket's all_reduce is
    issued (asynchronously) as soon as every one of its parameters has its
    gradient -- during the backward, while the earlier layers' backward runs
    on the compute stream.  Calling the object finishes the step: it issues
    the buckets that are still pending, waits for every reduction, averages,
    and makes every ``p.grad`` a view of its reduced bucket.

    Each bucket has two buffers used in turn: a step packs the local
    gradients into the buffer that the current ``p.grad`` views do not point
    into, so a gradient kept from the previous step (``zero_grad(set_to_none=
    False)``, or accumulation) is never reduced under autograd's feet.  The
    backward leaves fresh gradients in their own tensors (``zero_grad()`` sets
    them to None) and one concatenation packs a bucket.  A second backward
    before the call (gradient accumulation) re-packs and re-reduces the
    buckets it touched once their first reduction has finished, so the result
    is the reduced sum of everything accumulated.

    Every rank issues the same collectives in the same order: hooks fire in
    the backward's (deterministic) order and the pending buckets follow in
    bucket order.
    """

    def __init__(self, params, average: bool = True, group=None, buckets=None, overlap: bool = False):
        self.params = [p for p in params]
        self.average = average
        self.group = group
        self.buckets = buckets if buckets is not None else [list(range(len(self.params)))]
        dev = self.params[0].device if self.params else torch.device("cpu")
        self.bucket_of = [0] * len(self.params)
        self.flat = [[], []]                        # [side][bucket]
        self._views = [[None] * len(self.params), [None] * len(self.params)]
        for side in range(2):
            for b, idx in enumerate(self.buckets):
                buf = torch.zeros(sum(self.params[i].numel() for i in idx), dtype=torch.float32, device=dev)
                off = 0
                for i in idx:
                    n = self.params[i].numel()
                    self._views[side][i] = buf[off:off + n].view_as(self.params[i])
                    self.bucket_of[i] = b
                    off += n
                self.flat[side].append(buf)
        self.side = 0   # buffers this step packs into and reduces
        self._reset()
        self.overlap = overlap and self._active()
        if self.overlap:
            for i, p in enumerate(self.params):
                p.register_post_accumulate_grad_hook(self._hook(i))

    @property
    def views(self):
        """The views the gradients point at after the last call."""
        return self._views[1 - self.side]

    def _active(self) -> bool:
        return dist.is_initialized() and dist.get_world_size(self.group) > 1

    def _reset(self):
        self.ready = [set() for _ in self.buckets]
        self.work = [None] * len(self.buckets)
        self.dirty = [False] * len(self.buckets)

    def _hook(self, i):
        def hook(_p):
            b = self.bucket_of[i]
            if self.work[b] is not None:   # accumulated again after the bucket was issued
                self.dirty[b] = True
                return
            self.ready[b].add(i)
            if len(self.ready[b]) == len(self.buckets[b]):
                self._issue(b)
        return hook

    def _issue(self, b):
        idx = self.buckets[b]
        torch.cat([(self.params[i].grad if self.params[i].grad is not None
                    else torch.zeros_like(self.params[i])).reshape(-1) for i in idx], out=self.flat[self.side][b])
        self.work[b] = dist.all_reduce(self.flat[self.side][b], group=self.group, async_op=True)

    def zero_grad(self):
        for p in self.params:
            p.grad = None

    def __call__(self):
        if not self._active():
            return
        for b in range(len(self.buckets)):
            if self.work[b] is None:
                self._issue(b)
            elif self.dirty[b]:
                self.work[b].wait()
                self._issue(b)
        world = dist.get_world_size(self.group)
        for b in range(len(self.buckets)):
            self.work[b].wait()
            if self.average:
                self.flat[self.side][b].div_(world)
        for p, v in zip(self.params, self._views[self.side]):
            p.grad = v
        self.side ^= 1
        self._reset()


# ---------------------------------------------------------------------------
# node-range partitioning with halo exchange
# ---------------------------------------------------------------------------

def node_ranges(n_nodes: int, world: int) -> List[int]:
    """Contiguous, near-equal node ranges: rank r owns [b[r], b[r+1])."""
    return [(n_nodes * r) // world for r in range(world + 1)]


@dataclasses.dataclass
class HaloPlan:
    """Exchange lists of one rank for a node-range partition.

    own_lo, own_hi: owned global node range.
    halo: (n_halo,) global ids of the non-owned source nodes, grouped by owner
          rank in increasing rank order, increasing id inside a group;
          local index of halo k is n_own + k.
    recv_counts[p]: how many halo rows come from rank p.
    send_idx[p]: local (owned) row indices this rank sends to rank p.
    row, col: the local edge list (destination local ids in [0, n_own),
          source local ids in [0, n_own + n_halo)).
    """

    rank: int
    world: int
    own_lo: int
    own_hi: int
    halo: torch.Tensor
    recv_counts: List[int]
    send_idx: List[torch.Tensor]
    row: torch.Tensor
    col: torch.Tensor

    @property
    def n_own(self) -> int:
        return self.own_hi - self.own_lo

    @property
    def n_local(self) -> int:
        return self.n_own + int(self.halo.numel())

    @property
    def send_counts(self) -> List[int]:
        return [int(t.numel()) for t in self.send_idx]

    def to(self, device) -> "HaloPlan":
        """Keep the send lists on `device` (they index device rows every layer)."""
        self.send_idx = [t.to(device) for t in self.send_idx]
        return self


def local_edges(row: torch.Tensor, col: torch.Tensor, lo: int, hi: int):
    """Edges whose destination lies in [lo, hi), and their halo sources."""
    keep = (row >= lo) & (row < hi)
    r, c = row[keep], col[keep]
    outside = (c < lo) | (c >= hi)
    halo = torch.unique(c[outside])   # sorted ascending -> grouped by owner rank
    return r, c, halo


def build_halo_plan(row: torch.Tensor, col: torch.Tensor, n_nodes: int, rank: int, world: int,
                    group=None) -> HaloPlan:
    """Exchange plan for `rank`; every rank calls it (one all_to_all of counts
    and one of index lists).  `row`/`col` are the global edge list (CPU)."""
    b = node_ranges(n_nodes, world)
    lo, hi = b[rank], b[rank + 1]
    r, c, halo = local_edges(row, col, lo, hi)
    owner = torch.bucketize(halo, torch.tensor(b[1:-1], dtype=halo.dtype), right=True)
    recv_counts = [int((owner == p).sum()) for p in range(world)]
    # local ids: owned -> id - lo ; halo -> n_own + position in `halo`
    n_own = hi - lo
    pos = torch.searchsorted(halo, c)
    c_local = torch.where((c >= lo) & (c < hi), c - lo, n_own + pos)
    r_local = r - lo
    # tell every owner which of its nodes this rank needs
    send_idx = _exchange_requests(halo, recv_counts, b, rank, world, group)
    return HaloPlan(rank, world, lo, hi, halo, recv_counts, send_idx, r_local.long(), c_local.long())


def _exchange_requests(halo, recv_counts, b, rank, world, group):
    if world == 1:
        return [torch.zeros(0, dtype=torch.long)]
    dev = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend(group) == "nccl" \
        else torch.device("cpu")
    counts_out = torch.tensor(recv_counts, dtype=torch.long, device=dev)
    counts_in = torch.empty_like(counts_out)
    dist.all_to_all_single(counts_in, counts_out, group=group)
    reqs = halo.to(dev)
    got = torch.empty(int(counts_in.sum()), dtype=torch.long, device=dev)
    dist.all_to_all_single(got, reqs, output_split_sizes=counts_in.tolist(),
                           input_split_sizes=recv_counts, group=group)
    got = got.cpu() - b[rank]
    out, off = [], 0
    for p in range(world):
        n = int(counts_in[p])
        out.append(got[off:off + n].clone())
        off += n
    return out


class _HaloExchange(torch.autograd.Function):
    """[h_own] -> [h_own; h_halo] with h_halo fetched from the owners.

    Backward: the gradient rows of the halo are sent back and added to the
    owners' rows, summed in increasing source-rank order."""

    @staticmethod
    def forward(ctx, h_own, plan: HaloPlan, group, wire_dtype=None):
        ctx.plan, ctx.group = plan, group
        send = [h_own[idx] if idx.device == h_own.device else h_own[idx.to(h_own.device)]
                for idx in plan.send_idx]
        like = h_own
        if wire_dtype is not None and wire_dtype != h_own.dtype:
            # rows cross the wire rounded to wire_dtype (bf16 halves the bytes of h)
            send = [t.to(wire_dtype) for t in send]
            like = h_own[:0].to(wire_dtype)
        recv = _all_to_all_rows(send, plan.recv_counts, like, group).to(h_own.dtype)
        return torch.cat([h_own, recv], dim=0)

    @staticmethod
    def backward(ctx, g):
        plan, group = ctx.plan, ctx.group
        g = g.contiguous()
        g_own = g[:plan.n_own].clone()
        g_halo = g[plan.n_own:]
        # rows destined to each owner, in the order the owner sent them
        send, off = [], 0
        for p in range(plan.world):
            n = plan.recv_counts[p]
            send.append(g_halo[off:off + n])
            off += n
        back = _all_to_all_rows(send, plan.send_counts, g_own, group)
        off = 0
        for p in range(plan.world):
            n = plan.send_counts[p]
            if n:
                g_own.index_add_(0, plan.send_idx[p].to(g.device, non_blocking=True), back[off:off + n])
            off += n
        return g_own, None, None, None


def _all_to_all_rows(send: List[torch.Tensor], recv_counts: List[int], like: torch.Tensor, group):
    """Row all-to-all: send[p] goes to rank p; returns rows from ranks 0..P-1 concatenated."""
    world = len(send)
    width = like.shape[1:]
    if world == 1:
        return like.new_zeros((0, *width))
    out = like.new_empty((sum(recv_counts), *width))
    inp = torch.cat([s.reshape(-1, *width) for s in send], dim=0) if send else like.new_zeros((0, *width))
    dist.all_to_all_single(out, inp.contiguous(), output_split_sizes=recv_counts,
                           input_split_sizes=[int(s.shape[0]) for s in send], group=group)
    return out


def halo_exchange(h_own: torch.Tensor, plan: HaloPlan, group=None, wire_dtype=None) -> torch.Tensor:
    """Autograd-aware halo fetch: returns (n_own + n_halo, F) rows.  With
    `wire_dtype` (e.g. torch.bfloat16) the halo rows are sent in that type and
    arrive rounded to it; their gradients return in the rows' own type."""
    if plan.world == 1:
        return h_own
    return _HaloExchange.apply(h_own, plan, group, wire_dtype)


__all__ = ["partition_graphs", "layer_buckets", "GradAllReduce", "node_ranges", "HaloPlan", "build_halo_plan",
           "halo_exchange", "local_edges"]


def partitioned_forward(model, h_own: torch.Tensor, x_own: torch.Tensor, csr_local, plan: HaloPlan,
                        group=None):
    """EGNN.forward (egnn_clean.py:141-146) on one rank of a node partition.

    embedding_in on the owned rows; before every layer the halo rows of h
    and x are fetched; each layer runs on the local graph (owned rows plus
    halo rows, edges into owned rows only) and keeps its owned rows;
    embedding_out on the owned rows.  In bf16-GEMM mode the halo rows of h
    travel as bf16 (the coordinates and all gradients stay fp32).  Returns
    (h_out_own, x_out_own)."""
    from .egnn import linear
    n_own = plan.n_own
    h = linear(h_own, model.embedding_in)
    x = x_own
    wire = torch.bfloat16 if getattr(model, "precision", "fp32") == "bf16" else None
    for i in range(model.n_layers):
        h_loc = halo_exchange(h, plan, group, wire_dtype=wire)
        x_loc = halo_exchange(x, plan, group)
        h_loc, x_loc, _ = model._modules["gcl_%d" % i](h_loc, csr_local, x_loc)
        h, x = h_loc[:n_own], x_loc[:n_own]
    return linear(h.contiguous(), model.embedding_out), x


def global_sum(t: torch.Tensor, group=None) -> torch.Tensor:
    """Sum of `t` over all ranks in the forward; the gradient flows to the
    local term only (each rank back-propagates its own share)."""
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return t
    tot = t.detach().clone()
    dist.all_reduce(tot, group=group)
    return t + (tot - t.detach())


__all__ += ["partitioned_forward", "global_sum"]
