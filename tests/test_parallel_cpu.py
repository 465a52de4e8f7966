"""Multi-process logic on CPU ranks (gloo, world_size 2): graph partitioning,
gradient all-reduce, and the node-range halo exchange checked end to end
against the single-process oracle."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import egnn_oracle as O
from pymolecular_b200 import parallel as P


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _run(world, fn, *args):
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_entry, args=(r, world, port, fn, q, args)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=240) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for ok, msg in results:
        assert ok, msg
    return results


def _entry(rank, world, port, fn, q, args):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
        fn(rank, world, *args)
        dist.barrier()
        q.put((True, ""))
    except Exception as exc:  # report to the parent instead of hanging it
        import traceback
        q.put((False, f"rank {rank}: {exc}\n{traceback.format_exc()}"))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def test_partition_graphs_balanced_and_deterministic():
    g = torch.Generator().manual_seed(0)
    n = torch.randint(9, 30, (512,), generator=g).tolist()
    e = [k * (k - 1) for k in n]
    parts = P.partition_graphs(n, e, 8)
    assert sorted(sum(parts, [])) == list(range(512))
    loads = [sum(n[i] + e[i] for i in p) for p in parts]
    assert max(loads) / min(loads) < 1.01
    assert parts == P.partition_graphs(n, e, 8)


def test_node_ranges_cover():
    b = P.node_ranges(1000, 3)
    assert b[0] == 0 and b[-1] == 1000 and all(b[i] <= b[i + 1] for i in range(3))


def _grad_allreduce_worker(rank, world):
    torch.manual_seed(0)
    lin = torch.nn.Linear(4, 3)
    sync = P.GradAllReduce(lin.parameters())
    for bound in (False, True):   # gradients as fresh tensors, then as views of the flat buffer
        if bound:
            sync.zero_grad()
        else:
            lin.zero_grad(set_to_none=True)
        x = torch.full((2, 4), float(rank + 1))
        lin(x).sum().backward()
        expect = torch.full((3, 4), 2.0 * (1 + 2) / 2)   # mean over ranks of 2*(rank+1)
        sync()
        assert torch.allclose(lin.weight.grad, expect)
        assert torch.allclose(lin.bias.grad, torch.full((3,), 2.0))
        assert lin.weight.grad.data_ptr() == sync.views[0].data_ptr()


def test_grad_allreduce_two_ranks():
    _run(2, _grad_allreduce_worker)


class _Stack(torch.nn.Module):
    """Three modules named like the EGNN stack (embedding_in, gcl_0, embedding_out)."""

    def __init__(self):
        super().__init__()
        self.embedding_in = torch.nn.Linear(4, 6)
        self.gcl_0 = torch.nn.Sequential(torch.nn.Linear(6, 6), torch.nn.SiLU(), torch.nn.Linear(6, 6))
        self.embedding_out = torch.nn.Linear(6, 1)

    def forward(self, x):
        return self.embedding_out(self.gcl_0(self.embedding_in(x)))


def _bucket_worker(rank, world, overlap):
    """Per-module buckets (issued from the backward's hooks with overlap)
    give the same averaged gradients as one flat all-reduce; gradients kept
    in the buckets between steps (zero_grad(set_to_none=False)) and two
    backwards accumulated before one call are reduced in full."""
    torch.manual_seed(0)
    m = _Stack()
    names = [n for n, _ in m.named_parameters()]
    buckets = P.layer_buckets(names)
    assert [names[b[0]].split(".")[0] for b in buckets] == ["embedding_out", "gcl_0", "embedding_in"]
    sync = P.GradAllReduce(m.parameters(), buckets=buckets, overlap=overlap)
    x = [torch.randn(5, 4, generator=torch.Generator().manual_seed(10 * r + k)) for r in range(world)
         for k in range(2)]

    def expected(ks):
        # mean over ranks of the sum over the accumulated backwards
        ref = _Stack()
        ref.load_state_dict(m.state_dict())
        for r in range(world):
            for k in ks:
                ref(x[2 * r + k]).pow(2).sum().backward()
        return [p.grad / world for p in ref.parameters()]

    # step 1: fresh gradients
    sync.zero_grad()
    m(x[2 * rank]).pow(2).sum().backward()
    sync()
    for g, e in zip([p.grad for p in m.parameters()], expected([0])):
        assert torch.allclose(g, e, atol=1e-6), (g, e)
    # step 2: gradients stay in the buckets, zeroed in place; two backwards, one call
    m.zero_grad(set_to_none=False)
    m(x[2 * rank]).pow(2).sum().backward()
    m(x[2 * rank + 1]).pow(2).sum().backward()
    sync()
    for g, e in zip([p.grad for p in m.parameters()], expected([0, 1])):
        assert torch.allclose(g, e, atol=1e-6), (g, e)
    for p, v in zip(m.parameters(), sync.views):
        assert p.grad.data_ptr() == v.data_ptr()


@pytest.mark.parametrize("overlap", [False, True])
def test_bucketed_grad_allreduce_two_ranks(overlap):
    _run(2, _bucket_worker, overlap)


def _graph(seed, n=160, k=6):
    g = torch.Generator().manual_seed(seed)
    x = torch.rand(n, 3, generator=g, dtype=torch.float64) * 10
    d = torch.cdist(x, x) + torch.eye(n, dtype=torch.float64) * 1e9
    nbr = d.topk(k, largest=False).indices       # k nearest sources per destination
    row = torch.arange(n).repeat_interleave(k)
    col = nbr.reshape(-1)
    h = torch.randn(n, 16, generator=g, dtype=torch.float64)
    wh = torch.randn(n, 16, generator=g, dtype=torch.float64)
    wx = torch.randn(n, 3, generator=g, dtype=torch.float64)
    return row, col, x, h, wh, wx


def _halo_worker(rank, world, seed):
    row, col, x, h, wh, wx = _graph(seed)
    n = x.shape[0]
    params = O.init_params(16, 16, 1, 1, seed=seed, dtype=torch.float64)
    lp = {k[len("gcl_0."):]: v for k, v in params.items() if k.startswith("gcl_0.")}
    lp["coord_mlp.2.weight"] = lp["coord_mlp.2.weight"] * 300.0
    plan = P.build_halo_plan(row, col, n, rank, world)
    lo, hi = plan.own_lo, plan.own_hi
    leaf = {k: v.clone().requires_grad_(True) for k, v in lp.items()}
    h_own = h[lo:hi].clone().requires_grad_(True)
    x_own = x[lo:hi].clone().requires_grad_(True)
    h_loc = P.halo_exchange(h_own, plan)
    x_loc = P.halo_exchange(x_own, plan)
    ho, xo = O.e_gcl(leaf, "", h_loc, plan.row, plan.col, x_loc)
    loss = (ho[:plan.n_own] * wh[lo:hi]).sum() + (xo[:plan.n_own] * wx[lo:hi]).sum()
    loss.backward()
    grads = torch.cat([leaf[k].grad.reshape(-1) for k in sorted(leaf)])
    dist.all_reduce(grads)
    # single-process reference on the whole graph
    leaf2 = {k: v.clone().requires_grad_(True) for k, v in lp.items()}
    hh = h.clone().requires_grad_(True)
    xx = x.clone().requires_grad_(True)
    ho2, xo2 = O.e_gcl(leaf2, "", hh, row, col, xx)
    ((ho2 * wh).sum() + (xo2 * wx).sum()).backward()
    ref = torch.cat([leaf2[k].grad.reshape(-1) for k in sorted(leaf2)])
    assert torch.allclose(ho[:plan.n_own], ho2[lo:hi], atol=1e-12, rtol=0)
    assert torch.allclose(xo[:plan.n_own], xo2[lo:hi], atol=1e-12, rtol=0)
    assert torch.allclose(grads, ref, atol=1e-10, rtol=1e-10)
    assert torch.allclose(h_own.grad, hh.grad[lo:hi], atol=1e-10, rtol=1e-10)
    assert torch.allclose(x_own.grad, xx.grad[lo:hi], atol=1e-10, rtol=1e-10)
    assert plan.n_local > plan.n_own   # the partition really cuts edges


@pytest.mark.parametrize("world", [2, 3])
def test_halo_exchange_matches_single_process(world):
    _run(world, _halo_worker, 7)


def _global_sum_worker(rank, world):
    t = torch.tensor([float(rank + 1)], requires_grad=True)
    s = P.global_sum(t)
    assert float(s) == sum(range(1, world + 1))
    (s * 3.0).sum().backward()
    assert float(t.grad) == 3.0


def test_global_sum_gradient_stays_local():
    _run(2, _global_sum_worker)


def test_halo_plan_lists():
    row, col, *_ = _graph(3, n=90, k=4)
    # single-process plan views for two ranks built without a process group
    b = P.node_ranges(90, 2)
    r, c, halo = P.local_edges(row, col, b[0], b[1])
    assert torch.all((r >= b[0]) & (r < b[1]))
    assert torch.all((halo >= b[1]))
    assert torch.equal(halo, torch.unique(halo))


# ---------------------------------------------------------------------------
# failure detection on the host: a rank that dies, a collective that times out
# ---------------------------------------------------------------------------

def _failure_entry(rank, world, port, mode, q):
    import time
    from datetime import timedelta
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=4))
    t = torch.ones(16)
    dist.all_reduce(t)            # a healthy step first
    if rank == 1:
        if mode == "exit":
            q.put(("left", 0.0))
            q.close()
            q.join_thread()       # the message is out before the process dies
            os._exit(0)           # dies between steps, no collective in flight
        time.sleep(10)            # alive but never joins the next collective
        q.put(("slept", 0.0))
        return
    t0 = time.time()
    try:
        sync = P.GradAllReduce([torch.nn.Parameter(torch.zeros(4))])
        sync.params[0].grad = torch.ones(4)
        sync()
        q.put(("no error", time.time() - t0))
    except Exception as exc:      # the peer's absence surfaces as an error, not a hang
        q.put((type(exc).__name__, time.time() - t0))
    finally:
        q.close()
        q.join_thread()
        os._exit(0)               # no teardown handshake with a missing peer


@pytest.mark.parametrize("mode", ["exit", "stall"])
def test_missing_rank_surfaces_as_an_error(mode):
    """A gradient all-reduce whose peer has died (or never joins) ends with an
    exception on the surviving rank within the process-group timeout."""
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_failure_entry, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = [q.get(timeout=120) for _ in range(2)]
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    survivor = [g for g in got if g[0] not in ("left", "slept")]
    assert len(survivor) == 1, got
    name, elapsed = survivor[0]
    assert name != "no error", got
    assert elapsed < 60, got


def _wire_worker(rank, world):
    """Halo rows sent as bf16 arrive as the owners' rows rounded to bf16, and
    their gradients return to the owners in fp32."""
    row, col, x, h, _, _ = _graph(3)
    n = x.shape[0]
    plan = P.build_halo_plan(row, col, n, rank, world)
    lo, hi = plan.own_lo, plan.own_hi
    hf = h.float()
    h_own = hf[lo:hi].clone().requires_grad_(True)
    got = P.halo_exchange(h_own, plan, wire_dtype=torch.bfloat16)
    assert got.dtype == torch.float32
    assert torch.equal(got[:plan.n_own], hf[lo:hi])
    assert torch.equal(got[plan.n_own:], hf[plan.halo].bfloat16().float())
    w = torch.arange(got.numel(), dtype=torch.float32).reshape(got.shape)
    (got * w).sum().backward()
    assert h_own.grad.dtype == torch.float32 and torch.isfinite(h_own.grad).all()


def test_halo_rows_in_bf16_two_ranks():
    _run(2, _wire_worker)
