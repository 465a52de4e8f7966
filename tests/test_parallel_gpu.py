"""The node-partitioned EGNN on two GPUs (NCCL) against one GPU.

One kNN point cloud is split into two Morton-ordered node ranges; each rank
runs `partitioned_forward` (halo rows of h and x fetched before every layer,
edges into owned rows only) and the backward, and the parameter gradients
are summed over the ranks.  Each rank also runs the whole graph alone on its
own GPU with the same weights; the owned rows of the outputs, the input
gradients of the owned rows and the summed parameter gradients must agree.

fp32 mode: every owned row sees the same edges in the same order, so the
forward agrees to float32 rounding (2e-5 relative);
the gradients add per-rank partial sums in another order (1e-4).
bf16 mode: the halo rows of h cross the wire in bf16, so the owned rows next
to a cut see their neighbours' features rounded once more; the results stay
within the bf16 tolerance of the single-GPU run.

Needs two GPUs; skipped otherwise.  Ranks are spawned processes with a short
process-group timeout, NVLS off and a bounded wait in the parent.
"""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

N_NODES = 12288


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rel(a, b):
    a, b = a.detach().double().cpu(), b.detach().double().cpu()
    den = b.abs().max().item()
    return (a - b).abs().max().item() / (den if den > 0 else 1.0)


def _worker(rank, world, precision):
    import torch.distributed as dist
    from pymolecular_b200 import CSR, EGNN, parallel
    from pymolecular_b200.datasets import CONFIGS, make_workload

    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    mc = CONFIGS[5]
    b = make_workload(5, seed=3, n_nodes=N_NODES)
    torch.manual_seed(0)
    model = EGNN(mc.in_node_nf, mc.hidden_nf, mc.out_node_nf, n_layers=mc.n_layers, device=dev,
                 precision=precision)
    params = list(model.parameters())
    g = torch.Generator().manual_seed(11)
    w_out = torch.randn(b.n_nodes, mc.out_node_nf, generator=g).to(dev)
    w_x = torch.randn(b.n_nodes, 3, generator=g).to(dev)

    # the whole graph on this GPU alone
    h = b.h.to(dev).requires_grad_(True)
    x = b.x.to(dev).requires_grad_(True)
    ho, xo = model(h, x, CSR.from_edges(b.row, b.col, n_nodes=b.n_nodes, device=dev))
    ((ho * w_out).sum() + (xo * w_x).sum()).backward()
    ref_grads = [p.grad.clone() for p in params]
    for p in params:
        p.grad = None

    # this rank's node range
    plan = parallel.build_halo_plan(b.row, b.col, b.n_nodes, rank, world).to(dev)
    lo, hi = plan.own_lo, plan.own_hi
    assert plan.n_local > plan.n_own          # the cut really crosses edges
    csr = CSR.from_edges(plan.row, plan.col, n_nodes=plan.n_local, device=dev)
    h_own = b.h[lo:hi].to(dev).requires_grad_(True)
    x_own = b.x[lo:hi].to(dev).requires_grad_(True)
    po, px = parallel.partitioned_forward(model, h_own, x_own, csr, plan)
    ((po * w_out[lo:hi]).sum() + (px * w_x[lo:hi]).sum()).backward()
    parallel.GradAllReduce(params, average=False)()
    torch.cuda.synchronize(dev)

    fwd_tol, grad_tol = (2e-5, 1e-4) if precision == "fp32" else (2e-2, 2e-2)
    errs = {"h_out": _rel(po, ho[lo:hi]), "x_out": _rel(px, xo[lo:hi]),
            "dh": _rel(h_own.grad, h.grad[lo:hi]), "dx": _rel(x_own.grad, x.grad[lo:hi])}
    for name, p, r in zip([n for n, _ in model.named_parameters()], params, ref_grads):
        errs[name] = _rel(p.grad, r)
    bad = {k: v for k, v in errs.items()
           if v > (fwd_tol if k in ("h_out", "x_out") else grad_tol)}
    dist.barrier()                             # both ranks take the same collective steps
    assert not bad, (precision, bad)


def _entry(rank, world, port, precision, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    from datetime import timedelta
    import torch.distributed as dist
    try:
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
        _worker(rank, world, precision)
        q.put((True, ""))
    except Exception as exc:  # report to the parent instead of hanging it
        import traceback
        q.put((False, f"rank {rank}: {exc}\n{traceback.format_exc()}"))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


@pytest.mark.parametrize("precision", ["fp32", "bf16"])
def test_partitioned_two_gpus_match_one_gpu(precision):
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_entry, args=(r, world, port, precision, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        results = [q.get(timeout=300) for _ in range(world)]
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for ok, msg in results:
        assert ok, msg
