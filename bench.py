#!/usr/bin/env python
"""EGNN training-step benchmark (layer fwd+bwd edges/s, molecules/s).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 2] [--impl b200|reference]

One step = forward of the whole EGNN over one batch of synthetic graphs,
graph-sum MSE loss, backward, gradient all-reduce (N > 1) and an SGD update.
Default workload: config 2 (512 molecules, 7 layers, H=128, bf16 GEMM
inputs, fp32 accumulate).  Multi-GPU runs are graph-batch data parallel with
weak scaling: every rank steps its own 512-graph batch and the gradients are
summed with NCCL.  Prints ONE JSON line on rank 0.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

L2_BYTES = 126 * 1024 * 1024


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", type=int, default=2)
    ap.add_argument("--precision", default=None, help="override the config's GEMM precision")
    ap.add_argument("--n-graphs", type=int, default=None, help="shrink the batch (profiling runs)")
    ap.add_argument("--n-nodes", type=int, default=None, help="config 5: node count (default 2^20)")
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--allreduce", default="flat", choices=["layers", "flat"],
                    help="data parallel: one flat all-reduce after the backward (flat, measured equal or "
                         "faster at 2 and 8 GPUs) or per-layer buckets all-reduced as the backward "
                         "produces them (layers)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the fp32-mode and other-workload measurements of the default 1-GPU run")
    ap.add_argument("--no-graphs", action="store_true",
                    help="time eager steps instead of replays of the captured training step")
    ap.add_argument("--profile", action="store_true",
                    help="profiler target: 1 warm-up + --steps steps, no side passes, no JSON")
    return ap.parse_args()


# ---------------------------------------------------------------------------
# helpers
# ---------------------------------------------------------------------------

def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


class ClockSampler:
    """nvidia-smi clocks/throttle sampling while the benchmark runs."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = Path(os.environ.get("TMPDIR", "/tmp")) / f"egnn_clocks_{os.getpid()}.csv"

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in self.path.read_text().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                rows.append((float(f[1]), float(f[2]), float(f[3]) if f[3] not in ("[N/A]", "N/A") else 0.0,
                             f[4], f[5], f[6], f[7], f[8]))
            except ValueError:
                continue
        try:
            self.path.unlink()
        except OSError:
            pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        loaded = [r for r in rows if r[2] > 200.0] or rows
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in loaded:
            for n, v in zip(names, r[4:8]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(r[0] for r in loaded), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": sorted(reasons), "samples": len(loaded),
                "power_w_max": max(r[2] for r in rows)}


def ncu_traffic(config: int, kernel: str, edges: int):
    """DRAM bytes per launch measured by ncu for this kernel and workload
    (profiles/ncu_traffic.json), scaled to `edges` edges per launch; None if
    no capture covers it."""
    p = ROOT / "profiles" / "ncu_traffic.json"
    try:
        rec = json.loads(p.read_text())[f"config{config}"][kernel]
    except (OSError, KeyError, ValueError):
        return None
    return rec["bytes_per_launch"] * edges / rec["edges_per_launch"]


def model_flops(cfg, n_nodes, n_edges):
    """Credited (algorithmic) flops of one training step, factored EGNN count.

    Per layer: edges 12 H^2 (phi_e layer 2 and phi_x layer 1: forward, dgrad,
    wgrad), nodes 30 H^2 (P/Q projections and node MLP: forward, dgrad,
    wgrad).  Recompute is not credited.
    """
    H, L = cfg.hidden_nf, cfg.n_layers
    return L * (12 * H * H * n_edges + 30 * H * H * n_nodes)


# ---------------------------------------------------------------------------
# CPU reference arm: the oracle port of egnn_clean.EGNN on the host cores
# ---------------------------------------------------------------------------

def cpu_step_timer(cfg_id, n_graphs_sample, steps, warmup, threads):
    import torch
    from oracle import egnn_oracle as O
    from pymolecular_b200.datasets import CONFIGS, make_workload
    torch.set_num_threads(threads)
    mc = CONFIGS[cfg_id]
    if cfg_id == 5:
        # a block of config 5's point cloud: the same density (2^20 points in
        # a 200 A box) and 32 nearest neighbours per node
        from pymolecular_b200.datasets import point_cloud
        b = point_cloud(n_graphs_sample, box=200.0 * (n_graphs_sample / float(1 << 20)) ** (1.0 / 3.0), seed=0)
    else:
        b = make_workload(cfg_id, n_graphs=n_graphs_sample)
    p = O.init_params(mc.in_node_nf, mc.hidden_nf, mc.out_node_nf, mc.n_layers, seed=0)
    gi = b.graph_index()
    times = []
    for i in range(warmup + steps):
        t0 = time.perf_counter()
        O.model_grads(p, b.h, b.x, b.row, b.col, gi, b.target)
        if i >= warmup:
            times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    return {"layer_edges_per_s": mc.n_layers * b.n_edges / t, "molecules_per_s": b.n_graphs / t,
            "step_s": t, "edges": b.n_edges, "graphs": b.n_graphs, "nodes": b.n_nodes}


def cpu_sample_size(cfg_id):
    """Graphs (config-5: nodes) the CPU arm times: configs 1-2 whole; the
    seeded subsets of configs 3-5 whose fp32 intermediates fit the host."""
    return {1: 96, 2: 512, 3: 1, 4: 16, 5: 16384}[cfg_id]


def full_size(cfg_id):
    from pymolecular_b200.datasets import GRAPHS_PER_BATCH
    return GRAPHS_PER_BATCH[cfg_id] if cfg_id != 5 else 1 << 20


def run_reference(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return 0
    from pymolecular_b200.datasets import CONFIGS
    mc = CONFIGS[args.config]
    threads = os.cpu_count() or 1
    sample = cpu_sample_size(args.config)
    # a CPU step of the whole config 2 takes seconds: at most 10 timed steps
    # and one warm-up keep the arm within a few minutes
    steps, warmup = max(1, min(args.steps, 10)), max(1, min(args.warmup, 1))
    r = cpu_step_timer(args.config, sample, steps, warmup, threads)
    unit = "layer-edges/s"
    line = {
        "impl": "reference", "metric": "egnn_train_layer_edges_per_s", "value": r["layer_edges_per_s"],
        "unit": unit, "n_gpus": args.gpus, "steps": steps, "warmup": warmup,
        "steps_requested": args.steps, "warmup_requested": args.warmup,
        "ms_per_step": r["step_s"] * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded)",
        "config": {"workload": f"config{args.config}", "graphs": r["graphs"], "nodes": r["nodes"],
                   "edges": r["edges"], "layers": mc.n_layers, "hidden": mc.hidden_nf, "precision": "fp32",
                   "same_workload_as_b200_arm": sample == full_size(args.config)},
        "molecules_per_s": r["molecules_per_s"],
        "cpu_baseline": {"value": r["layer_edges_per_s"], "unit": unit, "cores": threads, "kind": "port",
                         "sample": f"{r['graphs']} graphs / {r['nodes']} nodes / {r['edges']} edges of "
                                   f"config{args.config}, fp32 oracle (egnn_clean restatement), median of "
                                   f"{steps} steps"},
        "e2e": {"value": r["layer_edges_per_s"], "unit": unit, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# B200 arm
# ---------------------------------------------------------------------------

class Problem:
    """One rank's share of the workload and its training step.

    Data-parallel configs (1-4): the rank steps its own seeded batch of graphs
    (weak scaling) and gradients are averaged with one NCCL all-reduce.
    Config 5 on N > 1 GPUs: the single graph is split into Morton-ordered node
    ranges with a halo exchange before every layer (strong scaling) and the
    gradients are summed.
    """

    def __init__(self, args, world, rank, dev):
        import torch
        from pymolecular_b200 import CSR, EGNN, graph_sum_mse, parallel
        from pymolecular_b200.datasets import CONFIGS, make_workload
        self.torch, self.parallel, self.CSR = torch, parallel, CSR
        self.graph_sum_mse = graph_sum_mse
        self.dev, self.world, self.rank = dev, world, rank
        self.cfg_id = args.config
        self.mc = mc = CONFIGS[args.config]
        self.precision = args.precision or mc.precision
        self.halo = args.config == 5 and world > 1
        if self.halo:
            b = make_workload(5, seed=0, n_nodes=args.n_nodes)
            self.plan = parallel.build_halo_plan(b.row, b.col, b.n_nodes, rank, world).to(dev)
            lo, hi = self.plan.own_lo, self.plan.own_hi
            self.h_host, self.x_host = b.h[lo:hi].contiguous(), b.x[lo:hi].contiguous()
            self.row_host, self.col_host = self.plan.row, self.plan.col
            self.n_nodes_csr = self.plan.n_local
            self.edges_job = b.n_edges
            self.graphs_job = 1
            self.target = b.target
            self.scaling = "strong"
        else:
            b = make_workload(args.config, seed=rank, n_graphs=args.n_graphs, n_nodes=args.n_nodes)
            self.h_host, self.x_host = b.h, b.x
            self.row_host, self.col_host = b.row, b.col
            self.n_nodes_csr = b.n_nodes
            self.edges_job = b.n_edges * world
            self.graphs_job = b.n_graphs * world
            self.graph_ptr = b.graph_ptr
            self.target = b.target
            self.scaling = "weak"
        self.batch = b
        self.edges_rank = int(self.row_host.numel())
        self.nodes_rank = int(self.h_host.shape[0])
        torch.manual_seed(0)
        self.model = EGNN(mc.in_node_nf, mc.hidden_nf, mc.out_node_nf, n_layers=mc.n_layers, device=dev,
                          precision=self.precision)
        self.params = list(self.model.parameters())
        self.opt = torch.optim.SGD(self.params, lr=1e-4)
        self.allreduce = "flat" if self.halo else args.allreduce
        names = [n for n, _ in self.model.named_parameters()]
        self.sync_grads = parallel.GradAllReduce(
            self.params, average=not self.halo,
            buckets=parallel.layer_buckets(names) if self.allreduce == "layers" else None,
            overlap=self.allreduce == "layers")
        self.csr = CSR.from_edges(self.row_host, self.col_host, n_nodes=self.n_nodes_csr, device=dev)
        self.h = self.h_host.to(dev)
        self.x = self.x_host.to(dev)
        self.tgt = self.target.to(dev)
        if not self.halo:
            self.gp = self.graph_ptr.to(dev)

    def loss(self, h_out, gp=None, tgt=None):
        torch = self.torch
        tgt = self.tgt if tgt is None else tgt
        if self.halo:
            pred = self.parallel.global_sum(h_out[:, 0].sum())
            return ((pred - tgt[0]) ** 2)
        # per-graph sums of the node outputs (graphs are contiguous node ranges)
        # and their MSE, forward and backward in the library's loss kernels
        return self.graph_sum_mse(h_out[:, 0], self.gp if gp is None else gp, tgt)

    def forward(self, h, x, csr):
        if self.halo:
            return self.parallel.partitioned_forward(self.model, h, x, csr, self.plan)
        return self.model(h, x, csr)

    def zero_grad(self):
        if self.world > 1:
            self.sync_grads.zero_grad()
        else:
            self.opt.zero_grad(set_to_none=True)

    def step(self):
        self.zero_grad()
        ho, _ = self.forward(self.h, self.x, self.csr)
        loss = self.loss(ho)
        loss.backward()
        self.sync_grads()
        self.opt.step()
        # detached: a captured step must not keep its autograd graph alive
        # past the capture (later eager steps would then accumulate into
        # nodes that belong to the capture stream)
        return loss.detach()

    def host_buffers(self):
        bufs = {"h": self.h_host.pin_memory(), "x": self.x_host.pin_memory(),
                "row": self.row_host.pin_memory(), "col": self.col_host.pin_memory(),
                "tgt": self.target.pin_memory()}
        if not self.halo:
            bufs["gp"] = self.graph_ptr.pin_memory()
        return bufs

    def e2e_step(self, host, loss_host, check=True):
        """Public-API step from pinned host tensors: H2D copies, CSR built on the
        device from the edge list, forward, loss, backward, update, loss D2H.
        check=False defers the edge-index validation to the device (the step
        can then be captured as a CUDA graph); the CSR is returned so that the
        caller can read its flag."""
        d = {k: v.to(self.dev, non_blocking=True) for k, v in host.items()}
        csr = self.CSR.from_edges(d["row"], d["col"], n_nodes=self.n_nodes_csr, device=self.dev, check=check)
        self.zero_grad()
        ho, _ = self.forward(d["h"], d["x"], csr)
        loss = self.loss(ho, d.get("gp"), d["tgt"])
        loss.backward()
        self.sync_grads()
        self.opt.step()
        loss_host.copy_(loss.detach().reshape(1), non_blocking=True)
        return csr


KERNELS = ("edge_bwd", "edge_fwd", "node_pass", "src_pass", "edge_fixup", "part_reduce", "node_gemm", "node_wgrad",
           "gemm_small",
           "linear_small", "wgrad_small", "colsum", "gemm_reduce", "prep", "edge_rows_gemm", "edge_rows_wgrad",
           "edge_rows_u", "edge_rows_agg", "edge_rows_wimg", "graph_mse")


def measure(prob, args, world, dev, steps, warmup, graphs=True, e2e=True):
    """Times `steps` training steps of `prob` (CUDA events, L2 flushed between
    steps, max over ranks), then a separate pass with the library's kernel
    timer, then (optionally) the end-to-end public-API step.  Returns a dict."""
    import torch
    import torch.distributed as dist
    from pymolecular_b200 import _native

    flush = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device=dev)
    for _ in range(warmup - 1):
        prob.step()
    torch.cuda.synchronize()
    _native.lib().egnn_launch_count_reset()
    prob.step()                      # last warm-up step: count this library's launches per step
    torch.cuda.synchronize()
    launches_per_step = int(_native.lib().egnn_launch_count())

    # The timed steps replay the whole training step (forward, backward, the
    # gradient all-reduce, SGD update) captured once as a CUDA graph; the
    # node-partitioned config (host-sized halo exchanges) runs eagerly.
    graphed = None
    run_step = prob.step
    if graphs and not prob.halo:
        from pymolecular_b200.graphs import GraphedStep
        graphed = GraphedStep(prob.step, warmup=1)
        run_step = graphed.replay
        run_step()                   # one untimed replay
        torch.cuda.synchronize()

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    for k in range(steps):
        flush.fill_(float(k))
        starts[k].record()
        run_step()
        ends[k].record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends))
    t = torch.tensor([ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_per_step = float(t.item()) / steps

    # live kernel timing (events around each launch on its own stream; a
    # separate eager pass, since it perturbs the step)
    _native.lib().egnn_kernel_timing(1)
    kt_steps = min(steps, 5)
    for k in range(kt_steps):
        flush.fill_(float(k))
        prob.step()
    torch.cuda.synchronize()
    ktimes = {n: _native.kernel_time(n) for n in KERNELS}
    _native.lib().egnn_kernel_timing(0)
    status = _native.lib().egnn_device_status(_native.stream_ptr())

    e2e_rec = None
    if e2e:
        e2e_rec = measure_e2e(prob, args, world, dev, steps, graphs)
    if graphed is not None:
        graphed.release()
    del flush
    return {"ms_per_step": ms_per_step, "launches": launches_per_step * steps, "ktimes": ktimes,
            "kt_steps": kt_steps, "status": status, "graphed": graphed is not None, "e2e": e2e_rec}


def measure_e2e(prob, args, world, dev, steps, graphs):
    """The same metric through the public API from pinned host buffers."""
    import torch
    import torch.distributed as dist
    mc = prob.mc
    host = prob.host_buffers()
    h2d = sum(v.numel() * v.element_size() for v in host.values())
    loss_host = torch.empty(1, dtype=torch.float32).pin_memory()

    def time_e2e(run):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            run()
        e1.record()
        torch.cuda.synchronize()
        te = torch.tensor([e0.elapsed_time(e1)], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        return float(te.item()) / steps

    def e2e_line(ms, path):
        return {"value": mc.n_layers * prob.edges_job / (ms * 1e-3), "unit": "layer-edges/s",
                "ms_per_step": ms, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4,
                "molecules_per_s": prob.graphs_job / (ms * 1e-3), "path": path}

    # eager: every call from Python, edge indices validated with a host read-back
    for _ in range(2):
        prob.e2e_step(host, loss_host)
    eager_ms = time_e2e(lambda: prob.e2e_step(host, loss_host))
    eager = e2e_line(eager_ms, "eager EGNN.forward(h, x, csr) per step: pinned H2D of h, x, edge list, "
                               "targets; CSR.from_edges on the device; backward; SGD; loss D2H")
    if not graphs or prob.halo:
        return eager
    # the same public-API step captured once with GraphedStep: each replay
    # copies the pinned host buffers in, builds the CSR (validation flag kept
    # on the device, read after the timed steps), runs the step and copies
    # the loss out
    from pymolecular_b200.graphs import GraphedStep
    holder = {}

    def captured():
        holder["csr"] = prob.e2e_step(host, loss_host, check=False)
        return None

    g_e2e = GraphedStep(captured, warmup=1)
    g_e2e.replay()
    torch.cuda.synchronize()
    graph_ms = time_e2e(g_e2e.replay)
    holder["csr"].raise_if_invalid()
    rec = e2e_line(graph_ms, "GraphedStep over the same public-API step (pinned H2D of h, x, edge list, "
                             "targets; CSR.from_edges(check=False) on the device; forward; backward; "
                             "SGD; loss D2H), replayed once per step")
    rec["eager"] = {k: eager[k] for k in ("value", "ms_per_step", "path")}
    g_e2e.release()
    return rec


def _per_step(ktimes, names, kt_steps):
    return sum(ktimes[n][0] for n in names) / kt_steps


def roofline(prob, m, peaks, clk, dev):
    """Roofline records of the kernel groups of one measured workload.

    Tensor-pipe groups: credited (algorithmic) flops, the factored EGNN
    count (recompute not credited), over the groups' CUDA-event time,
    against the measured sustained bf16 peak (bf16 mode) or the nominal FP32
    pipe (fp32 mode: FFMA kernels).  HBM groups: algorithmic bytes over time
    against the measured HBM bandwidth.  Returns (dominant, groups)."""
    import torch
    mc, kt, n = prob.mc, m["ktimes"], m["kt_steps"]
    H, L, E, N = mc.hidden_nf, mc.n_layers, prob.edges_rank, prob.nodes_rank
    bf = prob.precision == "bf16"
    props = torch.cuda.get_device_properties(dev)
    mhz = (clk or {}).get("sm_max_mhz") or 1965.0
    fp32_peak = props.multi_processor_count * 128 * 2 * mhz * 1e6 / 1e12
    tc_peak, hbm = peaks["bf16_tflops_sustained"], peaks["hbm_gbs"]
    groups = {}

    def tensor(name, flops_step, ms_step, launches, on_tc=True, extra=None):
        if ms_step <= 0:
            return
        ach = flops_step / (ms_step * 1e-3) / 1e12
        peak = tc_peak if on_tc else fp32_peak
        rec = {"bound": "tensor" if on_tc else "fp32_pipe", "achieved": ach, "peak": peak, "unit": "TFLOP/s",
               "frac": ach / peak, "peak_source": (f"{peaks['source']} bf16 sustained" if on_tc else
                                                   "nominal FP32 pipe (SMs x 128 lanes x 2 x max SM clock)"),
               "ms_per_step": ms_step, "launches_per_step": launches / n,
               "flops_per_launch": flops_step / max(launches / n, 1e-9)}
        rec.update(extra or {})
        groups[name] = rec

    def memory(name, bytes_step, ms_step, launches, note):
        if ms_step <= 0:
            return
        ach = bytes_step / (ms_step * 1e-3) / 1e9
        groups[name] = {"bound": "hbm", "achieved": ach, "peak": hbm, "unit": "GB/s", "frac": ach / hbm,
                        "peak_source": f"{peaks['source']} HBM copy", "ms_per_step": ms_step,
                        "launches_per_step": launches / n, "bytes_per_launch": bytes_step / max(launches / n, 1e-9),
                        "bytes": note}

    rows_path = bf and H == 256
    tc_edge = bf and H == 128 and "edge_bwd" in kt and kt["edge_bwd"][1] > 0
    # per-edge GEMMs: forward 4 H^2 per edge (phi_e layer 2, phi_x layer 1),
    # backward 8 H^2 (their data and weight gradients)
    if rows_path:
        ms = _per_step(kt, ["edge_rows_gemm"], n)
        tensor("edge_rows_gemm", 8.0 * H * H * E * L, ms, kt["edge_rows_gemm"][1],
               extra={"credited": "4 of the 6 launches per layer (the backward's recompute is not credited)"})
        ms = _per_step(kt, ["edge_rows_wgrad"], n)
        tensor("edge_rows_wgrad", 4.0 * H * H * E * L, ms, kt["edge_rows_wgrad"][1])
    else:
        tensor("edge_fwd", 4.0 * H * H * E * L, _per_step(kt, ["edge_fwd"], n), kt["edge_fwd"][1], on_tc=tc_edge)
        tensor("edge_bwd", 8.0 * H * H * E * L, _per_step(kt, ["edge_bwd"], n), kt["edge_bwd"][1], on_tc=tc_edge)
    # node GEMMs (P|Q projection, node MLP; forward, data and weight
    # gradients: 30 H^2 per node and layer) with their split-K reductions
    # node GEMMs (P|Q projection, node MLP; 30 H^2 per node and layer): the
    # data GEMMs of the main chain (forward and data gradients, 20 H^2) and
    # the split-K weight gradients with their reductions (10 H^2), which run
    # on the side streams (their event times include waits for SMs the main
    # chain holds)
    ops = "split bf16 (hi*hi + hi*lo + lo*hi)" if bf else "fp32 FFMA"
    data_names, wg_names = ["node_gemm", "gemm_small"], ["node_wgrad", "gemm_reduce"]
    tensor("node_gemm", 20.0 * H * H * N * L, _per_step(kt, data_names, n),
           sum(kt[x][1] for x in data_names), on_tc=bf,
           extra={"kernels": data_names, "operands": ops, "flops": "20 H^2 per node and layer (data GEMMs)"})
    tensor("node_wgrad", 10.0 * H * H * N * L, _per_step(kt, wg_names, n),
           sum(kt[x][1] for x in wg_names), on_tc=bf,
           extra={"kernels": wg_names, "operands": ops, "flops": "10 H^2 per node and layer (side streams)"})
    # HBM groups count unique bytes: data a launch must move at least once
    # (gathered node rows and second reads are L2 or DRAM traffic, which the
    # ncu `traffic` figures show).
    # node pass (tensor-core paths): the bf16 dL/da1 row of every edge (2H;
    # read for its destination and again for its source), its g_d (16), the
    # transpose-CSR position (4); per node the row pointers, dL/dx', S_dst,
    # S_src (2 x 4H) and dL/dx
    if kt["node_pass"][1]:
        memory("node_pass", (E * (2 * H + 16 + 4) + N * (8 * H + 8 + 24)) * L,
               _per_step(kt, ["node_pass"], n), kt["node_pass"][1],
               "E (2H + 20) + N (8H + 32) per layer (unique bytes)")
    if kt["src_pass"][1]:
        memory("src_pass", (E * (4 * H + 16 + 4) + N * (4 * H + 8 + 24)) * L,
               _per_step(kt, ["src_pass"], n), kt["src_pass"][1], "E (4H + 20) + N (4H + 32) per layer")
    if rows_path:
        # gather, forward and backward launch: indices (8 per launch), the u1
        # tile row (2H per launch), backward also silu'(a1) fp16 (2H) and the
        # gradient factors (16); per launch the P|Q table (8H per node) and
        # the coordinates (16 per node) once
        memory("edge_rows_u", (E * (16 + 4 * H + 2 * H + 16) + N * 2 * (8 * H + 16)) * L,
               _per_step(kt, ["edge_rows_u"], n), kt["edge_rows_u"][1],
               "E (6H + 32) + N (16H + 32) per layer (unique bytes)")
        memory("edge_rows_agg", (E * (4 * H + 20) + N * (4 * H + 24)) * L,
               _per_step(kt, ["edge_rows_agg"], n), kt["edge_rows_agg"][1], "E (4H + 20) + N (4H + 24) per layer")
    if rows_path:
        dom = "edge_rows_gemm"
    else:
        dom = "edge_bwd"
    return dom, groups


def make_line(args, prob, m, world, clk, cpu, dev):
    mc = prob.mc
    H = mc.hidden_nf
    peaks = measured_peaks()
    dom, groups = roofline(prob, m, peaks, clk, dev)
    kt, n = m["ktimes"], m["kt_steps"]
    d = dict(groups.get(dom, {}))
    d["kernel"] = dom
    launches = max(kt[dom][1], 1) if dom in kt else 1
    d["per_launch_ms"] = kt[dom][0] / launches if dom in kt else None
    d["launches"] = kt[dom][1] if dom in kt else 0
    if prob.precision == "bf16" and H == 128:
        d["traffic"] = ncu_traffic(args.config, "edge_bwd", prob.edges_rank)
    elif prob.precision == "bf16" and H == 256:
        d["traffic"] = ncu_traffic(args.config, dom, prob.edges_rank)
    else:
        d["traffic"] = None
    d["traffic_unit"] = "bytes per launch (ncu capture)"
    d["groups"] = groups
    step_flops = model_flops(mc, prob.nodes_rank, prob.edges_rank) * world
    ms = m["ms_per_step"]
    return {
        "metric": "egnn_train_layer_edges_per_s",
        "value": mc.n_layers * prob.edges_job / (ms * 1e-3),
        "unit": "layer-edges/s",
        "n_gpus": world, "steps": args.steps, "warmup": max(args.warmup, 3),
        "ms_per_step": ms, "higher_is_better": True, "scaling": prob.scaling,
        "vs_baseline": None, "dtype": prob.precision,
        "data": "synthetic (seeded generators, random init)",
        "config": {"workload": f"config{prob.cfg_id}", "graphs_per_gpu": prob.graphs_job // world,
                   "nodes_per_gpu": prob.nodes_rank, "edges_per_gpu": prob.edges_rank,
                   "layers": mc.n_layers, "hidden": H, "precision": prob.precision,
                   "l2": "flushed between timed steps (252 MB write)",
                   "parallelism": ("nodepart" if prob.halo else "dp") + str(world), "optimizer": "SGD",
                   "allreduce": ("per-layer buckets, issued as the backward produces them"
                                 if prob.allreduce == "layers" else "one flat all-reduce after the backward")
                   if world > 1 else None,
                   "cuda_graph": m["graphed"]},
        "molecules_per_s": prob.graphs_job / (ms * 1e-3),
        "model_tflops": step_flops / (ms * 1e-3) / 1e12,
        "e2e": m["e2e"],
        "gpu_launches": m["launches"],
        "roofline": d,
        "kernel_ms_per_step": {k: round(v[0] / n, 4) for k, v in kt.items() if v[1]},
        "cpu_baseline": cpu,
        "clocks": clk,
        "device_status": "ok" if m["status"] == 0 else "error",
    }


def cpu_baseline(cfg_id, steps):
    threads = os.cpu_count() or 1
    sample = cpu_sample_size(cfg_id)
    r = cpu_step_timer(cfg_id, sample, steps, 1, threads)
    full = sample == full_size(cfg_id)
    return {"value": r["layer_edges_per_s"], "unit": "layer-edges/s", "cores": threads, "kind": "port",
            "molecules_per_s": r["molecules_per_s"], "step_s": r["step_s"],
            "sample": (f"{'the whole' if full else 'a seeded subset of'} config{cfg_id}: {r['graphs']} graphs / "
                       f"{r['nodes']} nodes / {r['edges']} edges, fp32 oracle restatement of egnn_clean.EGNN, "
                       f"median of {steps} steps" + ("" if full else "; per-edge throughput extrapolates"))}


def run_b200(args):
    import torch
    import torch.distributed as dist

    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=300))
    prob = Problem(args, world, rank, dev)

    if args.profile:
        prob.step()
        torch.cuda.synchronize()
        for _ in range(args.steps):
            prob.step()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return 0

    clocks = ClockSampler(local)
    clocks.start()
    warmup = max(args.warmup, 3)
    m = measure(prob, args, world, dev, args.steps, warmup, graphs=not args.no_graphs, e2e=not args.no_e2e)
    clk = clocks.stop()
    peak_vram = torch.cuda.max_memory_allocated(dev) / 2**30
    line = None
    if rank == 0:
        cpu = None
        if not args.no_cpu_baseline and world == 1:
            cpu = cpu_baseline(args.config, 5)
        line = make_line(args, prob, m, world, clk, cpu, dev)
        line["peak_vram_gb"] = peak_vram
    del prob
    torch.cuda.empty_cache()

    # ---- one GPU, default run: the same step in fp32 mode (an equal-precision
    # ratio against the fp32 CPU arm) and the other workloads, each with its
    # roofline (shorter runs, no end-to-end pass)
    if world == 1 and not args.no_extras:
        extra_steps = min(args.steps, 10)
        if rank == 0:
            line["extras"] = {}
        runs = [(args.config, "fp32")] + [(c, None) for c in (1, 2, 3, 4, 5) if c != args.config]
        if args.config != 3:
            runs.append((3, "bf16"))   # config 3 is quoted in both modes
        for cfg_id, prec in runs:
            sub = argparse.Namespace(**vars(args))
            sub.config, sub.precision, sub.n_graphs, sub.n_nodes = cfg_id, prec, None, None
            p2 = Problem(sub, world, rank, dev)
            clocks = ClockSampler(local)
            clocks.start()
            m2 = measure(p2, sub, world, dev, extra_steps, 3, graphs=not args.no_graphs, e2e=False)
            clk2 = clocks.stop()
            cpu2 = None
            if not args.no_cpu_baseline and prec is None:
                cpu2 = cpu_baseline(cfg_id, 2)
            if rank == 0:
                rec = make_line(sub, p2, m2, world, clk2, cpu2, dev)
                for k in ("metric", "unit", "higher_is_better", "vs_baseline", "data", "e2e", "n_gpus", "warmup"):
                    rec.pop(k, None)
                rec["steps"] = extra_steps
                line["extras"][f"config{cfg_id}_{p2.precision}"] = rec
            del p2
            torch.cuda.empty_cache()
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    return run_b200(args)


if __name__ == "__main__":
    sys.exit(main())
