import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def rel_err(a, b) -> float:
    """max |a - b| / max |b| (0 when both are empty or b is all zeros and a == b)."""
    a = a.detach().double().cpu()
    b = b.detach().double().cpu()
    if b.numel() == 0:
        return 0.0
    den = b.abs().max().item()
    num = (a - b).abs().max().item()
    if den == 0.0:
        return num
    return num / den


def graph_sum(values, graph_ptr):
    """Deterministic per-graph sum of node values (nodes grouped by graph).

    segment_reduce adds each graph's nodes in order; a float cumsum on the GPU
    is a look-back scan whose association order can change from run to run."""
    gp = graph_ptr.to(values.device)
    return torch.segment_reduce(values, "sum", lengths=gp[1:] - gp[:-1], unsafe=True)


def tolerances(ref, approx, floor, factor):
    """Per-tensor tolerance: max(floor, factor * error of `approx` against `ref`).

    `approx` is the reference algorithm computed at the precision under test
    (the fp32 oracle, or the rounding-exact bf16 model), so each tensor's bar
    is never tighter than what that precision can reach on it.
    """
    return {k: max(floor, factor * rel_err(approx[k], ref[k])) for k in ref}


BF16_TOL = 2e-2    # north star: bf16-GEMM mode against the fp64 reference
BF16_MODEL_TOL = 5e-3


def check_bf16(got, ref, emu, what=""):
    """bf16-GEMM bar: every tensor within 2e-2 of fp64, and within 5e-3 of the
    rounding-exact bf16 model (oracle/egnn_emulation.py) on every tensor that
    model itself computes to better than 5e-3."""
    errs = check_tensors(got, ref, {k: BF16_TOL for k in ref}, what + " vs fp64")
    emu_err = {k: rel_err(emu[k], ref[k]) for k in ref}
    tight = {k: (BF16_MODEL_TOL if emu_err[k] < BF16_MODEL_TOL else float("inf")) for k in ref}
    check_tensors(got, emu, tight, what + " vs rounding-exact bf16 model")
    return errs


def as_dict(res):
    """(h, x, dh, dx, {grads}) -> flat dict."""
    out = {"h": res[0], "x": res[1], "dh": res[2], "dx": res[3]}
    out.update({k: (v if v is not None else torch.zeros(1)) for k, v in res[4].items()})
    return out


def check_tensors(got, ref, tol, what=""):
    errs = {k: rel_err(got[k], ref[k]) for k in ref}
    bad = {k: (errs[k], tol[k]) for k in ref if not errs[k] <= tol[k]}
    assert not bad, f"{what}: (error, tolerance) over bar: {bad}"
    return errs


def golden_cases():
    return sorted(p.stem for p in GOLDEN.glob("*.pt"))


def load_golden(name):
    return torch.load(GOLDEN / f"{name}.pt", weights_only=False)


@pytest.fixture(scope="session")
def cuda_device():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)
