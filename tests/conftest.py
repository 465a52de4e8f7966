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


def golden_cases():
    return sorted(p.stem for p in GOLDEN.glob("*.pt"))


def load_golden(name):
    return torch.load(GOLDEN / f"{name}.pt", weights_only=False)


@pytest.fixture(scope="session")
def cuda_device():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)
