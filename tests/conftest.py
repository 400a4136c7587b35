import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def load_golden(name):
    return torch.load(os.path.join(GOLDEN, f"{name}.pt"), weights_only=False)


def golden_config(rec):
    """Rebuild the MoEConfig a fixture was generated with."""
    from reframework_b200.workloads import MoEConfig
    c = dict(rec["config"])
    c["dtype"] = getattr(torch, c["dtype"].replace("torch.", ""))
    return MoEConfig(**c)


def max_rel(a, r):
    """max|a - r| / max|r| over the whole tensor (fp32)."""
    a = a.float().cpu()
    r = r.float().cpu()
    return float((a - r).abs().max() / r.abs().max().clamp_min(1e-30))


@pytest.fixture(scope="session")
def cuda_ok():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return True
