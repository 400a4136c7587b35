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


ULP_REL = {torch.bfloat16: 2.0 ** -7, torch.float16: 2.0 ** -10}


def routing_mismatches(ids, ids_ref, logits_ref, top_k, round_dtype=None, max_frac=1e-3, max_count=None):
    """Tokens whose routed expert set differs from the reference's.

    A difference is accepted only when it is a numerical tie at the top-k
    boundary: every swapped expert's reference logit lies within the
    tolerance of the k-th largest logit — 1e-5 relative for an fp32 router,
    one ulp of the layer dtype when the logits are rounded to it (then the
    reference's own choice among equal values is implementation-defined).
    At most ``max_count`` such tokens (default: max(2, max_frac * T)) are
    accepted.  Returns the list of such tokens."""
    ids = ids.cpu().long()
    bad = []
    for t in (ids.sort(1).values != ids_ref.sort(1).values).any(1).nonzero().flatten().tolist():
        lg = logits_ref[t].float()
        kth = torch.topk(lg, top_k).values[-1]
        diff = set(ids[t].tolist()) ^ set(ids_ref[t].tolist())
        rel = ULP_REL.get(round_dtype, 1e-5)
        tol = rel * max(1.0, float(lg.abs().max()))
        gaps = [abs(float(lg[e] - kth)) for e in diff]
        assert max(gaps) <= tol, f"token {t}: ids {ids[t].tolist()} vs {ids_ref[t].tolist()}, gaps {gaps}"
        bad.append(t)
    cap = max(2, int(max_frac * ids.shape[0])) if max_count is None else max_count
    assert len(bad) <= cap, f"{len(bad)} tie-swapped tokens (at most {cap} accepted)"
    return bad


@pytest.fixture(scope="session")
def cuda_ok():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return True
