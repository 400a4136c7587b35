"""Pin the CPU oracle to the reference: every golden fixture (produced by
running the reference itself, tests/golden/make_golden.py) must be reproduced
by oracle/moe_oracle.py on the same seeded inputs."""

import os

import numpy as np
import pytest
import torch

from conftest import golden_config, load_golden, max_rel
from oracle import moe_oracle as O
from reframework_b200.workloads import generate

LAYER_CASES = ["c1_tiny_fp32", "fp16_default", "bf16_gelu_default", "fp32_gelu_tanh"]
HARNESS_CASES = ["c2_mini_bf16", "c3_mini_bf16", "c4_mini_bf16", "c4_mini_norenorm"]


def _oracle_forward(rec):
    cfg = golden_config(rec)
    d = generate(cfg)
    kw = {}
    if rec["mode"] == "entropy":
        kw["entropy_k_min"] = rec["entropy_k_min"]
    res = O.moe_forward(
        d["x"], d["gate"], d["w1"], d["w2"], top_k=cfg.top_k, renormalize=cfg.renormalize,
        bias=(d["bias"][0] if d["bias"] is not None else None),
        router_fp32=(rec["mode"] == "harness"), activation=cfg.activation,
        shared_w1=d.get("shared_w1"), shared_w2=d.get("shared_w2"),
        shared_gate=d.get("shared_gate"), **kw)
    return cfg, d, res


@pytest.mark.parametrize("name", LAYER_CASES + HARNESS_CASES + ["bf16_entropy_k"])
def test_oracle_matches_reference(name):
    rec = load_golden(name)
    cfg, d, res = _oracle_forward(rec)
    assert torch.equal(res["ids"], rec["ids"]), "routing ids differ from the reference"
    torch.testing.assert_close(res["weights"], rec["weights"], rtol=0, atol=0)
    # same torch CPU kernels in the same order: bit-identical
    assert torch.equal(res["out"], rec["out"]), max_rel(res["out"], rec["out"])


@pytest.mark.parametrize("name", LAYER_CASES + HARNESS_CASES)
def test_oracle_permutation_matches_reference_order(name):
    rec = load_golden(name)
    ids = rec["ids"].numpy()
    T, K = ids.shape
    counts, order = O.permutation(ids, golden_config(rec).experts)
    exps = rec["perm_experts"].tolist()
    assert [e for e in range(len(counts)) if counts[e]] == exps
    pos = 0
    for e, toks in zip(exps, rec["perm_tokens"]):
        seg = order[pos:pos + counts[e]]
        pos += counts[e]
        assert np.array_equal(seg // K, toks.numpy()), f"expert {e} token order differs"
        assert np.all(ids.reshape(-1)[seg] == e)


def test_oracle_streaming_matches_reference():
    rec = load_golden("c5_mini_stream")
    cfg = golden_config(rec)
    d = generate(cfg)
    for s in range(cfg.steps):
        w, ids = O.route(d["x"], d["gate"], cfg.top_k, cfg.renormalize, bias=d["bias"][s])
        assert torch.equal(ids, rec["ids"][s])
        out = O.forward_streaming(d["x"], d["w1"], d["w2"], w, ids, chunk_size=4)
        assert torch.equal(out, rec["out"][s]), max_rel(out, rec["out"][s])


def test_oracle_split_matches_reference():
    """The CPU/GPU split (hits in bf16, misses on int8 copies) step by step
    against the reference's own _forward_split, given the experts resident
    before each step; bit for bit."""
    rec = load_golden("int8_split_k1")
    cfg = golden_config(rec)
    d = generate(cfg)
    for s in range(cfg.steps):
        w, ids = O.route(d["x"], d["gate"], cfg.top_k, cfg.renormalize, bias=d["bias"][s])
        assert torch.equal(ids, rec["ids"][s])
        res = O.split_forward(d["x"], d["w1"], d["w2"], w, ids, set(rec["resident_before"][s].tolist()))
        assert torch.equal(res["out"], rec["out"][s]), (s, max_rel(res["out"], rec["out"][s]))
    assert any(rec["resident_before"][s].numel() for s in range(cfg.steps)), "some step has hits"


def test_oracle_int8_quantizer_and_gemm_are_exact():
    """sym_int8_quantize round-trips within half a step, and the int8 GEMM is
    exact integer arithmetic (the part of the int8 half a GPU reproduces bit
    for bit)."""
    g = torch.Generator().manual_seed(0)
    w = torch.randn(64, 96, generator=g)
    q, sc = O.sym_int8_quantize(w)
    assert q.dtype == torch.int8 and int(q.abs().max()) == 127
    assert float((q.float() * sc - w).abs().max()) <= sc / 2 + 1e-7
    z, sz = O.sym_int8_quantize(torch.zeros(3, 4))
    assert sz == 1.0 and not z.any()
    a = torch.randint(-127, 128, (17, 96), generator=g, dtype=torch.int8)
    assert torch.equal(torch._int_mm(a, q.t().contiguous()), a.int() @ q.int().t())


def test_oracle_ep_sum_matches_reference_ep():
    """The reference EP (replicate tokens, mask, all-reduce over 2 gloo ranks)
    equals the single-process layer up to fp summation order; the oracle's
    resident forward is the single-process layer."""
    rec = load_golden("ep2_mini_bf16")
    cfg, d, res = _oracle_forward(rec)
    assert torch.equal(res["ids"], rec["ids"])
    assert torch.equal(res["out"], rec["out_single"])
    assert max_rel(rec["out"], rec["out_single"]) < 1e-2


def test_shard_range_matches_reference_examples():
    assert O.shard_range(8, 2, 0) == (0, 4) and O.shard_range(8, 2, 1) == (4, 8)
    spans = [O.shard_range(10, 4, r) for r in range(4)]
    assert spans == [(0, 3), (3, 6), (6, 8), (8, 10)]


def test_oracle_bias_changes_routing():
    """A planted mistake in the oracle (dropping the bias) must be caught by the
    golden comparison — guards against a vacuous pin."""
    rec = load_golden("c2_mini_bf16")
    cfg = golden_config(rec)
    d = generate(cfg)
    w, ids = O.route(d["x"], d["gate"], cfg.top_k, cfg.renormalize, bias=None)
    assert not torch.equal(ids, rec["ids"])
