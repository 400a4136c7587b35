"""The drop-in layer API (reframework_b200.moe) against the reference goldens
and the reference's own behavioural tests, on the GPU."""

import pytest
import torch

from conftest import golden_config, load_golden, max_rel, routing_mismatches
from oracle import moe_oracle as O
from reframework_b200 import _lib
from reframework_b200.moe import FusedMoE, fused_experts, torch_fused_topk
from reframework_b200.workloads import generate

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
# tokens whose routed set differs from the golden fixture by a one-ulp logit tie,
# as observed on B200 for every fixture (16-bit and fp32 routers alike)
TIE_SWAPS_SEEN = 0


@pytest.fixture(autouse=True)
def _device_clean(cuda_ok):
    yield
    assert _lib.device_status() == 0


def tol(dtype):
    return 1e-4 if dtype == torch.float32 else 1e-2


def build_layer(cfg, d, *, harness):
    moe = FusedMoE(cfg.experts, cfg.top_k, cfg.hidden, cfg.inter, activation=cfg.activation,
                   renormalize=cfg.renormalize, dtype=cfg.dtype,
                   router_dtype=torch.float32 if harness else None,
                   num_shared_experts=cfg.shared_count, shared_intermediate_size=cfg.shared_inter,
                   shared_expert_gate=cfg.shared_gate)
    with torch.no_grad():
        moe.gate.copy_(d["gate"])
        for e in range(cfg.experts):
            moe.experts_w1[e].copy_(d["w1"][e])
            moe.experts_w2[e].copy_(d["w2"][e])
        if cfg.shared_count:
            moe.shared_w1.copy_(d["shared_w1"])
            moe.shared_w2.copy_(d["shared_w2"])
            if cfg.shared_gate:
                moe.shared_gate.copy_(d["shared_gate"])
    moe = moe.to(DEV)
    if harness and d["bias"] is not None:
        moe.set_router_bias(d["bias"][0])
    return moe


@pytest.mark.parametrize("name", ["c1_tiny_fp32", "c2_mini_bf16", "c3_mini_bf16", "c4_mini_bf16",
                                  "c4_mini_norenorm", "fp16_default", "bf16_gelu_default",
                                  "fp32_gelu_tanh", "bf16_entropy_k", "ep2_mini_bf16"])
def test_layer_matches_reference(name):
    rec = load_golden(name)
    cfg = golden_config(rec)
    d = generate(cfg)
    moe = build_layer(cfg, d, harness=rec["mode"] == "harness")
    if rec["mode"] == "entropy":
        moe.entropy_adaptive_k = True
        moe.entropy_k_min = rec["entropy_k_min"]
    x = d["x"].to(DEV)
    with torch.no_grad():
        w, ids = moe.route(x)
        out = moe(x)
        moe.precise_combine = True
        out_precise = moe(x)
    assert ids.dtype == torch.int64 and w.dtype == torch.float32
    harness = rec["mode"] == "harness"
    rdt = None if (harness or cfg.dtype == torch.float32) else cfg.dtype
    logits_ref = O.router_logits(d["x"], d["gate"], bias=d["bias"][0] if harness and d["bias"] else None,
                                 fp32=harness)
    # no fixture has a tie-swapped token on B200 (measured): any swap fails
    bad = routing_mismatches(ids, rec["ids"], logits_ref, cfg.top_k, round_dtype=rdt, max_count=TIE_SWAPS_SEEN)
    if harness or cfg.dtype == torch.float32:
        assert bad == [] and torch.equal(ids.cpu(), rec["ids"])
    keep = torch.ones(ids.shape[0], dtype=torch.bool)
    keep[bad] = False
    ref = rec["out_single"] if rec["mode"] == "ep2" else rec["out"]
    assert out.shape == ref.shape and out.dtype == ref.dtype
    err = max_rel(out.cpu()[keep], ref[keep])
    assert err < tol(cfg.dtype), f"max-rel {err:.3e}"
    # the fp32-accumulating combine is at least as close to the fp32-upcast
    # oracle as the reference itself is
    if cfg.dtype != torch.float32 and not cfg.shared_count and not bad:
        up = O.fused_experts(d["x"].float(), d["w1"].float(), d["w2"].float(), rec["weights"], rec["ids"],
                             cfg.activation)
        assert max_rel(out_precise, up) <= max(max_rel(ref, up), 4e-3)
        assert max_rel(out_precise, ref) < tol(cfg.dtype)


def test_offload_streaming_matches_reference():
    rec = load_golden("c5_mini_stream")
    cfg = golden_config(rec)
    d = generate(cfg)
    moe = build_layer(cfg, d, harness=True)
    cache = moe.build_offload_cache(DEV, lru_capacity=4)
    x = d["x"].to(DEV)
    for s in range(cfg.steps):
        moe.set_router_bias(d["bias"][s])
        with torch.no_grad():
            w, ids = moe.route(x)
            out = moe(x)
        assert torch.equal(ids.cpu(), rec["ids"][s])
        assert max_rel(out, rec["out"][s]) < 1e-2
    assert len(cache._lru) <= 4
    assert cache.stats.misses >= 4 and cache.stats.transfers_bytes > 0


def test_offload_equals_resident_exactly():
    """Same kernels, same order of summation: offload output == resident output."""
    from reframework_b200.workloads import CONFIGS, mini
    cfg = mini(CONFIGS["c5_mixtral22b_offload"], hidden=512, inter=512, tokens=300, steps=2)
    d = generate(cfg)
    a = build_layer(cfg, d, harness=True)
    b = build_layer(cfg, d, harness=True)
    b.build_offload_cache(DEV, lru_capacity=3)
    x = d["x"].to(DEV)
    for s in range(cfg.steps):
        a.set_router_bias(d["bias"][s])
        b.set_router_bias(d["bias"][s])
        with torch.no_grad():
            assert torch.equal(a(x), b(x))


def test_fused_experts_functional_api_and_linearity():
    rec = load_golden("c2_mini_bf16")
    cfg = golden_config(rec)
    d = generate(cfg)
    x, w1, w2 = d["x"].to(DEV), d["w1"].to(DEV), d["w2"].to(DEV)
    w, ids = rec["weights"].to(DEV), rec["ids"].to(DEV)
    out1 = fused_experts(x, w1, w2, w, ids)
    out1b = fused_experts(x, w1, w2, w, ids)
    assert torch.equal(out1, out1b), "not deterministic"
    out2 = fused_experts(x, w1, w2, w * 0.5, ids)
    assert torch.equal(out2, out1 * 0.5), "weight linearity"
    assert max_rel(out1, rec["out"]) < 1e-2
    # swapping the two most used experts changes the result
    a, b = torch.bincount(ids.reshape(-1).cpu(), minlength=cfg.experts).topk(2).indices.tolist()
    alt = torch.where(ids == a, b, torch.where(ids == b, a, ids))
    assert not torch.equal(fused_experts(x, w1, w2, w, alt), out1)
    # fp32 activations into bf16 experts: output keeps the activation dtype
    o32 = fused_experts(x.float(), w1, w2, w, ids)
    assert o32.dtype == torch.float32 and max_rel(o32, rec["out"]) < 1e-2


def test_torch_fused_topk_api():
    g = torch.Generator().manual_seed(0)
    lg = torch.randn(64, 8, generator=g)
    w, ids = torch_fused_topk(lg.to(DEV), 2, True)
    wr, ir = O.torch_fused_topk(lg, 2, True)
    assert torch.equal(ids.cpu(), ir) and ids.dtype == torch.int64
    torch.testing.assert_close(w.cpu(), wr, rtol=2e-5, atol=2e-6)


def test_state_dict_roundtrip_and_device_move():
    rec = load_golden("fp16_default")
    cfg = golden_config(rec)
    d = generate(cfg)
    src = build_layer(cfg, d, harness=False)
    sd = {k: v.detach().cpu().clone() for k, v in src.state_dict(prefix="model.layers.0.mlp").items()}
    assert "model.layers.0.mlp.experts.3.up_proj.weight" in sd
    assert sd["model.layers.0.mlp.experts.3.gate_proj.weight"].shape == (cfg.inter, cfg.hidden)
    dst = FusedMoE(cfg.experts, cfg.top_k, cfg.hidden, cfg.inter, dtype=cfg.dtype)
    dst.load_state_dict(sd, prefix="model.layers.0.mlp")
    dst = dst.to(DEV)
    x = d["x"].to(DEV)
    with torch.no_grad():
        assert torch.equal(dst(x), src(x))
        # in-place parameter edits are seen without any repack call
        dst.experts_w1[2].mul_(2.0)
        src_w1 = src.experts_w1[2]
        src_w1.mul_(2.0)
        assert torch.equal(dst(x), src(x))


def test_residual_fused_into_combine():
    rec = load_golden("c2_mini_bf16")
    cfg = golden_config(rec)
    d = generate(cfg)
    moe = build_layer(cfg, d, harness=True)
    x = d["x"].to(DEV)
    r = torch.randn_like(x)
    with torch.no_grad():
        a = moe(x, residual=r)
        b = moe(x).float() + r.float()
    assert max_rel(a, b) < 1e-2


def test_cpu_input_fails_loudly():
    moe = FusedMoE(4, 2, 64, 64, dtype=torch.bfloat16)
    with pytest.raises(_lib.RfMoeError):
        moe(torch.randn(3, 64, dtype=torch.bfloat16))


# ----- the reference's FusedMoE + offload + predictor behaviour tests, on CUDA
def _routed_moe(E=8):
    """Spike router (tests/test_moe_prefetch.py:198-218 of the reference):
    gate[e, e] = 10, so a token with 5.0 at dim d routes top-1 to expert d."""
    torch.manual_seed(0)
    mlp = FusedMoE(num_experts=E, top_k=1, hidden_size=16, intermediate_size=8, dtype=torch.float16)
    with torch.no_grad():
        mlp.gate.fill_(0.0)
        for e in range(E):
            mlp.gate[e, e] = 10.0
            mlp.experts_w1[e].normal_(0, 0.02)
            mlp.experts_w2[e].normal_(0, 0.02)
    return mlp.to(DEV)


def test_forward_drives_lookahead_reserve():
    mlp = _routed_moe(E=8)
    cache = mlp.build_offload_cache(DEV, lru_capacity=4)
    mlp.attach_predictor(window=8)
    assert mlp._predictor is not None and cache._predictor is mlp._predictor

    def spike(dim):
        x = torch.zeros(1, 16, dtype=torch.float16, device=DEV)
        x[0, dim] = 5.0
        return x

    for dim in range(5):
        with torch.no_grad():
            assert mlp(spike(dim)).shape == (1, 16)
    assert cache._next_reserve == frozenset({0})
    assert 0 in cache._lru and 4 in cache._lru
    assert cache.stats.predicts >= 1


def test_forward_prefill_does_not_lookahead():
    mlp = _routed_moe(E=8)
    cache = mlp.build_offload_cache(DEV, lru_capacity=8)
    mlp.attach_predictor(window=8)
    x = torch.zeros(4, 16, dtype=torch.float16, device=DEV)
    for dim in range(4):
        x[dim, dim] = 5.0
    with torch.no_grad():
        mlp(x)
    assert list(mlp._predictor._history) == []
    assert cache.stats.predicts == 0


@pytest.mark.parametrize("name", ["c3_mini_bf16", "c2_mini_bf16", "c1_tiny_fp32"])
def test_graph_capture_matches_eager(name):
    from reframework_b200.moe.graph import capture_forward
    rec = load_golden(name)
    cfg = golden_config(rec)
    d = generate(cfg)
    moe = build_layer(cfg, d, harness=rec["mode"] == "harness")
    x = d["x"].to(DEV)
    with torch.no_grad():
        eager = moe(x)
    g = capture_forward(moe, x)
    assert torch.equal(g(x), eager)
    x2 = torch.randn_like(x)
    with torch.no_grad():
        eager2 = moe(x2)
    assert torch.equal(g(x2), eager2)
    with pytest.raises(ValueError):
        g(x[:-1])


class _RMSNorm:
    """The parameters of reframework/layers/norm.py:18-24 (weight, eps, optional bias)."""

    def __init__(self, H, eps, bias, dtype, seed):
        g = torch.Generator().manual_seed(seed)
        self.weight = (1.0 + 0.1 * torch.randn(H, generator=g)).to(dtype).to(DEV)
        self.bias = (0.05 * torch.randn(H, generator=g)).to(dtype).to(DEV) if bias else None
        self.eps = eps

    def reference(self, r):
        """norm.py:27-35 in torch fp32, op by op."""
        x32 = r.to(torch.float32)
        norm = x32.pow(2).mean(-1, keepdim=True).add(self.eps).sqrt().reciprocal()
        out = x32 * norm
        out = out * self.weight.to(torch.float32)
        if self.bias is not None:
            out = out + self.bias.to(torch.float32)
        return out.to(r.dtype)


@pytest.mark.parametrize("name,bias", [("c2_mini_bf16", False), ("c3_mini_bf16", True), ("fp16_default", False),
                                       ("c1_tiny_fp32", True)])
def test_forward_add_residual_fuses_the_next_rmsnorm(name, bias):
    """forward_add_residual == (norm(moe(x) + r), moe(x) + r): the new residual
    is bit-identical to the unfused forward(x, residual=r); the normed rows match
    norm.py's fp32 restatement up to the order of the row sum."""
    rec = load_golden(name)
    cfg = golden_config(rec)
    d = generate(cfg)
    moe = build_layer(cfg, d, harness=rec["mode"] == "harness")
    x = d["x"].to(DEV)
    g = torch.Generator().manual_seed(3)
    r = torch.randn(x.shape, generator=g).to(x.dtype).to(DEV)
    norm = _RMSNorm(cfg.hidden, 1e-6, bias, cfg.dtype, seed=4)
    with torch.no_grad():
        normed, res = moe.forward_add_residual(x, r, norm)
        res_ref = moe(x, residual=r)
    assert torch.equal(res, res_ref)
    ref = norm.reference(res_ref)
    assert max_rel(normed, ref) < (1e-5 if cfg.dtype == torch.float32 else 1e-2)
    if cfg.dtype != torch.float32:
        same = (normed == ref).float().mean().item()
        assert same > 0.98, f"only {same:.3f} of the normed values bit-identical"
