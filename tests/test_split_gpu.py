"""The expert split on the GPU (hits in the layer dtype, misses on int8
copies): the int8 kernels are exact where the reference's arithmetic is exact
(integer GEMMs, the quantizer), and the layer matches the reference's own split
forward (golden fixture) step by step."""

import pytest
import torch

from conftest import golden_config, load_golden, max_rel
from oracle import moe_oracle as O
from reframework_b200 import _lib
from reframework_b200 import kernels as K
from reframework_b200.moe import FusedMoE
from reframework_b200.workloads import generate

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


@pytest.fixture(autouse=True)
def _device_clean(cuda_ok):
    yield
    assert _lib.device_status() == 0


def _segments(counts, align=128):
    offs, o = [], 0
    for c in counts:
        offs.append(o)
        o += (c + align - 1) // align * align
    return torch.tensor(offs, dtype=torch.int32), torch.tensor(counts, dtype=torch.int32), max(o, 1)


@pytest.mark.parametrize("Kdim,N,counts", [(64, 64, [5, 0, 70]), (272, 200, [130, 1, 0, 64]), (1024, 96, [300])])
def test_int8_gemm_is_exact(Kdim, N, counts):
    """Unit scales and weights: the down GEMM returns the int32 sums exactly
    (|sum| < 2^24), listed experts through a slot table."""
    g = torch.Generator().manual_seed(Kdim + N)
    E = len(counts)
    offs, cnt, rows = _segments(counts)
    a = torch.randint(-127, 128, (rows, Kdim), generator=g, dtype=torch.int8)
    w = torch.randint(-127, 128, (E + 1, N, Kdim), generator=g, dtype=torch.int8)
    slot = torch.tensor([(e + 1) % (E + 1) for e in range(E)], dtype=torch.int32)  # not the identity
    groups = torch.tensor([e for e in range(E) if counts[e]][::-1], dtype=torch.int32)
    src_slot = torch.arange(rows, dtype=torch.int32)
    out = torch.full((rows, N), float("nan"), device=DEV)
    K.int8_grouped_gemm(a.to(DEV), w.to(DEV), offs.to(DEV), cnt.to(DEV), groups.to(DEV), slot.to(DEV),
                        torch.ones(len(groups), device=DEV), torch.ones(E, device=DEV), 1, out, gated=False,
                        row_weights=torch.ones(rows, device=DEV), src_slot=src_slot.to(DEV))
    out = out.cpu()
    for e in range(E):
        if not counts[e]:
            continue
        r0 = int(offs[e])
        ref = (a[r0:r0 + counts[e]].int() @ w[int(slot[e])].int().t()).float()
        assert torch.equal(out[r0:r0 + counts[e]], ref), f"expert {e}"


@pytest.mark.parametrize("gated", [True, False])
@pytest.mark.parametrize("act", ["silu", "gelu_tanh"])
@pytest.mark.parametrize("Kdim,N,counts", [(1024, 352, [300, 0, 17, 129]), (272, 200, [130, 1, 0, 64])])
def test_int8_tensor_core_gemm_equals_dp4a(gated, act, Kdim, N, counts):
    """tcgen05.mma kind::i8 (exact int32 sums in TMEM) and the dp4a CUDA-core
    kernel give the same bits: same int32 sums, the same fp32 scale products,
    activation and routing weight, and (gated) the same per-expert max."""
    g = torch.Generator().manual_seed(Kdim * 3 + N + gated)
    E = len(counts)
    offs, cnt, rows = _segments(counts)
    a = torch.randint(-127, 128, (rows, Kdim), generator=g, dtype=torch.int8).to(DEV)
    w = torch.randint(-127, 128, (E + 1, (2 if gated else 1) * N, Kdim), generator=g, dtype=torch.int8).to(DEV)
    slot = torch.tensor([(e + 1) % (E + 1) for e in range(E)], dtype=torch.int32).to(DEV)
    groups = torch.tensor([e for e in range(E) if counts[e]][::-1], dtype=torch.int32).to(DEV)
    a_sc = (torch.rand(len(groups), generator=g) * 1e-3 + 1e-4).to(DEV)
    w_sc = (torch.rand(E, generator=g) * 1e-3 + 1e-4).to(DEV)
    rw = torch.rand(rows, generator=g).to(DEV)
    src = torch.randperm(rows, generator=g).to(torch.int32).to(DEV)
    res = []
    for impl in (0, 1):  # 0: tensor cores where the shape allows, 1: CUDA cores only
        _lib.set_gemm_impl(impl)
        out = torch.full((rows, N), float("nan"), device=DEV)
        amax = torch.zeros(len(groups), device=DEV)
        K.int8_grouped_gemm(a, w, offs.to(DEV), cnt.to(DEV), groups, slot, a_sc, w_sc, 1, out, gated=gated,
                            activation=act, amax_out=amax if gated else None,
                            row_weights=None if gated else rw, src_slot=None if gated else src)
        res.append((out.cpu(), amax.cpu()))
    _lib.set_gemm_impl(0)
    for e in range(E):
        r0 = int(offs[e])
        seg = slice(r0, r0 + counts[e])
        assert torch.equal(res[0][0][seg], res[1][0][seg]), f"expert {e}"
    if gated:
        assert torch.equal(res[0][1], res[1][1])


def test_int8_quantize_matches_the_reference_quantizer():
    g = torch.Generator().manual_seed(1)
    counts = [40, 0, 3, 129]
    offs, cnt, rows = _segments(counts)
    x = (torch.randn(rows, 96, generator=g) * 3).bfloat16()
    x[int(offs[2]):int(offs[2]) + 3] = 0  # an all-zero block: scale 1, zero codes
    groups = torch.tensor([0, 2, 3], dtype=torch.int32)
    q = torch.zeros(rows, 96, dtype=torch.int8, device=DEV)
    scales, amax = torch.empty(3, device=DEV), torch.empty(3, device=DEV)
    K.int8_quantize(x.to(DEV), offs.to(DEV), cnt.to(DEV), groups.to(DEV), q, scales, amax)
    q, scales = q.cpu(), scales.cpu()
    for i, e in enumerate(groups.tolist()):
        r0 = int(offs[e])
        rq, rs = O.sym_int8_quantize(x[r0:r0 + counts[e]].float())
        assert torch.equal(q[r0:r0 + counts[e]], rq), f"expert {e}"
        assert float(scales[i]) == torch.tensor(rs, dtype=torch.float32).item()


def _split_layer(cfg, d):
    moe = FusedMoE(cfg.experts, cfg.top_k, cfg.hidden, cfg.inter, activation=cfg.activation,
                   renormalize=cfg.renormalize, dtype=cfg.dtype, router_dtype=torch.float32)
    with torch.no_grad():
        moe.gate.copy_(d["gate"])
        for e in range(cfg.experts):
            moe.experts_w1[e].copy_(d["w1"][e])
            moe.experts_w2[e].copy_(d["w2"][e])
    moe = moe.to(DEV)
    cache = moe.build_offload_cache(DEV, lru_capacity=4)
    moe.enable_cpu_split()
    assert moe.cpu_split
    return moe, cache


def test_split_forward_matches_the_reference_split():
    """Top-1 steps of the reference's own _forward_split: same routing, same
    experts resident before every step, same counters; outputs within the
    bf16 bar (the int8 half's fp32 activation may differ from torch's CPU
    kernels by an ulp before it is quantized again)."""
    rec = load_golden("int8_split_k1")
    cfg = golden_config(rec)
    d = generate(cfg)
    moe, cache = _split_layer(cfg, d)
    x = d["x"].to(DEV)
    for s in range(cfg.steps):
        assert sorted(cache._lru) == rec["resident_before"][s].tolist(), f"step {s}"
        moe.set_router_bias(d["bias"][s])
        with torch.no_grad():
            out = moe(x)
        ref = O.split_forward(d["x"], d["w1"], d["w2"], *O.route(d["x"], d["gate"], cfg.top_k, cfg.renormalize,
                                                                 bias=d["bias"][s]),
                              set(rec["resident_before"][s].tolist()))
        assert torch.equal(ref["out"], rec["out"][s])
        assert max_rel(out, rec["out"][s]) < 1e-2, (s, max_rel(out, rec["out"][s]))
    assert sorted(cache._lru) == rec["resident_after"].tolist()
    st = cache.stats.as_dict()
    for k in ("hits", "misses", "evictions", "transfer_mb"):
        assert st[k] == rec["cache_stats"][k], k
    assert cache.int8_transfer_bytes > 0


@pytest.mark.parametrize("top_k", [2, 4])
def test_split_forward_matches_the_oracle_for_top_k(top_k):
    """K > 1 (where the reference maps slots to the wrong tokens): against
    the oracle's split with slot (t, k) -> token t."""
    from reframework_b200.workloads import CONFIGS, mini
    cfg = mini(CONFIGS["c5_mixtral22b_offload"], hidden=256, inter=256, tokens=80, steps=3, top_k=top_k, seed=11,
               name=f"split_k{top_k}")
    d = generate(cfg)
    moe, cache = _split_layer(cfg, d)
    x = d["x"].to(DEV)
    for s in range(cfg.steps):
        before = set(cache._lru)
        moe.set_router_bias(d["bias"][s])
        with torch.no_grad():
            out = moe(x)
        w, ids = O.route(d["x"], d["gate"], cfg.top_k, cfg.renormalize, bias=d["bias"][s])
        ref = O.split_forward(d["x"], d["w1"], d["w2"], w, ids, before)
        assert max_rel(out, ref["out"]) < 1e-2, (s, max_rel(out, ref["out"]))
