"""Parity at the benchmark's full size (Mixtral-8x7B shape, 4096 tokens) and a
GEMM case where every CTA runs many tiles (accumulator double buffering and
barrier phase wrap-around)."""

import numpy as np
import pytest
import torch

from conftest import max_rel, routing_mismatches
from oracle import moe_oracle as O
from reframework_b200 import _lib
from reframework_b200 import kernels as K
from reframework_b200.moe import FusedMoE
from reframework_b200.workloads import CONFIGS, generate

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


@pytest.fixture(autouse=True)
def _device_clean(cuda_ok):
    _lib.set_gemm_impl(0)
    yield
    assert _lib.device_status() == 0


@pytest.mark.parametrize("act", ["silu", "gelu"])
def test_grouped_gemm_many_tiles_per_cta(act):
    g = torch.Generator(device=DEV).manual_seed(17)
    dtype = torch.bfloat16
    H, I = 1024, 2048
    counts = [1500, 1300, 0, 1777, 900]
    offs = [0]
    for c in counts:
        offs.append(offs[-1] + (c + 127) // 128 * 128)
    E = len(counts)
    a = torch.randn(offs[-1], H, generator=g, device=DEV, dtype=dtype)
    w1 = torch.randn(E, 2 * I, H, generator=g, device=DEV, dtype=dtype) * 0.03
    w2 = torch.randn(E, H, I, generator=g, device=DEV, dtype=dtype) * 0.03
    off_t = torch.tensor(offs, dtype=torch.int32, device=DEV)
    cnt_t = torch.tensor(counts, dtype=torch.int32, device=DEV)
    h = torch.empty(offs[-1], I, dtype=dtype, device=DEV)
    y = torch.empty(offs[-1], H, dtype=dtype, device=DEV)
    K.grouped_gemm_gated(a, w1, off_t, cnt_t, h, activation=act)
    K.grouped_gemm_down(h, w2, off_t, cnt_t, y)
    for e, c in enumerate(counts):
        if c == 0:
            continue
        xa = a[offs[e]:offs[e] + c].float()
        hr = O.gated_act_and_mul(act, (xa @ w1[e].float().t()).to(dtype)).float()
        yr = h[offs[e]:offs[e] + c].float() @ w2[e].float().t()
        assert max_rel(h[offs[e]:offs[e] + c], hr) < 8e-3, f"h expert {e}"
        assert max_rel(y[offs[e]:offs[e] + c], yr) < 8e-3, f"y expert {e}"
    y_first = y.clone()
    K.grouped_gemm_gated(a, w1, off_t, cnt_t, h, activation=act)
    K.grouped_gemm_down(h, w2, off_t, cnt_t, y)
    assert torch.equal(y, y_first), "second run differs"


def test_c2_full_size_parity_with_oracle():
    """Full benchmark size: routing ids and the per-expert permutation equal the
    oracle's bit for bit; the output is within max-rel 1e-2 (bf16)."""
    cfg = CONFIGS["c2_mixtral_bf16"]
    torch.set_num_threads(max(1, torch.get_num_threads()))
    d = generate(cfg)
    ref = O.moe_forward(d["x"], d["gate"], d["w1"], d["w2"], top_k=cfg.top_k, bias=d["bias"][0],
                        router_fp32=True)
    moe = FusedMoE(cfg.experts, cfg.top_k, cfg.hidden, cfg.inter, dtype=cfg.dtype,
                   router_dtype=torch.float32, device=DEV)
    with torch.no_grad():
        moe.gate.copy_(d["gate"])
        w1b, w2b = moe._resident_banks()
        w1b.copy_(d["w1"])
        w2b.copy_(d["w2"])
    moe.set_router_bias(d["bias"][0])
    x = d["x"].to(DEV)
    with torch.no_grad():
        w, ids = moe.route(x)
        out = moe(x)
        out2 = moe(x)
    assert torch.equal(out, out2), "not deterministic"
    assert routing_mismatches(ids, ref["ids"], ref["logits"], cfg.top_k) == []
    assert torch.equal(ids.cpu(), ref["ids"]), "fp32 routing must be bit-exact at full size"
    # permutation: the GPU's expert-grouped row order is the reference's
    p = K.permute(ids.to(torch.int32), cfg.experts)
    counts, order = O.permutation(ids.cpu().numpy(), cfg.experts)
    off = p.offsets.cpu().numpy()
    src = p.src_slot.cpu().numpy()
    got = np.concatenate([src[off[e]:off[e] + counts[e]] for e in range(cfg.experts)])
    assert np.array_equal(got, order)
    err = max_rel(out, ref["out"])
    same = float((out.cpu() == ref["out"]).float().mean())
    print(f"full-size C2: max-rel {err:.3e}, bit-identical outputs {same:.4f}")
    assert err < 1e-2, f"max-rel {err:.3e}"
    assert same > 0.9, f"only {same:.3f} of the outputs equal the reference's bits"
    # weight linearity holds exactly at full size
    w_half = (w * 0.5).contiguous()
    o_half = torch.empty_like(out)
    pp = K.permute(ids.to(torch.int32), cfg.experts, x=x)
    h = torch.empty(pp.rows_cap, cfg.inter, dtype=cfg.dtype, device=DEV)
    K.grouped_gemm_gated(pp.x_perm, w1b, pp.offsets, pp.counts, h)
    yv = torch.empty(pp.rows_cap, cfg.hidden, dtype=cfg.dtype, device=DEV)
    K.grouped_gemm_down(h, w2b, pp.offsets, pp.counts, yv)
    K.combine(yv, pp.row_of_slot, w_half, o_half)
    assert torch.equal(o_half, out * 0.5)
