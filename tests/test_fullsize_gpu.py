"""Parity at the benchmark configurations' full sizes (C2 Mixtral-8x7B, C3
decode, C4 DeepSeek-V2-Lite with its expert-parallel split emulated, C5 with the
offload cache) and a GEMM case where every CTA runs many tiles (accumulator
double buffering and barrier phase wrap-around)."""

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
    h = torch.zeros(offs[-1], I, dtype=dtype, device=DEV)
    y = torch.zeros(offs[-1], H, dtype=dtype, device=DEV)
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
    for e, c in enumerate(counts):  # the rows the GEMMs own (pad rows are never written)
        assert torch.equal(y[offs[e]:offs[e] + c], y_first[offs[e]:offs[e] + c]), f"second run differs (expert {e})"


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


def _layer_from(cfg, d):
    """A resident FusedMoE on the GPU holding the workload's weights (fp32
    router with the config's bias, shared experts as configured)."""
    moe = FusedMoE(cfg.experts, cfg.top_k, cfg.hidden, cfg.inter, activation=cfg.activation,
                   renormalize=cfg.renormalize, dtype=cfg.dtype, router_dtype=torch.float32,
                   num_shared_experts=cfg.shared_count, shared_intermediate_size=cfg.shared_inter,
                   shared_expert_gate=cfg.shared_gate, device=DEV)
    with torch.no_grad():
        moe.gate.copy_(d["gate"])
        w1b, w2b = moe._resident_banks()
        w1b.copy_(d["w1"])
        w2b.copy_(d["w2"])
        if cfg.shared_count:
            moe.shared_w1.copy_(d["shared_w1"])
            moe.shared_w2.copy_(d["shared_w2"])
            if cfg.shared_gate:
                moe.shared_gate.copy_(d["shared_gate"])
    if d["bias"] is not None:
        moe.set_router_bias(d["bias"][0])
    return moe


def _oracle_forward(cfg, d):
    return O.moe_forward(d["x"], d["gate"], d["w1"], d["w2"], top_k=cfg.top_k, renormalize=cfg.renormalize,
                         bias=d["bias"][0] if d["bias"] is not None else None, router_fp32=True,
                         activation=cfg.activation,
                         shared_w1=d.get("shared_w1") if cfg.shared_count else None,
                         shared_w2=d.get("shared_w2") if cfg.shared_count else None,
                         shared_gate=d.get("shared_gate") if cfg.shared_gate else None)


def _check_full_size(cfg, label):
    d = generate(cfg)
    ref = _oracle_forward(cfg, d)
    moe = _layer_from(cfg, d)
    x = d["x"].to(DEV)
    with torch.no_grad():
        w, ids = moe.route(x)
        out = moe(x)
        out2 = moe(x)
    assert torch.equal(out, out2), "not deterministic"
    assert routing_mismatches(ids, ref["ids"], ref["logits"], cfg.top_k) == []
    assert torch.equal(ids.cpu(), ref["ids"]), "fp32 routing must be bit-exact at full size"
    torch.testing.assert_close(w.cpu(), ref["weights"], rtol=2e-5, atol=2e-6)
    p = K.permute(ids.to(torch.int32), cfg.experts)
    counts, order = O.permutation(ids.cpu().numpy(), cfg.experts)
    off = p.offsets.cpu().numpy()
    src = p.src_slot.cpu().numpy()
    assert np.array_equal(p.counts.cpu().numpy(), counts)
    got = np.concatenate([src[off[e]:off[e] + counts[e]] for e in range(cfg.experts)])
    assert np.array_equal(got, order), "permutation differs from the reference's selection order"
    err = max_rel(out, ref["out"])
    same = float((out.cpu() == ref["out"]).float().mean())
    print(f"full-size {label}: max-rel {err:.3e}, bit-identical outputs {same:.4f}")
    assert err < 1e-2, f"max-rel {err:.3e}"
    return moe, d, out


def test_c3_full_size_parity_with_oracle():
    """Qwen1.5-MoE decode at its benchmark size (H2048 E60 top-4 I1408, 64
    tokens, Zipf(1.1) router bias, one shared SwiGLU expert of 5632 gated by
    sigmoid(x.w_s)): fp32-router ids and the permutation bit-exact, output
    within max-rel 1e-2 of the oracle (reference fused.py:32-87 plus the
    harness's gated shared expert)."""
    _check_full_size(CONFIGS["c3_qwen_decode"], "C3")


@pytest.mark.parametrize("renormalize", [True, False])
def test_c4_full_size_parity_with_oracle(renormalize):
    """DeepSeek-V2-Lite shape at its benchmark size (H2048 E64 top-6 I1408,
    8192 tokens, two shared experts of 1408), renormalised and not."""
    from dataclasses import replace
    cfg = replace(CONFIGS["c4_dsv2lite_ep"], renormalize=renormalize)
    _check_full_size(cfg, f"C4 renormalize={renormalize}")


def _emulated_ep_forward(moe, x, R, placement, overlap=False):
    """The expert-parallel forward of EPFusedMoE's device-planned path, R ranks
    emulated on one GPU with separate buffers: every rank's route + compact
    permute, device plan, dispatch push, regroup, gated GEMM, down GEMM with the
    return exchange in its epilogue, and combine (+ the shared experts).  The
    stages run rank by rank in stream order, so each bounded wait starts only
    after every push it waits for has run.  ``overlap``: the overlapped
    dispatch (rows for the other ranks pushed, own rows placed straight into
    the GEMM rows and their gated GEMM run before the wait, then the other
    sources' rows regrouped and their gated GEMM).  Returns the concatenated
    outputs."""
    import ctypes
    from reframework_b200.parallel.ep import shard_range  # noqa: F401  (placement built by the caller)
    L = _lib.lib()
    T, H = x.shape
    E, Kk, I = moe.num_experts, moe.top_k, moe.intermediate_size
    st = torch.cuda.current_stream(DEV).cuda_stream
    bounds = [(T * r // R, T * (r + 1) // R) for r in range(R)]
    routed = []
    for lo, hi in bounds:
        w, ids32, _, _, sscale = moe._router(x[lo:hi].contiguous(), ids32=True, ids64=False)
        routed.append((w, ids32, sscale, K.permute(ids32, E, align=1)))
    # the counts all-gather through the peer-store kernels: every rank's row into
    # every rank's table, then each rank's bounded collect
    cnt = torch.stack([r[3].counts for r in routed]).contiguous()
    tables = [torch.zeros(R, E, dtype=torch.int32, device=DEV) for _ in range(R)]
    cflags = [torch.zeros(R, dtype=torch.int32, device=DEV) for _ in range(R)]
    for me in range(R):
        assert L.rf_moe_ep_counts_push(routed[me][3].counts.data_ptr(), E, R, me,
                                       (ctypes.c_void_p * R)(*[t.data_ptr() for t in tables]),
                                       (ctypes.c_void_p * R)(*[f.data_ptr() + 4 * me for f in cflags]), 3, st) == 0
    for me in range(R):
        got = torch.empty(R, E, dtype=torch.int32, device=DEV)
        assert L.rf_moe_ep_counts_collect(cflags[me].data_ptr(), tables[me].data_ptr(), R, E, 3, got.data_ptr(),
                                          st) == 0
        assert torch.equal(got, cnt), f"rank {me}: collected counts table differs"
    flat = torch.tensor([e for s in placement.slots for e in s], dtype=torch.int32, device=DEV)
    offs = torch.tensor(np.cumsum([0] + [len(s) for s in placement.slots]), dtype=torch.int32, device=DEV)
    nslots = int(flat.numel())
    tmax = max(hi - lo for lo, hi in bounds)
    recv_cap, back_cap = R * tmax * Kk, tmax * Kk
    row_bytes = H * x.element_size()
    recv = [torch.zeros(recv_cap, H, dtype=x.dtype, device=DEV) for _ in range(R)]
    back = [torch.zeros(back_cap, H, dtype=x.dtype, device=DEV) for _ in range(R)]
    ctrl = [torch.zeros(2 * R, dtype=torch.int32, device=DEV) for _ in range(R)]
    done = torch.zeros(R, dtype=torch.int32, device=DEV)
    ptrs = lambda ts: (ctypes.c_void_p * R)(*[t.data_ptr() for t in ts])  # noqa: E731
    flags = lambda d_, me: (ctypes.c_void_p * R)(*[ctrl[d].data_ptr() + 4 * (d_ * R + me) for d in range(R)])  # noqa: E731
    ws, segs, groups = [], [], []
    for me in range(R):
        S = len(placement.slots[me])
        nb = L.rf_moe_ep_devplan_workspace_size(R, E, S, nslots)
        lay = np.zeros(_lib.EP_DEVPLAN_LAYOUT_N, np.int64)
        assert L.rf_moe_ep_devplan_layout(R, E, S, nslots, lay.ctypes.data) == 0
        wsp = torch.zeros(nb, dtype=torch.uint8, device=DEV)
        rows_cap = recv_cap + S * (K.ALIGN - 1)
        assert L.rf_moe_ep_devplan(cnt.data_ptr(), flat.data_ptr(), offs.data_ptr(), R, E, me, S, nslots, K.ALIGN,
                                   4, recv_cap, back_cap, rows_cap, wsp.data_ptr(), nb, st) == 0
        ws.append(wsp)
        segs.append((wsp[lay[0]:lay[0] + 4 * (S + 1)].view(torch.int32), wsp[lay[1]:lay[1] + 4 * S].view(torch.int32),
                     rows_cap))
        loc, rem = wsp[lay[18]:lay[18] + 8 * S].view(torch.int32), wsp[lay[19]:lay[19] + 16 * S].view(torch.int32)
        groups.append((loc[:S], loc[S:], rem[:2 * S], rem[2 * S:],
                       torch.arange(S, dtype=torch.int32, device=DEV).repeat_interleave(2)))
    epoch = 1
    w1b, w2b = moe._resident_banks()
    xls = [torch.empty(segs[me][2], H, dtype=x.dtype, device=DEV) for me in range(R)]
    hs = [torch.empty(segs[me][2], I, dtype=x.dtype, device=DEV) for me in range(R)]
    banks = []
    for me in range(R):
        sl = torch.tensor(placement.slots[me], dtype=torch.long, device=DEV)
        banks.append((w1b[sl].contiguous(), w2b[sl].contiguous()))
    for me, (lo, hi) in enumerate(bounds):  # dispatch
        S = len(placement.slots[me])
        assert L.rf_moe_ep_devplan_push(ws[me].data_ptr(), R, E, S, nslots, 2 if overlap else 0,
                                        x[lo:hi].data_ptr(), routed[me][3].src_slot.data_ptr(), Kk, row_bytes,
                                        ptrs(recv), flags(0, me), epoch, done.data_ptr() + 4 * me, st) == 0
        if overlap:  # own rows into the GEMM rows, their gated GEMM before the wait
            assert L.rf_moe_ep_devplan_push(ws[me].data_ptr(), R, E, S, nslots, 3, x[lo:hi].data_ptr(),
                                            routed[me][3].src_slot.data_ptr(), Kk, row_bytes, ptrs([xls[me]] * R),
                                            flags(0, me), epoch, done.data_ptr() + 4 * me, st) == 0
            K.grouped_gemm_gated(xls[me], banks[me][0], groups[me][0], groups[me][1], hs[me],
                                 activation=moe.activation)
    for me in range(R):  # expert ranks: regroup, gated GEMM, down GEMM + return
        assert L.rf_moe_ep_wait(ctrl[me].data_ptr(), R, epoch, st) == 0
        S = len(placement.slots[me])
        seg_off, seg_cnt, rows_cap = segs[me]
        xl, h = xls[me], hs[me]
        b1, b2 = banks[me]
        if overlap:
            assert L.rf_moe_ep_devplan_regroup_remote(ws[me].data_ptr(), R, E, S, nslots, recv[me].data_ptr(),
                                                      xl.data_ptr(), row_bytes, st) == 0
            K.grouped_gemm_gated(xl, b1, groups[me][2], groups[me][3], h, slot=groups[me][4],
                                 activation=moe.activation)
        else:
            assert L.rf_moe_ep_devplan_regroup(ws[me].data_ptr(), R, E, S, nslots, recv[me].data_ptr(),
                                               xl.data_ptr(), row_bytes, st) == 0
            K.grouped_gemm_gated(xl, b1, seg_off, seg_cnt, h, activation=moe.activation)
        assert L.rf_moe_ep_devplan_down_return(ws[me].data_ptr(), R, E, S, nslots, h.data_ptr(), b2.data_ptr(),
                                               rows_cap, H, I, _lib.dtype_code(x.dtype), ptrs(back), flags(1, me),
                                               epoch, done.data_ptr() + 4 * me, st) == 0
    outs = []
    sb = moe._shared_banks()
    for me, (lo, hi) in enumerate(bounds):  # token ranks: shared experts + combine
        assert L.rf_moe_ep_wait(ctrl[me].data_ptr() + 4 * R, R, epoch, st) == 0
        w, ids32, sscale, p = routed[me]
        xr = x[lo:hi].contiguous()
        shared_y = K.shared_experts(xr, sb[0], sb[1], moe.activation) if sb is not None else None
        o = torch.empty(hi - lo, H, dtype=x.dtype, device=DEV)
        K.combine(back[me][:(hi - lo) * Kk], p.row_of_slot, w, o, shared_y=shared_y, shared_scale=sscale)
        outs.append(o)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0, "an emulated rank timed out or overflowed its plan"
    return torch.cat(outs)


@pytest.mark.parametrize("R,redundant,overlap", [(8, 0, False), (8, 2, False), (4, 1, False), (8, 2, True),
                                                 (4, 1, True)])
def test_c4_full_size_ep_emulated_matches_single_process(R, redundant, overlap):
    """C4 at its benchmark size split over R expert-parallel ranks emulated on
    one GPU (contiguous expert shards, optionally with hot-expert replicas):
    the concatenated rank outputs equal the single-process layer bit for bit
    (reference contract: reframework/parallel/ep.py:120-150 against
    reframework/moe/moe_layer.py:451-519)."""
    from reframework_b200.parallel.eplb import Placement, place_experts
    from reframework_b200.parallel.ep import shard_range
    cfg = CONFIGS["c4_dsv2lite_ep"]
    d = generate(cfg)
    moe = _layer_from(cfg, d)
    x = d["x"].to(DEV)
    with torch.no_grad():
        ref = moe(x)
        _, ids = moe.route(x)
    shards = [shard_range(cfg.experts, R, r) for r in range(R)]
    if redundant:
        load = torch.bincount(ids.reshape(-1).cpu(), minlength=cfg.experts).numpy()
        placement = place_experts(load, shards, redundant)
        assert sum(len(s) for s in placement.slots) > cfg.experts
    else:
        placement = Placement(tuple(tuple(range(a, b)) for a, b in shards))
    with torch.no_grad():
        got = _emulated_ep_forward(moe, x, R, placement, overlap=overlap)
    assert torch.equal(got, ref), f"R={R} overlap={overlap}: EP output differs from the single-process layer"


def test_c5_full_size_offload_equals_resident():
    """Mixtral-8x22B shape at its benchmark size (H6144 E8 top-2 I16384, 2048
    tokens per step, per-step Dirichlet(0.3) router bias) with the expert
    offload cache of 4 device slots: six steps of the exact streaming forward
    (experts copied from the pinned host pool into evicted slots on the copy
    stream while earlier experts compute) give the resident layer's outputs bit
    for bit — the same kernels over the same rows; the resident layer's parity
    with the reference is checked at full size above (C2) and on the fixtures.
    The cache counts one hit or miss per routed expert and step."""
    cfg = CONFIGS["c5_mixtral22b_offload"]
    d = generate(cfg, device=str(DEV), with_x=False)

    def layer():
        m = FusedMoE(cfg.experts, cfg.top_k, cfg.hidden, cfg.inter, dtype=cfg.dtype,
                     router_dtype=torch.float32, device=DEV)
        with torch.no_grad():
            m.gate.copy_(d["gate"])
            w1b, w2b = m._resident_banks()
            w1b.copy_(d["w1"])
            w2b.copy_(d["w2"])
        return m

    resident, offloaded = layer(), layer()
    cache = offloaded.build_offload_cache(DEV, lru_capacity=4)
    torch.cuda.empty_cache()
    g = torch.Generator(device=DEV).manual_seed(cfg.seed + 101)
    x = torch.randn(cfg.tokens, cfg.hidden, generator=g, device=DEV, dtype=cfg.dtype)
    routed = 0
    with torch.no_grad():
        for s in range(6):
            resident.set_router_bias(d["bias"][s])
            offloaded.set_router_bias(d["bias"][s])
            a = resident(x)
            b = offloaded(x)
            routed += int((torch.bincount(resident.route(x)[1].reshape(-1), minlength=cfg.experts) > 0).sum())
            assert torch.equal(a, b), f"step {s}: offloaded output differs from the resident layer"
    st = cache.stats
    assert st.hits + st.misses == routed
    assert st.misses > 0 and st.hits > 0


@pytest.mark.parametrize("name", ["c2_mixtral_bf16", "c3_qwen_decode"])
def test_full_size_graph_replay_equals_eager(name):
    """The bench configurations' forwards captured in a CUDA graph (the decode
    path's form) replay to the eager forward's bits, twice in a row (the tile
    counters and permute scratch are reused across replays)."""
    from reframework_b200.moe.graph import capture_forward
    cfg = CONFIGS[name]
    d = generate(cfg, device=str(DEV), with_x=False)
    moe = FusedMoE(cfg.experts, cfg.top_k, cfg.hidden, cfg.inter, dtype=cfg.dtype, router_dtype=torch.float32,
                   num_shared_experts=cfg.shared_count, shared_intermediate_size=cfg.shared_inter,
                   shared_expert_gate=cfg.shared_gate, device=DEV)
    with torch.no_grad():
        moe.gate.copy_(d["gate"])
        w1b, w2b = moe._resident_banks()
        w1b.copy_(d["w1"])
        w2b.copy_(d["w2"])
        if cfg.shared_count:
            moe.shared_w1.copy_(d["shared_w1"])
            moe.shared_w2.copy_(d["shared_w2"])
            if cfg.shared_gate:
                moe.shared_gate.copy_(d["shared_gate"])
    if d["bias"] is not None:
        moe.set_router_bias(d["bias"][0])
    del d
    g = torch.Generator(device=DEV).manual_seed(cfg.seed + 101)
    x = torch.randn(cfg.tokens, cfg.hidden, generator=g, device=DEV, dtype=cfg.dtype)
    with torch.no_grad():
        eager = moe(x).clone()
        graphed = capture_forward(moe, x)
        first = graphed(x).clone()
        second = graphed(x).clone()
    assert torch.equal(first, eager) and torch.equal(second, eager)
