"""Stage-by-stage parity of the CUDA kernels (through the C ABI) against the
CPU oracle and the reference golden fixtures."""

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from conftest import ULP_REL, golden_config, load_golden, max_rel, routing_mismatches
from oracle import moe_oracle as O
from reframework_b200 import _lib
from reframework_b200 import kernels as K
from reframework_b200.workloads import generate

pytestmark = pytest.mark.gpu
DEV = "cuda"
# tokens whose routed set differs from the golden fixture by a one-ulp logit tie,
# as observed on B200 for every fixture (16-bit and fp32 routers alike)
TIE_SWAPS_SEEN = 0
ROUTE_CASES = ["c1_tiny_fp32", "c2_mini_bf16", "c3_mini_bf16", "c4_mini_bf16", "c4_mini_norenorm",
               "fp16_default", "bf16_gelu_default", "fp32_gelu_tanh", "bf16_entropy_k"]


@pytest.fixture(autouse=True)
def _device_clean(cuda_ok):
    _lib.set_gemm_impl(0)
    yield
    _lib.set_gemm_impl(0)
    assert _lib.device_status() == 0, "a kernel set the device error word"


def _route_inputs(rec):
    cfg = golden_config(rec)
    d = generate(cfg)
    harness = rec["mode"] == "harness"
    bias = d["bias"][0] if (harness and d["bias"] is not None) else None
    round_dtype = None if (harness or cfg.dtype == torch.float32) else cfg.dtype
    return cfg, d, bias, round_dtype


@pytest.mark.parametrize("name", ROUTE_CASES)
def test_router_matches_reference(name):
    rec = load_golden(name)
    cfg, d, bias, rdt = _route_inputs(rec)
    w, ids32, ids64, lg, _ = K.router_topk(
        d["x"].to(DEV), d["gate"].to(DEV), cfg.top_k, renormalize=cfg.renormalize,
        bias=None if bias is None else bias.to(DEV), round_dtype=rdt,
        entropy_k_min=rec.get("entropy_k_min", 0), want_logits=True, ids64=True)
    logits_ref = O.router_logits(d["x"], d["gate"], bias=bias, fp32=rec["mode"] == "harness")
    # no fixture has a tie-swapped token on B200 (measured): any swap fails
    bad = routing_mismatches(ids64, rec["ids"], logits_ref, cfg.top_k, round_dtype=rdt, max_count=TIE_SWAPS_SEEN)
    if rec["mode"] == "harness":
        assert bad == [], "fp32 router: routing must be bit-exact"
    assert torch.equal(ids32.cpu().long(), ids64.cpu())
    ok = torch.ones(rec["ids"].shape[0], dtype=torch.bool)
    ok[bad] = False
    same_order = (ids64.cpu() == rec["ids"]).all(1) & ok
    torch.testing.assert_close(w.cpu()[same_order], rec["weights"][same_order], rtol=2e-5, atol=2e-6)
    ulp = ULP_REL.get(rdt, 1e-5)
    torch.testing.assert_close(lg.cpu(), logits_ref.float(), rtol=max(1e-4, ulp), atol=1e-4)


def test_router_logits_only_mode_matches_torch_fused_topk():
    g = torch.Generator().manual_seed(11)
    logits = torch.randn(300, 60, generator=g)
    for renorm in (True, False):
        w, _, ids, _, _ = K.router_topk(logits.to(DEV), None, 4, renormalize=renorm, ids64=True, ids32=False)
        wr, ir = O.torch_fused_topk(logits, 4, renorm)
        assert torch.equal(ids.cpu(), ir)
        torch.testing.assert_close(w.cpu(), wr, rtol=2e-5, atol=2e-6)


def test_router_shared_gate_sigmoid():
    g = torch.Generator().manual_seed(5)
    x = torch.randn(70, 256, generator=g).bfloat16()
    gate = (torch.randn(16, 256, generator=g) * 0.02).bfloat16()
    sg = (torch.randn(256, generator=g) * 0.02).bfloat16()
    _, _, _, _, ss = K.router_topk(x.to(DEV), gate.to(DEV), 2, shared_gate=sg.to(DEV))
    ref = torch.sigmoid(x.float() @ sg.float())
    torch.testing.assert_close(ss.cpu(), ref, rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("E,H", [(8, 4096), (60, 2048), (64, 2048), (130, 512)])
def test_router_tensor_core_path_matches_cuda_cores(E, H):
    """16-bit gates run the logits on the tensor cores; the CUDA-core kernel
    (forced with set_gemm_impl(1)) computes the same fp32 sums in another
    order: logits agree to fp32 rounding, the shared gate too, and top-k only
    differs where two probabilities are within that rounding."""
    g = torch.Generator().manual_seed(E + H)
    T = 333
    x = torch.randn(T, H, generator=g).bfloat16().to(DEV)
    cat = (torch.randn(E + 1, H, generator=g) * 0.02).bfloat16().to(DEV)
    gate, sg = cat[:E], cat[E]            # adjacent: the tensor-core path
    res = []
    for impl in (0, 1):
        _lib.set_gemm_impl(impl)
        res.append(K.router_topk(x, gate, 4, shared_gate=sg, want_logits=True, ids64=True))
    (w0, _, i0, l0, s0), (w1, _, i1, l1, s1) = res
    scale = l1.abs().max().item()
    assert (l0 - l1).abs().max().item() <= 1e-5 * scale
    torch.testing.assert_close(s0, s1, rtol=1e-5, atol=1e-6)
    p = torch.softmax(l1, -1)
    kth = p.topk(5, -1).values
    near_tie = (kth[:, 3] - kth[:, 4]) < 1e-5
    same = (i0 == i1).all(1)
    assert bool((same | near_tie).all())


@pytest.mark.parametrize("dtype,E", [(torch.bfloat16, 61), (torch.float16, 8), (torch.float32, 61)])
def test_router_is_batch_invariant(dtype, E):
    """A token's logits, ids and weights do not depend on how many other tokens
    share the call (tensor-core path for 16-bit, CUDA-core slices for fp32)."""
    g = torch.Generator().manual_seed(7)
    H = 1024
    x = torch.randn(300, H, generator=g).to(dtype).to(DEV)
    cat = (torch.randn(E + 1, H, generator=g) * 0.02).to(dtype).to(DEV)
    full = K.router_topk(x, cat[:E], 4, shared_gate=cat[E], want_logits=True, ids64=True)
    for lo, hi in ((0, 37), (123, 300), (5, 6)):
        part = K.router_topk(x[lo:hi].contiguous(), cat[:E], 4, shared_gate=cat[E], want_logits=True,
                             ids64=True)
        for a, b in zip(full, part):
            if a is not None:
                assert torch.equal(a[lo:hi], b)


@pytest.mark.parametrize("name", ["c1_tiny_fp32", "c2_mini_bf16", "c3_mini_bf16", "c4_mini_bf16", "fp16_default"])
def test_permute_matches_reference_order(name):
    rec = load_golden(name)
    cfg = golden_config(rec)
    d = generate(cfg)
    ids = rec["ids"]
    T, Kk = ids.shape
    x = d["x"].to(DEV)
    p = K.permute(ids.to(DEV, torch.int32), cfg.experts, x=x)
    counts, order = O.permutation(ids.numpy(), cfg.experts)
    off = p.offsets.cpu().numpy()
    assert np.array_equal(p.counts.cpu().numpy(), counts)
    assert np.all(off[:-1] % K.ALIGN == 0)
    src = p.src_slot.cpu().numpy()
    ros = p.row_of_slot.cpu().numpy()
    pos = 0
    for e in range(cfg.experts):
        seg = src[off[e]:off[e] + counts[e]]
        assert np.array_equal(seg, order[pos:pos + counts[e]]), f"expert {e} order"
        assert np.all(src[off[e] + counts[e]:off[e + 1]] == -1)
        pos += counts[e]
    assert np.array_equal(src[ros], np.arange(T * Kk))
    xp = p.x_perm.cpu()
    rows = torch.from_numpy(src[:off[-1]]).long()
    valid = rows >= 0
    assert torch.equal(xp[:off[-1]][valid], d["x"][rows[valid] // Kk])
    assert torch.count_nonzero(xp[:off[-1]][~valid]) == 0


@pytest.mark.parametrize("align", [1, 128])
@pytest.mark.parametrize("T,Kk,E", [(1, 1, 1), (37, 3, 5), (20000, 6, 64), (4096, 2, 8), (0, 2, 8)])
def test_permute_random_stable(T, Kk, E, align):
    g = torch.Generator().manual_seed(T + E)
    ids = torch.randint(0, E, (T, Kk), generator=g, dtype=torch.int32)
    if T > 10:
        ids[: T // 3] = 0  # a heavy expert spanning several blocks
    p = K.permute(ids.to(DEV), E, align=align)
    counts, order = O.permutation(ids.numpy(), E)
    assert np.array_equal(p.counts.cpu().numpy(), counts)
    off = p.offsets.cpu().numpy()
    src = p.src_slot.cpu().numpy()
    got = np.concatenate([src[off[e]:off[e] + counts[e]] for e in range(E)]) if T else np.zeros(0)
    assert np.array_equal(got, order)


@pytest.mark.parametrize("align", [1, 64, 128, 256])
@pytest.mark.parametrize("T,Kk,E,dtype", [
    (1, 1, 1, torch.bfloat16), (37, 3, 5, torch.float32), (64, 4, 60, torch.bfloat16),
    (256, 4, 256, torch.float16),   # the largest decode-sized case: 1024 pairs, 256 experts
    (256, 4, 257, torch.bfloat16),  # one expert past it: separate scatter and gather launches
    (300, 4, 60, torch.bfloat16),   # 1200 pairs: several blocks
])
def test_permute_with_gather_random(T, Kk, E, dtype, align):
    """The permute with its row gather (one launch for decode-sized calls, two
    or three otherwise): the stable order of the oracle, x_perm rows equal to
    the token rows, zeros on pad rows, and every pair's row."""
    g = torch.Generator().manual_seed(T * 7 + E)
    ids = torch.randint(0, E, (T, Kk), generator=g, dtype=torch.int32)
    if T > 10:
        ids[: T // 3, 0] = E - 1  # a heavy expert
    x = torch.randn(T, 96, generator=g).to(dtype)
    p = K.permute(ids.to(DEV), E, align=align, x=x.to(DEV))
    counts, order = O.permutation(ids.numpy(), E)
    assert np.array_equal(p.counts.cpu().numpy(), counts)
    off = p.offsets.cpu().numpy()
    assert np.all(off[:-1] % align == 0) and off[-1] == sum((c + align - 1) // align * align for c in counts)
    src = p.src_slot.cpu().numpy()
    ros = p.row_of_slot.cpu().numpy()
    got = np.concatenate([src[off[e]:off[e] + counts[e]] for e in range(E)])
    assert np.array_equal(got, order)
    assert np.array_equal(src[ros], np.arange(T * Kk))
    used = int(off[-1])
    rows = torch.from_numpy(src[:used]).long()
    valid = rows >= 0
    assert int(valid.sum()) == T * Kk
    xp = p.x_perm.cpu()[:used]
    assert torch.equal(xp[valid], x[rows[valid] // Kk])
    assert torch.count_nonzero(xp[~valid]) == 0


def test_bad_expert_id_in_decode_permute_with_gather():
    ids = torch.tensor([[0, 9], [3, 1]], dtype=torch.int32, device=DEV)  # 9 >= E
    x = torch.randn(2, 64, dtype=torch.bfloat16, device=DEV)
    p = K.permute(ids, 4, x=x)
    assert p.row_of_slot.cpu().tolist()[1] == -1
    assert p.counts.cpu().tolist() == [1, 1, 0, 1]
    assert _lib.device_status() == 1


def _segments(counts, align=128):
    offs = [0]
    for c in counts:
        offs.append(offs[-1] + (c + align - 1) // align * align)
    return offs


def _torch_grouped(a, w1, w2, counts, offs, act, slot=None):
    h_ref, y_ref = {}, {}
    I = w2.shape[2]
    for e, c in enumerate(counts):
        if c == 0:
            continue
        s = e if slot is None else slot[e]
        xa = a[offs[e]:offs[e] + c].float()
        gu = (xa @ w1[s].float().t()).to(a.dtype)  # the reference stores the GEMM output in the layer dtype
        h = O.gated_act_and_mul(act, gu).float()
        h_ref[e] = h
        y_ref[e] = h.to(a.dtype).float() @ w2[s].float().t()
    return h_ref, y_ref


@pytest.mark.parametrize("impl", [0, 1, 2, 3, 4, 5])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("H,I,counts,act", [
    (256, 256, [130, 0, 1, 300], "silu"),
    (320, 384, [128, 257, 5], "gelu"),
    (1024, 1408, [700, 64, 129, 3, 0, 256], "silu"),
    (512, 136, [90, 400], "gelu_tanh"),
])
def test_grouped_gemms_vs_torch(impl, dtype, H, I, counts, act):
    _lib.set_gemm_impl(impl)
    g = torch.Generator().manual_seed(H + I)
    E = len(counts)
    offs = _segments(counts)
    rows = offs[-1] + 3
    a = torch.randn(rows, H, generator=g).to(dtype)
    w1 = (torch.randn(E, 2 * I, H, generator=g) * 0.05).to(dtype)
    w2 = (torch.randn(E, H, I, generator=g) * 0.05).to(dtype)
    off_t = torch.tensor(offs, dtype=torch.int32, device=DEV)
    cnt_t = torch.tensor(counts, dtype=torch.int32, device=DEV)
    h = torch.zeros(rows, I, dtype=dtype, device=DEV)
    y = torch.zeros(rows, H, dtype=dtype, device=DEV)
    K.grouped_gemm_gated(a.to(DEV), w1.to(DEV), off_t, cnt_t, h, activation=act)
    K.grouped_gemm_down(h, w2.to(DEV), off_t, cnt_t, y)
    h_ref, y_ref = _torch_grouped(a, w1, w2, counts, offs, act)
    hc, yc = h.cpu(), y.cpu()
    for e, c in enumerate(counts):
        if c == 0:
            continue
        assert max_rel(hc[offs[e]:offs[e] + c], h_ref[e]) < 8e-3, f"h expert {e}"
        assert max_rel(yc[offs[e]:offs[e] + c], y_ref[e]) < 8e-3, f"y expert {e}"
        # rows past the expert's count are never written
        assert torch.count_nonzero(hc[offs[e] + c:offs[e + 1]]) == 0


@pytest.mark.parametrize("act", ["silu", "gelu"])
@pytest.mark.parametrize("H,I,counts", [
    (1024, 1408, [700, 64, 129, 3, 0, 256]),   # prefill-like: several m-blocks per expert
    (2048, 1408, [5, 1, 0, 9, 2, 4, 0, 7]),     # decode-like: a few rows per expert
])
def test_tile_width_is_bitwise_invariant(H, I, counts, act):
    """Tile widths 256 / 128 / 64 run the same MMA chain per output element,
    so the automatic per-launch choice never changes a result bit (the
    expert-parallel layer, whose launches see fewer rows, relies on this)."""
    g = torch.Generator().manual_seed(H * 7 + I)
    dtype = torch.bfloat16
    E = len(counts)
    offs = _segments(counts)
    rows = offs[-1]
    a = torch.randn(rows, H, generator=g).to(dtype).to(DEV)
    w1 = (torch.randn(E, 2 * I, H, generator=g) * 0.05).to(dtype).to(DEV)
    w2 = (torch.randn(E, H, I, generator=g) * 0.05).to(dtype).to(DEV)
    off_t = torch.tensor(offs, dtype=torch.int32, device=DEV)
    cnt_t = torch.tensor(counts, dtype=torch.int32, device=DEV)
    outs = []
    for impl in (2, 3, 4):
        _lib.set_gemm_impl(impl)
        h = torch.zeros(rows, I, dtype=dtype, device=DEV)
        y = torch.zeros(rows, H, dtype=dtype, device=DEV)
        K.grouped_gemm_gated(a, w1, off_t, cnt_t, h, activation=act)
        K.grouped_gemm_down(h, w2, off_t, cnt_t, y)
        outs.append((h, y))
    for h, y in outs[1:]:
        assert torch.equal(h, outs[0][0]) and torch.equal(y, outs[0][1])


@pytest.mark.parametrize("act", ["silu", "gelu_tanh"])
@pytest.mark.parametrize("H,I,counts", [
    (1024, 1408, [700, 64, 129, 3, 0, 256]),
    (2048, 1408, [5, 1, 0, 9, 2, 4, 0, 7]),
    (512, 136, [90, 400, 17]),                  # feature blocks past I and H
])
def test_pair_kernel_matches_single_cta_kernel(H, I, counts, act):
    """The CTA-pair kernel (weights on the MMA's M side, tokens on N) against
    the single-CTA kernel: every output element is an fp32 sum over the same
    64-deep k-blocks of 16-wide MMA steps; the two must agree within the
    rounding of one fp32 accumulation order (bit-identical outputs expected
    for most elements), and the pair kernel must not write rows past an
    expert's count."""
    g = torch.Generator().manual_seed(H * 3 + I)
    dtype = torch.bfloat16
    E = len(counts)
    offs = _segments(counts)
    rows = offs[-1]
    a = torch.randn(rows, H, generator=g).to(dtype).to(DEV)
    w1 = (torch.randn(E, 2 * I, H, generator=g) * 0.05).to(dtype).to(DEV)
    w2 = (torch.randn(E, H, I, generator=g) * 0.05).to(dtype).to(DEV)
    off_t = torch.tensor(offs, dtype=torch.int32, device=DEV)
    cnt_t = torch.tensor(counts, dtype=torch.int32, device=DEV)
    outs = []
    for impl in (2, 5):
        _lib.set_gemm_impl(impl)
        h = torch.zeros(rows, I, dtype=dtype, device=DEV)
        y = torch.zeros(rows, H, dtype=dtype, device=DEV)
        K.grouped_gemm_gated(a, w1, off_t, cnt_t, h, activation=act)
        K.grouped_gemm_down(outs[0][0] if outs else h, w2, off_t, cnt_t, y)  # same h into both down GEMMs
        outs.append((h, y))
    (h2, y2), (h5, y5) = outs
    same_h = float((h2 == h5).float().mean())
    same_y = float((y2 == y5).float().mean())
    print(f"pair vs single-CTA: identical h {same_h:.4f}, y {same_y:.4f}")
    assert max_rel(h5, h2) < 8e-3 and max_rel(y5, y2) < 8e-3
    for e, c in enumerate(counts):
        assert torch.count_nonzero(h5[offs[e] + c:offs[e + 1]]) == 0
        assert torch.count_nonzero(y5[offs[e] + c:offs[e + 1]]) == 0


def test_pair_kernel_tile_claims_concurrent_launches_and_counter_reuse():
    """The CTA-pair kernel claims its tiles from a per-launch counter: launches
    running at the same time on different streams (each holding part of the
    GPU, so pairs start late) and more launches in a row than there are
    counters must all give the bits of a lone launch."""
    g = torch.Generator().manual_seed(77)
    dtype = torch.bfloat16
    counts = [300, 17, 0, 256, 90, 5, 128, 40]
    E, H, I = len(counts), 1024, 704
    offs = _segments(counts)
    rows = offs[-1]
    a = torch.randn(rows, H, generator=g).to(dtype).to(DEV)
    w1 = (torch.randn(E, 2 * I, H, generator=g) * 0.05).to(dtype).to(DEV)
    w2 = (torch.randn(E, H, I, generator=g) * 0.05).to(dtype).to(DEV)
    off_t = torch.tensor(offs, dtype=torch.int32, device=DEV)
    cnt_t = torch.tensor(counts, dtype=torch.int32, device=DEV)
    _lib.set_gemm_impl(0)
    h_ref = torch.zeros(rows, I, dtype=dtype, device=DEV)
    y_ref = torch.zeros(rows, H, dtype=dtype, device=DEV)
    K.grouped_gemm_gated(a, w1, off_t, cnt_t, h_ref)
    K.grouped_gemm_down(h_ref, w2, off_t, cnt_t, y_ref)
    torch.cuda.synchronize()
    streams = [torch.cuda.Stream(device=DEV) for _ in range(3)]
    outs = []
    for rep in range(24):  # 24 x 3 streams x 2 launches: every counter row used more than once
        hs, ys = [], []
        for st in streams:
            st.wait_stream(torch.cuda.current_stream(DEV))
            with torch.cuda.stream(st):
                h = torch.zeros(rows, I, dtype=dtype, device=DEV)
                y = torch.zeros(rows, H, dtype=dtype, device=DEV)
                K.grouped_gemm_gated(a, w1, off_t, cnt_t, h)
                K.grouped_gemm_down(h, w2, off_t, cnt_t, y)
            hs.append(h)
            ys.append(y)
        for st in streams:
            torch.cuda.current_stream(DEV).wait_stream(st)
        outs.append((hs, ys))
    torch.cuda.synchronize()
    for hs, ys in outs:
        for h, y in zip(hs, ys):
            assert torch.equal(h, h_ref) and torch.equal(y, y_ref)
    assert _lib.device_status() == 0


@pytest.mark.parametrize("impl", [0, 1, 2, 5])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_down_gemm_addend_rounds_like_the_reference(impl, dtype):
    """rf_moe_grouped_gemm_down_add: out = round(addend + round(h . w2^T)) in
    the layer dtype, bit for bit what two separately rounded shared-expert
    outputs summed in that dtype give (in place, addend == out, too)."""
    if dtype == torch.float32 and impl not in (0, 1):
        pytest.skip("fp32 layers run on CUDA cores only")
    _lib.set_gemm_impl(impl)
    g = torch.Generator().manual_seed(21)
    T, H, I = 300, 512, 384
    h = torch.randn(T, I, generator=g).to(dtype).to(DEV)
    w2 = (torch.randn(1, H, I, generator=g) * 0.05).to(dtype).to(DEV)
    add = torch.randn(T, H, generator=g).to(dtype).to(DEV)
    off, cnt = K.dense_segment(DEV, T)
    y = torch.empty(T, H, dtype=dtype, device=DEV)
    K.grouped_gemm_down(h, w2, off, cnt, y)
    want = (add.float() + y.float()).to(dtype)
    got = torch.empty_like(y)
    K.grouped_gemm_down(h, w2, off, cnt, got, addend=add)
    assert torch.equal(got, want)
    inplace = add.clone()
    K.grouped_gemm_down(h, w2, off, cnt, inplace, addend=inplace)
    assert torch.equal(inplace, want)


def test_grouped_gemm_slot_table_and_groups():
    """Experts read through an expert->slot table, only the listed groups run."""
    g = torch.Generator().manual_seed(3)
    dtype = torch.bfloat16
    H, I, counts = 256, 256, [100, 200, 50, 130]
    E = len(counts)
    offs = _segments(counts)
    a = torch.randn(offs[-1], H, generator=g).to(dtype)
    S = 6
    w1 = (torch.randn(S, 2 * I, H, generator=g) * 0.05).to(dtype)
    w2 = (torch.randn(S, H, I, generator=g) * 0.05).to(dtype)
    slot = [4, 0, 5, 2]
    groups = [3, 1]
    h = torch.zeros(offs[-1], I, dtype=dtype, device=DEV)
    y = torch.zeros(offs[-1], H, dtype=dtype, device=DEV)
    kw = dict(slot=torch.tensor(slot, dtype=torch.int32, device=DEV),
              groups=torch.tensor(groups, dtype=torch.int32, device=DEV))
    off_t = torch.tensor(offs, dtype=torch.int32, device=DEV)
    cnt_t = torch.tensor(counts, dtype=torch.int32, device=DEV)
    K.grouped_gemm_gated(a.to(DEV), w1.to(DEV), off_t, cnt_t, h, **kw)
    K.grouped_gemm_down(h, w2.to(DEV), off_t, cnt_t, y, **kw)
    h_ref, y_ref = _torch_grouped(a, w1, w2, counts, offs, "silu", slot=slot)
    yc = y.cpu()
    for e in range(E):
        seg = yc[offs[e]:offs[e] + counts[e]]
        if e in groups:
            assert max_rel(seg, y_ref[e]) < 8e-3
        else:
            assert torch.count_nonzero(seg) == 0


def test_fp32_grouped_gemm_tolerance():
    """fp32 layers run on CUDA cores with fp32 FMA: within 1e-4 of fp64."""
    g = torch.Generator().manual_seed(9)
    H, I, counts = 1024, 2816, [20, 0, 75, 33]
    offs = _segments(counts)
    a = torch.randn(offs[-1], H, generator=g)
    w1 = torch.randn(len(counts), 2 * I, H, generator=g) * 0.02
    w2 = torch.randn(len(counts), H, I, generator=g) * 0.02
    off_t = torch.tensor(offs, dtype=torch.int32, device=DEV)
    cnt_t = torch.tensor(counts, dtype=torch.int32, device=DEV)
    h = torch.zeros(offs[-1], I, device=DEV)
    y = torch.zeros(offs[-1], H, device=DEV)
    K.grouped_gemm_gated(a.to(DEV), w1.to(DEV), off_t, cnt_t, h)
    K.grouped_gemm_down(h, w2.to(DEV), off_t, cnt_t, y)
    for e, c in enumerate(counts):
        if c == 0:
            continue
        xa = a[offs[e]:offs[e] + c].double()
        hr = O.gated_act_and_mul("silu", xa @ w1[e].double().t())
        yr = hr @ w2[e].double().t()
        assert max_rel(y.cpu()[offs[e]:offs[e] + c], yr) < 1e-4


@pytest.mark.parametrize("impl", [0, 2, 3, 4])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("T,topk,E", [(300, 2, 8), (64, 4, 60), (1000, 6, 16), (5, 1, 3)])
def test_gated_gemm_with_fused_gather_is_bitwise_equal(impl, dtype, T, topk, E):
    """The gated GEMM fetching token rows with TMA gather4 (no expert-ordered
    copy) multiplies the same rows as the explicit gather + gated GEMM."""
    _lib.set_gemm_impl(impl)
    g = torch.Generator().manual_seed(T + topk + E)
    H, I = 512, 384
    x = torch.randn(T, H, generator=g).to(dtype).to(DEV)
    ids = torch.stack([torch.randperm(E, generator=g)[:topk] for _ in range(T)]).int().to(DEV)
    w1 = (torch.randn(E, 2 * I, H, generator=g) * 0.05).to(dtype).to(DEV)
    p = K.permute(ids, E, x=x)
    ref = torch.zeros(p.rows_cap, I, dtype=dtype, device=DEV)
    K.grouped_gemm_gated(p.x_perm, w1, p.offsets, p.counts, ref)
    out = torch.zeros(p.rows_cap, I, dtype=dtype, device=DEV)
    assert K.grouped_gemm_gated_gather(x, p.src_slot, topk, w1, p.offsets, p.counts, out)
    assert torch.equal(out, ref)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("counts", [[20, 0, 75, 33], [1, 2, 3, 17, 0, 16, 5, 40]])
def test_simt_skinny_and_tiled_kernels_agree_bitwise(dtype, counts):
    """The CUDA-core path picks its skinny kernel when the row capacity implies
    few rows per expert and its tiled kernel otherwise; both run the same fp32
    FMA chain per output, so a larger buffer (tiled) gives the same bits."""
    _lib.set_gemm_impl(1)
    g = torch.Generator().manual_seed(len(counts))
    H, I = 512, 704
    E = len(counts)
    offs = _segments(counts)
    a = torch.randn(offs[-1], H, generator=g).to(dtype).to(DEV)
    w1 = (torch.randn(E, 2 * I, H, generator=g) * 0.05).to(dtype).to(DEV)
    w2 = (torch.randn(E, H, I, generator=g) * 0.05).to(dtype).to(DEV)
    off_t = torch.tensor(offs, dtype=torch.int32, device=DEV)
    cnt_t = torch.tensor(counts, dtype=torch.int32, device=DEV)
    res = []
    for extra in (0, 16384):  # capacity for few rows -> skinny; a large one -> tiled
        rows = offs[-1] + extra
        ap = torch.zeros(rows, H, dtype=dtype, device=DEV)
        ap[:offs[-1]] = a
        h = torch.zeros(rows, I, dtype=dtype, device=DEV)
        y = torch.zeros(rows, H, dtype=dtype, device=DEV)
        K.grouped_gemm_gated(ap, w1, off_t, cnt_t, h)
        K.grouped_gemm_down(h, w2, off_t, cnt_t, y)
        res.append((h[:offs[-1]], y[:offs[-1]]))
    assert torch.equal(res[0][0], res[1][0]) and torch.equal(res[0][1], res[1][1])


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_combine_vs_torch(dtype):
    g = torch.Generator().manual_seed(1)
    T, Kk, H, rows = 50, 3, 512, 400
    y = torch.randn(rows, H, generator=g).to(dtype)
    ros = torch.randperm(rows, generator=g)[: T * Kk].int()
    ros[7] = -1  # a dropped slot contributes nothing
    w = torch.rand(T, Kk, generator=g)
    sy = torch.randn(T, H, generator=g).to(dtype)
    ss = torch.rand(T, generator=g)
    res = torch.randn(T, H, generator=g).to(dtype)
    kw = dict(shared_y=sy.to(DEV), shared_scale=ss.to(DEV), residual=res.to(DEV))
    # precise mode: fp32 accumulation, one rounding
    out = torch.empty(T, H, dtype=dtype, device=DEV)
    K.combine(y.to(DEV), ros.to(DEV), w.to(DEV), out, precise=True, **kw)
    yy = torch.where(ros.view(T, Kk, 1) >= 0, y.float()[ros.long().clamp_min(0)].view(T, Kk, H), 0)
    ref = (yy * w.unsqueeze(-1)).sum(1) + ss.unsqueeze(-1) * sy.float() + res.float()
    tol = 1e-6 if dtype == torch.float32 else 8e-3
    assert max_rel(out.cpu(), ref) < tol
    # default mode: the reference's rounding points, rows in ascending row (= expert) order
    out = torch.empty(T, H, dtype=dtype, device=DEV)
    K.combine(y.to(DEV), ros.to(DEV), w.to(DEV), out, **kw)
    emu = torch.zeros(T, H, dtype=dtype)
    for t in range(T):
        slots = sorted((int(ros[t * Kk + k]), k) for k in range(Kk) if int(ros[t * Kk + k]) >= 0)
        for r, k in slots:
            emu[t] = emu[t] + y[r] * w[t, k].to(dtype)
    emu = emu + (sy.float() * ss.unsqueeze(-1)).to(dtype)
    emu = emu + res
    assert torch.equal(out.cpu(), emu)


def test_gather_rows_roundtrip():
    g = torch.Generator().manual_seed(2)
    src = torch.randn(100, 96, generator=g).bfloat16().to(DEV)
    idx = torch.tensor([5, -1, 99, 0, 5], dtype=torch.int32, device=DEV)
    out = torch.full((5, 96), 7.0, dtype=torch.bfloat16, device=DEV)
    K.gather_rows(src, idx, out)
    assert torch.equal(out[0], src[5]) and torch.equal(out[2], src[99]) and torch.equal(out[3], src[0])
    assert torch.count_nonzero(out[1]) == 0


def test_bad_expert_id_is_reported_not_faulted():
    ids = torch.tensor([[0, 9]], dtype=torch.int32, device=DEV)  # 9 >= E
    p = K.permute(ids, 4)
    assert p.row_of_slot.cpu().tolist()[1] == -1
    assert _lib.device_status() == 1
