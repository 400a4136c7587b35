"""Expert parallelism on GPUs: a 1-rank NCCL group on one GPU (the whole
dispatch / regroup / GEMM / return path with a trivial exchange), and 2-rank
runs (token-sharded and replicated contracts) when two GPUs are visible.
Multi-rank cases run as child processes with a short process-group timeout."""

import os
import socket
import subprocess
import sys

import pytest
import torch

from conftest import ROOT, golden_config, load_golden, max_rel

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _build(cfg, d, dev):
    from reframework_b200.moe import FusedMoE
    moe = FusedMoE(cfg.experts, cfg.top_k, cfg.hidden, cfg.inter, dtype=cfg.dtype,
                   router_dtype=torch.float32, num_shared_experts=cfg.shared_count,
                   shared_intermediate_size=cfg.shared_inter, shared_expert_gate=cfg.shared_gate)
    with torch.no_grad():
        moe.gate.copy_(d["gate"])
        for e in range(cfg.experts):
            moe.experts_w1[e].copy_(d["w1"][e])
            moe.experts_w2[e].copy_(d["w2"][e])
        if cfg.shared_count:
            moe.shared_w1.copy_(d["shared_w1"])
            moe.shared_w2.copy_(d["shared_w2"])
    moe = moe.to(dev)
    if d["bias"] is not None:
        moe.set_router_bias(d["bias"][0])
    return moe


def test_ep_single_rank_matches_fused(cuda_ok):
    import torch.distributed as dist
    from reframework_b200 import _lib
    from reframework_b200.parallel import dist as D
    from reframework_b200.parallel.ep import EPFusedMoE
    from reframework_b200.workloads import generate
    rec = load_golden("c4_mini_bf16")
    cfg = golden_config(rec)
    d = generate(cfg)
    dev = torch.device("cuda", 0)
    D.init(backend="nccl", init_method=f"tcp://127.0.0.1:{_free_port()}", rank=0, world_size=1,
           ep_size=1, timeout_s=60, device_id=dev)
    try:
        full = _build(cfg, d, dev)
        ep = EPFusedMoE.from_full(full, 1, 0, token_sharded=True)
        x = d["x"].to(dev)
        with torch.no_grad():
            a = full(x)
            b = ep(x)
        assert torch.equal(a, b)
        assert max_rel(b, rec["out"]) < 1e-2
        assert int(ep.last_counts_dev.sum()) == cfg.tokens * cfg.top_k  # every pair exchanged
        assert _lib.device_status() == 0
        ep.close()
    finally:
        D.destroy()


WORKER = r"""
import os, sys, torch
sys.path.insert(0, {root!r})
sys.path.insert(0, os.path.join({root!r}, "tests"))
from conftest import golden_config, load_golden, max_rel
from reframework_b200.parallel import dist as D
from reframework_b200.parallel.ep import EPFusedMoE
from reframework_b200.workloads import generate
from test_ep_gpu import _build
rank = int(os.environ["RANK"]); world = int(os.environ["WORLD_SIZE"])
dev = torch.device("cuda", rank)
torch.cuda.set_device(dev)
D.init(backend="nccl", init_method="tcp://127.0.0.1:{port}", rank=rank, world_size=world, ep_size=world,
       timeout_s=60, device_id=dev)
rec = load_golden("c4_mini_bf16")
cfg = golden_config(rec)
d = generate(cfg)
full = _build(cfg, d, dev)
x = d["x"].to(dev)
with torch.no_grad():
    ref = full(x)
    ep_rep = EPFusedMoE.from_full(full, world, rank, token_sharded=False)
    rep = ep_rep(x)   # reference contract
    T = x.shape[0]
    lo, hi = T * rank // world, T * (rank + 1) // world
    ep_sh = EPFusedMoE.from_full(full, world, rank, token_sharded=True)
    shard = ep_sh(x[lo:hi])          # rows cross NVLink as peer stores
    ep_nc = EPFusedMoE.from_full(full, world, rank, token_sharded=True)
    ep_nc.p2p = False
    nccl = ep_nc(x[lo:hi])           # rows through NCCL all-to-alls
    again = ep_sh(x[lo:hi])          # second step on the same peer buffers
assert torch.equal(shard, ref[lo:hi]), "token-sharded rows differ from the single-process layer"
assert torch.equal(nccl, shard) and torch.equal(again, shard), "peer-memory and NCCL exchanges differ"
assert torch.equal(rep, ref), "replicated-contract output differs"
assert max_rel(rep, rec["out"]) < 1e-2
# redundant experts: replica weights fetched from their owners, rows of an
# expert split across its holders; the result must not change by a bit
ep = EPFusedMoE.from_full(full, world, rank, token_sharded=True)
with torch.no_grad():
    ep(x[lo:hi])
    pl = ep.rebalance(redundant=2)
    assert sum(len(s) for s in pl.slots) > cfg.experts  # at least one replica somewhere
    bal = ep(x[lo:hi])
assert torch.equal(bal, ref[lo:hi]), "rebalanced EP output differs"
# an uneven step: the last rank holds every token, the others an empty batch
ep_un = EPFusedMoE.from_full(full, world, rank, token_sharded=True)
ep_un.max_tokens_per_rank = T
mine = x if rank == world - 1 else x[:0]
with torch.no_grad():
    un = ep_un(mine)
assert un.shape == (mine.shape[0], cfg.hidden)
assert torch.equal(un, ref[:mine.shape[0]]), "EP step with an empty rank differs"
ep_un.close()
from reframework_b200 import _lib
assert _lib.device_status() == 0, "a kernel set the device error word"
for m in (ep_rep, ep_sh, ep_nc, ep):
    m.close()
D.barrier()
D.destroy()
print("rank", rank, "ok")
"""


def test_ep_two_ranks_match_single_process(cuda_ok):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    port = _free_port()
    code = WORKER.format(root=ROOT, port=port)
    env = dict(os.environ, WORLD_SIZE="2", NCCL_NVLS_ENABLE="0")
    procs = [subprocess.Popen([sys.executable, "-c", code], env=dict(env, RANK=str(r)),
                              stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True) for r in range(2)]
    outs = []
    for p in procs:
        try:
            out, _ = p.communicate(timeout=240)
        except subprocess.TimeoutExpired:
            p.kill()
            out, _ = p.communicate()
        outs.append(out)
    bad = [r for r, p in enumerate(procs) if p.returncode != 0]
    report = "\n".join(f"--- rank {r} (exit {procs[r].returncode}):\n{outs[r][-2500:]}" for r in range(len(procs)))
    assert not bad, f"ranks {bad} failed:\n{report}"


@pytest.mark.parametrize("R", [40, 64])
def test_device_plan_with_many_holders_matches_host_plan(cuda_ok, R):
    """The device planner splits a replicated expert's rows on one warp (one
    lane per holder) and falls back to its first thread past 32 holders: with
    an expert on every rank, one on 21 ranks and one on 6 (and ranks that hold
    no primary expert), every rank's plan tables equal the host planner's."""
    import numpy as np
    from reframework_b200 import _lib
    from reframework_b200.parallel.ep import shard_range
    L = _lib.lib()
    dev = torch.device("cuda", 0)
    E = 8
    rng = np.random.default_rng(R)
    slots = [list(range(*shard_range(E, R, r))) for r in range(R)]
    for r in range(R):
        if 0 not in slots[r]:
            slots[r].append(0)
        if 8 <= r < 29 and 1 not in slots[r]:
            slots[r].append(1)
        if 30 <= r < 36 and 2 not in slots[r]:
            slots[r].append(2)
    p = np.exp(rng.normal(size=E))
    cnt_np = np.stack([rng.multinomial(int(rng.integers(0, 3000)), p / p.sum()) for _ in range(R)]).astype(np.int32)
    flat = np.ascontiguousarray([e for s in slots for e in s], dtype=np.int32)
    offs = np.ascontiguousarray(np.cumsum([0] + [len(s) for s in slots]), dtype=np.int32)
    cnt = torch.from_numpy(cnt_np).to(dev)
    flat_d, offs_d = torch.from_numpy(flat).to(dev), torch.from_numpy(offs).to(dev)
    M = np.zeros(R * R, np.int64)
    assert L.rf_moe_ep_pair_rows(cnt_np.ctypes.data, R, E, flat.ctypes.data, offs.ctypes.data, 4, M.ctypes.data) == 0
    M = M.reshape(R, R)
    st = torch.cuda.current_stream(dev).cuda_stream
    nslots = int(flat.size)
    cap_recv = int(cnt_np.sum()) + 1
    back_cap = int(cnt_np.sum(1).max()) + 1
    for me in (0, 7, 8, 29, 33, R - 1):
        S = len(slots[me])
        nb = L.rf_moe_ep_devplan_workspace_size(R, E, S, nslots)
        w = torch.zeros(nb, dtype=torch.uint8, device=dev)
        lo = np.zeros(_lib.EP_DEVPLAN_LAYOUT_N, np.int64)
        assert L.rf_moe_ep_devplan_layout(R, E, S, nslots, lo.ctypes.data) == 0
        assert L.rf_moe_ep_devplan(cnt.data_ptr(), flat_d.data_ptr(), offs_d.data_ptr(), R, E, me, S, nslots, 128, 4,
                                   cap_recv, back_cap, cap_recv + S * 128, w.data_ptr(), nb, st) == 0
        torch.cuda.synchronize()
        wb = w.cpu().numpy()
        i64 = lambda off, n: wb[off:off + 8 * n].view(np.int64)  # noqa: E731
        i32 = lambda off, n: wb[off:off + 4 * n].view(np.int32)  # noqa: E731
        send = np.zeros(R, np.int64)
        recvs = np.zeros(R, np.int64)
        hl = np.zeros(15, np.int64)
        buf = np.zeros(4 * int(cnt_np.sum()) + 4096, np.int32)
        assert L.rf_moe_ep_plan(cnt_np.ctypes.data, R, E, me, flat.ctypes.data, offs.ctypes.data, 128, 4,
                                send.ctypes.data, recvs.ctypes.data, buf.ctypes.data, buf.size, hl.ctypes.data) == 0
        assert i32(lo[2], 1)[0] == 0, "device plan overflowed"
        assert np.array_equal(i64(lo[6], R + 1), np.concatenate([[0], np.cumsum(send)]))
        assert np.array_equal(i64(lo[8], R + 1), np.concatenate([[0], np.cumsum(recvs)]))
        assert np.array_equal(i64(lo[7], R), M[:me].sum(0) if me else np.zeros(R))
        assert np.array_equal(i64(lo[9], R), M[:, :me].sum(1) if me else np.zeros(R))
        seg = lambda i: buf[hl[2 * i]:hl[2 * i] + hl[2 * i + 1]]  # noqa: E731
        assert np.array_equal(i32(lo[0], S + 1), seg(2)) and np.array_equal(i32(lo[1], S), seg(3))
        assert i32(lo[10], 1)[0] == hl[13] and i64(lo[11], 1)[0] == hl[12]
    assert _lib.device_status() == 0


@pytest.mark.parametrize("seed", range(4))
def test_device_plan_matches_host_plan_and_round_trips(cuda_ok, seed):
    """rf_moe_ep_devplan == rf_moe_ep_plan / rf_moe_ep_pair_rows for every rank,
    and dispatch -> regroup -> return through the device plan hands every
    (token, slot) its own row back at its permuted row (the combine's layout).  R ranks are emulated on one GPU with
    separate buffers; only the push kernels run (nothing waits here)."""
    import ctypes
    import numpy as np
    from reframework_b200 import _lib
    from reframework_b200 import kernels as K
    from reframework_b200.parallel.ep import shard_range
    from reframework_b200.parallel.eplb import place_experts
    L = _lib.lib()
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(seed)
    R = int(rng.integers(1, 7))
    E = int(rng.integers(R, 3 * R + 4))
    topk = int(rng.integers(1, min(E, 4) + 1))
    H = 64
    shards = [shard_range(E, R, r) for r in range(R)]
    Ts = [int(rng.integers(0, 200)) for _ in range(R)]
    xs, perms = [], []
    g = torch.Generator().manual_seed(seed)
    for r in range(R):
        xs.append(torch.randn(Ts[r], H, generator=g).bfloat16().to(dev))
        ids = torch.stack([torch.randperm(E, generator=g)[:topk] for _ in range(Ts[r])]) if Ts[r] else \
            torch.zeros(0, topk, dtype=torch.int64)
        perms.append(K.permute(ids.int().to(dev), E, align=1))
    cnt = torch.stack([p.counts for p in perms]).contiguous()
    cnt_np = cnt.cpu().numpy().astype(np.int32)
    pl = place_experts(cnt_np.sum(0) + 1, shards, int(rng.integers(0, 3)))
    flat = np.ascontiguousarray([e for s in pl.slots for e in s], dtype=np.int32)
    offs = np.ascontiguousarray(np.cumsum([0] + [len(s) for s in pl.slots]), dtype=np.int32)
    flat_d, offs_d = torch.from_numpy(flat).to(dev), torch.from_numpy(offs).to(dev)
    M = np.zeros(R * R, np.int64)
    assert L.rf_moe_ep_pair_rows(cnt_np.ctypes.data, R, E, flat.ctypes.data, offs.ctypes.data, 4, M.ctypes.data) == 0
    M = M.reshape(R, R)
    row_bytes = H * 2
    st = torch.cuda.current_stream(dev).cuda_stream
    nslots = int(flat.size)
    cap_recv = max(sum(Ts) * topk, 1)
    recv = [torch.zeros(cap_recv, H, dtype=torch.bfloat16, device=dev) for _ in range(R)]
    back = [torch.zeros(max(Ts[r] * topk, 1), H, dtype=torch.bfloat16, device=dev) for r in range(R)]
    ctrl = [torch.zeros(2 * R + 4, dtype=torch.int32, device=dev) for _ in range(R)]
    ws, lay = [], []
    for me in range(R):
        S = len(pl.slots[me])
        nb = L.rf_moe_ep_devplan_workspace_size(R, E, S, nslots)
        w = torch.zeros(nb, dtype=torch.uint8, device=dev)
        lo = np.zeros(_lib.EP_DEVPLAN_LAYOUT_N, np.int64)
        assert L.rf_moe_ep_devplan_layout(R, E, S, nslots, lo.ctypes.data) == 0
        rows_cap = cap_recv + S * 128
        assert L.rf_moe_ep_devplan(cnt.data_ptr(), flat_d.data_ptr(), offs_d.data_ptr(), R, E, me, S, nslots, 128, 4,
                                   cap_recv, max(Ts) * topk, rows_cap, w.data_ptr(), nb, st) == 0
        ws.append(w)
        lay.append(lo)
    torch.cuda.synchronize()
    for me in range(R):
        S = len(pl.slots[me])
        wb, lo = ws[me].cpu().numpy(), lay[me]
        i64 = lambda off, n: wb[off:off + 8 * n].view(np.int64)
        i32 = lambda off, n: wb[off:off + 4 * n].view(np.int32)
        send = np.zeros(R, np.int64)
        recvs = np.zeros(R, np.int64)
        hl = np.zeros(15, np.int64)
        buf = np.zeros(4 * int(cnt_np.sum()) + 4096, np.int32)
        assert L.rf_moe_ep_plan(cnt_np.ctypes.data, R, E, me, flat.ctypes.data, offs.ctypes.data, 128, 4,
                                send.ctypes.data, recvs.ctypes.data, buf.ctypes.data, buf.size, hl.ctypes.data) == 0
        assert i32(lo[2], 1)[0] == 0, "device plan overflowed"
        assert np.array_equal(i64(lo[6], R + 1), np.concatenate([[0], np.cumsum(send)]))
        assert np.array_equal(i64(lo[8], R + 1), np.concatenate([[0], np.cumsum(recvs)]))
        assert np.array_equal(i64(lo[7], R), M[:me].sum(0) if me else np.zeros(R))
        assert np.array_equal(i64(lo[9], R), M[:, :me].sum(1) if me else np.zeros(R))
        seg = lambda i: buf[hl[2 * i]:hl[2 * i] + hl[2 * i + 1]]
        assert np.array_equal(i32(lo[0], S + 1), seg(2)) and np.array_equal(i32(lo[1], S), seg(3))
        assert i32(lo[10], 1)[0] == hl[13] and i64(lo[11], 1)[0] == hl[12]

    def ptrs(ts):
        return (ctypes.c_void_p * R)(*[t.data_ptr() for t in ts])

    done = torch.zeros(R, dtype=torch.int32, device=dev)
    for me in range(R):  # dispatch pushes
        S = len(pl.slots[me])
        flags = (ctypes.c_void_p * R)(*[ctrl[d].data_ptr() + 4 * me for d in range(R)])
        src = xs[me] if Ts[me] else recv[me][:0]
        assert L.rf_moe_ep_devplan_push(ws[me].data_ptr(), R, E, S, nslots, 0, src.data_ptr(),
                                        perms[me].src_slot.data_ptr(), topk, row_bytes, ptrs(recv), flags, 7,
                                        done.data_ptr() + 4 * me, st) == 0
    ys = []
    for me in range(R):  # regroup; the "experts" return their input rows
        S = len(pl.slots[me])
        xl = torch.zeros(cap_recv + S * 128, H, dtype=torch.bfloat16, device=dev)
        assert L.rf_moe_ep_devplan_regroup(ws[me].data_ptr(), R, E, S, nslots, recv[me].data_ptr(), xl.data_ptr(),
                                           row_bytes, st) == 0
        ys.append(xl)
    # the overlapped dispatch (dir 2 to the other ranks into fresh buffers, dir 3
    # own rows straight into the GEMM rows, remote-only regroup) fills the same
    # GEMM rows, and its group tables cover exactly the slot segments
    recv2 = [torch.zeros_like(b) for b in recv]
    ctrl2 = [torch.zeros(R, dtype=torch.int32, device=dev) for _ in range(R)]
    xl2 = [torch.zeros_like(y) for y in ys]
    for me in range(R):
        S = len(pl.slots[me])
        flags = (ctypes.c_void_p * R)(*[ctrl2[d].data_ptr() + 4 * me for d in range(R)])
        src = xs[me] if Ts[me] else recv[me][:0]
        for mode, dst in ((2, ptrs(recv2)), (3, ptrs([xl2[me]] * R))):
            assert L.rf_moe_ep_devplan_push(ws[me].data_ptr(), R, E, S, nslots, mode, src.data_ptr(),
                                            perms[me].src_slot.data_ptr(), topk, row_bytes, dst, flags, 5,
                                            done.data_ptr() + 4 * me, st) == 0
    for me in range(R):
        S = len(pl.slots[me])
        assert L.rf_moe_ep_devplan_regroup_remote(ws[me].data_ptr(), R, E, S, nslots, recv2[me].data_ptr(),
                                                  xl2[me].data_ptr(), row_bytes, st) == 0
    torch.cuda.synchronize()
    assert all(bool((c == 5).all()) for c in ctrl2), "dir 2 raised its flags in every peer"
    for me in range(R):
        S = len(pl.slots[me])
        wb, lo = ws[me].cpu().numpy(), lay[me]
        i32 = lambda off, n: wb[off:off + 4 * n].view(np.int32)
        soff, scnt = i32(lo[0], S + 1), i32(lo[1], S)
        loc, rem = i32(lo[18], 2 * S), i32(lo[19], 4 * S)
        covered = []
        for j in range(S):
            parts = [(int(rem[2 * j]), int(rem[2 * S + 2 * j])), (int(loc[j]), int(loc[S + j])),
                     (int(rem[2 * j + 1]), int(rem[2 * S + 2 * j + 1]))]
            pos = int(soff[j])
            for a, n in parts:  # below this rank, own, above: contiguous, in that order
                assert a == pos and n >= 0, f"rank {me} slot {j}: groups {parts} vs segment {soff[j]}+{scnt[j]}"
                pos += n
            assert pos == soff[j] + scnt[j]
            covered.append(torch.arange(int(soff[j]), pos))
        if covered:
            idx = torch.cat(covered).to(dev)
            assert torch.equal(xl2[me][idx], ys[me][idx]), f"rank {me}: overlapped dispatch rows differ"
    for me in range(R):  # return pushes
        S = len(pl.slots[me])
        flags = (ctypes.c_void_p * R)(*[ctrl[d].data_ptr() + 4 * (R + me) for d in range(R)])
        assert L.rf_moe_ep_devplan_push(ws[me].data_ptr(), R, E, S, nslots, 1, ys[me].data_ptr(), None, 1, row_bytes,
                                        ptrs(back), flags, 7, done.data_ptr() + 4 * me, st) == 0
    for me in range(R):
        if Ts[me] == 0:
            continue
        got = back[me][perms[me].row_of_slot.long()]
        want = xs[me].repeat_interleave(topk, 0)
        assert torch.equal(got, want), f"rank {me}: rows did not come back"
    torch.cuda.synchronize()
    assert all(bool((c[:2 * R] == 7).all()) for c in ctrl), "every rank raised its flags in every peer"

    # the down GEMM with the return exchange in its epilogue stores exactly the
    # rows of "down GEMM, then the return push"
    w2s = [(torch.randn(len(pl.slots[me]), H, H, generator=g) * 0.1).bfloat16().to(dev) for me in range(R)]
    fused = [torch.zeros_like(b) for b in back]
    plain = [torch.zeros_like(b) for b in back]
    for me in range(R):
        S = len(pl.slots[me])
        lo = lay[me]
        seg_off = ws[me][lo[0]:lo[0] + 4 * (S + 1)].view(torch.int32)
        seg_cnt = ws[me][lo[1]:lo[1] + 4 * S].view(torch.int32)
        rows = ys[me].shape[0]
        y = torch.zeros(rows, H, dtype=torch.bfloat16, device=dev)
        K.grouped_gemm_down(ys[me], w2s[me], seg_off, seg_cnt, y)
        flags = (ctypes.c_void_p * R)(*[ctrl[d].data_ptr() + 4 * (R + me) for d in range(R)])
        assert L.rf_moe_ep_devplan_push(ws[me].data_ptr(), R, E, S, nslots, 1, y.data_ptr(), None, 1, row_bytes,
                                        ptrs(plain), flags, 8, done.data_ptr() + 4 * me, st) == 0
        assert L.rf_moe_ep_devplan_down_return(ws[me].data_ptr(), R, E, S, nslots, ys[me].data_ptr(),
                                               w2s[me].data_ptr(), rows, H, H, _lib.dtype_code(torch.bfloat16),
                                               ptrs(fused), flags, 9, done.data_ptr() + 4 * me, st) == 0
    torch.cuda.synchronize()
    for me in range(R):
        n = Ts[me] * topk
        assert torch.equal(fused[me][:n], plain[me][:n]), f"rank {me}: fused return differs"
    assert all(bool((c[R:2 * R] == 9).all()) for c in ctrl), "the fused GEMM raised its flags in every peer"
    assert _lib.device_status() == 0


def test_device_plan_too_small_buffers_move_nothing(cuda_ok):
    """A plan that needs more rows than the receive buffers hold fails on every
    rank at once (the capacity check is global): the error word reads
    RF_DEV_PLAN_OVERFLOW, the GEMM segments are empty, the pushes write no row
    and still raise their flags (so no peer waits out its limit)."""
    import ctypes
    import numpy as np
    from reframework_b200 import _lib
    L = _lib.lib()
    dev = torch.device("cuda", 0)
    R, E, topk, H = 2, 4, 2, 64
    slots = [[0, 1], [2, 3]]
    flat = torch.tensor([e for s in slots for e in s], dtype=torch.int32, device=dev)
    offs = torch.tensor([0, 2, 4], dtype=torch.int32, device=dev)
    Ts = [40, 24]
    cnt = torch.tensor([[20, 20, 20, 20], [12, 12, 12, 12]], dtype=torch.int32, device=dev)  # T*K per rank
    recv_cap = 50  # rank 0 receives 40 + 24 = 64 rows
    st = torch.cuda.current_stream(dev).cuda_stream
    assert _lib.device_status() == 0
    ws, lay = [], []
    for me in range(R):
        nb = L.rf_moe_ep_devplan_workspace_size(R, E, 2, 4)
        w = torch.full((nb,), 0x55, dtype=torch.uint8, device=dev)  # stale bytes everywhere
        lo = np.zeros(_lib.EP_DEVPLAN_LAYOUT_N, np.int64)
        assert L.rf_moe_ep_devplan_layout(R, E, 2, 4, lo.ctypes.data) == 0
        assert L.rf_moe_ep_devplan(cnt.data_ptr(), flat.data_ptr(), offs.data_ptr(), R, E, me, 2, 4, 128, 4,
                                   recv_cap, max(Ts) * topk, recv_cap + 2 * 127, w.data_ptr(), nb, st) == 0
        ws.append(w)
        lay.append(lo)
    assert _lib.device_status() == 3  # RF_DEV_PLAN_OVERFLOW (read and cleared)
    for me in range(R):
        wb, lo = ws[me].cpu().numpy(), lay[me]
        assert wb[lo[2]:lo[2] + 4].view(np.int32)[0] == 1, f"rank {me}: plan not flagged"
        assert not wb[lo[0]:lo[0] + 12].view(np.int32).any() and not wb[lo[1]:lo[1] + 8].view(np.int32).any()
        assert wb[lo[4]:lo[4] + 8].view(np.int64)[0] == 0 and wb[lo[3]:lo[3] + 8].view(np.int64)[0] == 0
    recv = [torch.zeros(recv_cap, H, dtype=torch.bfloat16, device=dev) for _ in range(R)]
    ctrl = [torch.zeros(2 * R, dtype=torch.int32, device=dev) for _ in range(R)]
    done = torch.zeros(R, dtype=torch.int32, device=dev)
    x = torch.randn(max(Ts), H, device=dev).bfloat16()
    src_slot = torch.arange(max(Ts) * topk, dtype=torch.int32, device=dev)
    for me in range(R):
        flags = (ctypes.c_void_p * R)(*[ctrl[d].data_ptr() + 4 * me for d in range(R)])
        assert L.rf_moe_ep_devplan_push(ws[me].data_ptr(), R, E, 2, 4, 0, x.data_ptr(), src_slot.data_ptr(), topk,
                                        H * 2, (ctypes.c_void_p * R)(*[t.data_ptr() for t in recv]), flags, 5,
                                        done.data_ptr() + 4 * me, st) == 0
    torch.cuda.synchronize()
    assert all(not bool(t.any()) for t in recv), "a failed plan moved rows"
    assert all(bool((c[:R] == 5).all()) for c in ctrl), "flags must rise even when nothing moves"
    assert _lib.device_status() == 0


def test_bounded_flag_wait_gives_up_and_reports(cuda_ok):
    """Failure detection on the device without a fault: a stream-ordered wait
    for a flag that no rank ever raises (the picture of a peer that died
    between steps) gives up after its 2 s limit, records RF_DEV_WAIT_TIMEOUT in
    the device error word and returns, so the context and the stream stay
    usable.  Reference analogue: the per-rank timeout of
    reframework/parallel/dist.py:173-175."""
    import time
    from reframework_b200 import _lib
    L = _lib.lib()
    dev = torch.device("cuda", 0)
    assert _lib.device_status() == 0
    flags = torch.zeros(1, dtype=torch.int32, device=dev)
    st = torch.cuda.current_stream(dev).cuda_stream
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    assert L.rf_moe_ep_wait(flags.data_ptr(), 1, 7, st) == 0
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    assert 1.5 < waited < 60, f"the wait gave up after {waited:.2f} s"
    assert _lib.device_status() == 2  # RF_DEV_WAIT_TIMEOUT (read and cleared)
    # the stream still runs work, and a raised flag ends the same wait at once
    v = torch.arange(4096, device=dev, dtype=torch.int64).sum()
    assert int(v) == 4095 * 4096 // 2
    flags.fill_(7)
    t0 = time.perf_counter()
    assert L.rf_moe_ep_wait(flags.data_ptr(), 1, 7, st) == 0
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 1.0
    assert _lib.device_status() == 0
