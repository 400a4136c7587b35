"""Expert-parallel host logic on CPU: dispatch plan arithmetic, and the
all-to-all exchange over world_size-2 gloo ranks (the expert compute is a
test-side stand-in; the GPU kernels are covered by the gpu tests)."""

import os
import socket

import numpy as np
import pytest
import torch

from oracle import moe_oracle as O
from reframework_b200.parallel import dist as D
from reframework_b200.parallel.ep import plan_dispatch, plan_exchange, shard_range
from reframework_b200.parallel.eplb import place_experts, split_rows


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_shard_range_matches_reference():
    for E, R in [(8, 2), (8, 8), (64, 8), (10, 4), (3, 4), (60, 8)]:
        spans = [shard_range(E, R, r) for r in range(R)]
        assert spans == [O.shard_range(E, R, r) for r in range(R)]
        assert spans[0][0] == 0 and spans[-1][1] == E
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))


def test_plan_dispatch_indices_are_consistent():
    rng = np.random.default_rng(0)
    E, R = 10, 4
    shards = [shard_range(E, R, r) for r in range(R)]
    cnt = rng.integers(0, 50, size=(R, E))
    cnt[1, 3] = 0
    for rank in range(R):
        pl = plan_dispatch(cnt, rank, shards)
        s, e = shards[rank]
        assert pl.send_splits == [int(cnt[rank, a:b].sum()) for a, b in shards]
        assert pl.recv_splits == [int(cnt[r, s:e].sum()) for r in range(R)]
        assert np.all(pl.local_offsets[:-1] % 128 == 0)
        inv = pl.inverse_index
        assert len(set(inv.tolist())) == inv.size  # injective
        assert np.array_equal(pl.gather_index[inv], np.arange(inv.size))
        assert (pl.gather_index >= 0).sum() == pl.recv_total
        # each received row lands in its expert's segment, sources in rank order
        pos = 0
        for r in range(R):
            for j in range(e - s):
                n = int(cnt[r, s + j])
                dst = inv[pos:pos + n]
                lo = pl.local_offsets[j] + int(cnt[:r, s + j].sum())
                assert np.array_equal(dst, np.arange(lo, lo + n))
                pos += n


def test_plan_with_more_ranks_than_experts():
    cnt = np.array([[3, 1], [0, 2], [5, 0]])
    shards = [shard_range(2, 3, r) for r in range(3)]
    pl = plan_dispatch(cnt, 2, shards)  # rank 2 owns no expert
    assert pl.recv_total == 0 and pl.rows_capacity == 0
    assert pl.send_splits == [5, 0, 0]


def _exchange_worker(rank, ctx, E, T, Kk, seed, redundant):
    torch.manual_seed(seed + rank)
    H = 16
    ids = torch.randint(0, E, (T, Kk), dtype=torch.int64)
    ids[: T // 2, 0] = 0  # skew: expert 0 is hot on every rank
    x = torch.randn(T, H)
    counts, order = O.permutation(ids.numpy(), E)
    x_perm = x[torch.from_numpy(order // Kk)]
    expert_of_row = ids.reshape(-1)[torch.from_numpy(order)]
    R = ctx.world_size
    shards = [shard_range(E, R, r) for r in range(R)]
    gathered = D.all_gather(torch.from_numpy(counts).int())
    cnt = torch.stack(gathered).numpy()
    placement = place_experts(cnt.sum(0), shards, redundant)
    quota = split_rows(cnt, placement) if redundant else None
    plan = plan_exchange(cnt, rank, placement, quota)
    send = x_perm if plan.send_index is None else x_perm[torch.from_numpy(plan.send_index).long()]
    recv = torch.empty(plan.recv_total, H)
    D.all_to_all_v(recv, send, plan.recv_splits, plan.send_splits)
    # stand-in expert compute on the regrouped rows: y = x * (1 + global expert of the slot)
    gi = torch.from_numpy(plan.gather_index[:plan.rows_capacity]).long()
    xl = torch.where((gi >= 0).unsqueeze(1), recv[gi.clamp_min(0)] if plan.recv_total else torch.zeros(gi.numel(), H),
                     torch.zeros(1, H))
    y = torch.zeros_like(xl)
    for j, e in enumerate(placement.slots[rank]):
        lo = int(plan.local_offsets[j])
        n = int(plan.local_counts[j])
        y[lo:lo + n] = xl[lo:lo + n] * (1 + e)
    y_send = y[torch.from_numpy(plan.inverse_index).long()] if plan.recv_total else torch.empty(0, H)
    y_back = torch.empty(T * Kk, H)
    D.all_to_all_v(y_back, y_send, plan.send_splits, plan.recv_splits)
    if plan.send_index is not None:
        y_perm = torch.empty_like(y_back)
        y_perm[torch.from_numpy(plan.send_index).long()] = y_back
        y_back = y_perm
    expect = x_perm * (1 + expert_of_row.float()).unsqueeze(1)
    assert torch.equal(y_back, expect), f"rank {rank}: rows did not come back to their slots"
    if redundant:
        # every rank's computed row count is within one expert-run of the mean
        loads = quota.sum(axis=0)
        assert loads.max() - loads.min() <= max(2, cnt.sum() // 4)


@pytest.mark.parametrize("E,T,Kk,redundant", [(8, 40, 2, 0), (5, 33, 3, 0), (1, 7, 1, 0), (8, 64, 2, 1),
                                              (4, 50, 2, 2)])
def test_ep_exchange_gloo_world2(E, T, Kk, redundant):
    D.run(_exchange_worker, world_size=2, backend="gloo",
          init_method=f"tcp://127.0.0.1:{_free_port()}", ep_size=2, args=(E, T, Kk, 3, redundant))


@pytest.mark.parametrize("seed", range(12))
def test_native_planner_matches_numpy_planner(seed):
    """rf_moe_ep_plan (C++, in the library) == plan_exchange + split_rows (numpy)."""
    import ctypes
    from reframework_b200 import _lib
    rng = np.random.default_rng(seed)
    R = int(rng.integers(1, 9))
    E = int(rng.integers(R, 3 * R + 3))
    shards = [shard_range(E, R, r) for r in range(R)]
    probs = rng.dirichlet(np.full(E, 0.5))
    cnt = np.stack([rng.multinomial(int(rng.integers(0, 300)), probs) for _ in range(R)]).astype(np.int32)
    redundant = int(rng.integers(0, 3))
    pl = place_experts(cnt.sum(0) + 1, shards, redundant)
    flat = np.ascontiguousarray([e for s in pl.slots for e in s], dtype=np.int32)
    offs = np.ascontiguousarray(np.cumsum([0] + [len(s) for s in pl.slots]), dtype=np.int32)
    for rank in range(R):
        quota = split_rows(cnt, pl, rounds=4) if sum(len(s) for s in pl.slots) > E else None
        ref = plan_exchange(cnt, rank, pl, quota)
        send = np.zeros(R, np.int64)
        recv = np.zeros(R, np.int64)
        lay = np.zeros(15, np.int64)
        buf = np.zeros(4 * int(cnt.sum()) + 2048, np.int32)
        rc = _lib.lib().rf_moe_ep_plan(cnt.ctypes.data, R, E, rank, flat.ctypes.data, offs.ctypes.data, 128, 4,
                                       send.ctypes.data, recv.ctypes.data, buf.ctypes.data, buf.size,
                                       lay.ctypes.data)
        assert rc == 0, _lib.lib().rf_moe_last_error()
        seg = lambda i: buf[lay[2 * i]:lay[2 * i] + lay[2 * i + 1]]
        assert list(send) == ref.send_splits and list(recv) == ref.recv_splits
        assert lay[12] == ref.rows_capacity
        assert np.array_equal(seg(0)[:max(ref.rows_capacity, 1)], ref.gather_index[:max(ref.rows_capacity, 1)])
        assert np.array_equal(seg(1), ref.inverse_index)
        assert np.array_equal(seg(2), ref.local_offsets) and np.array_equal(seg(3), ref.local_counts)
        if ref.send_index is None:
            assert lay[13] == 1
        else:
            assert lay[13] == 0 and np.array_equal(seg(4), ref.send_index)
            assert np.array_equal(seg(5)[seg(4)], np.arange(seg(4).size))


@pytest.mark.parametrize("seed", range(8))
def test_pair_rows_matrix_matches_every_ranks_plan(seed):
    """rf_moe_ep_pair_rows: row s = rank s's send splits, column d = rank d's
    receive splits (so one-sided pushes land where the all-to-all would put them)."""
    from reframework_b200 import _lib
    rng = np.random.default_rng(100 + seed)
    R = int(rng.integers(1, 9))
    E = int(rng.integers(R, 3 * R + 3))
    shards = [shard_range(E, R, r) for r in range(R)]
    cnt = np.stack([rng.multinomial(int(rng.integers(0, 300)), rng.dirichlet(np.full(E, 0.5)))
                    for _ in range(R)]).astype(np.int32)
    pl = place_experts(cnt.sum(0) + 1, shards, int(rng.integers(0, 3)))
    flat = np.ascontiguousarray([e for s in pl.slots for e in s], dtype=np.int32)
    offs = np.ascontiguousarray(np.cumsum([0] + [len(s) for s in pl.slots]), dtype=np.int32)
    M = np.zeros(R * R, np.int64)
    assert _lib.lib().rf_moe_ep_pair_rows(cnt.ctypes.data, R, E, flat.ctypes.data, offs.ctypes.data, 4,
                                          M.ctypes.data) == 0
    M = M.reshape(R, R)
    for rank in range(R):
        send = np.zeros(R, np.int64)
        recv = np.zeros(R, np.int64)
        lay = np.zeros(15, np.int64)
        buf = np.zeros(4 * int(cnt.sum()) + 2048, np.int32)
        assert _lib.lib().rf_moe_ep_plan(cnt.ctypes.data, R, E, rank, flat.ctypes.data, offs.ctypes.data, 128, 4,
                                         send.ctypes.data, recv.ctypes.data, buf.ctypes.data, buf.size,
                                         lay.ctypes.data) == 0
        assert np.array_equal(M[rank], send) and np.array_equal(M[:, rank], recv)


def test_native_planner_reports_small_buffer():
    from reframework_b200 import _lib
    cnt = np.array([[5, 3], [2, 7]], np.int32)
    flat = np.array([0, 1], np.int32)
    offs = np.array([0, 1, 2], np.int32)
    send, recv, lay = np.zeros(2, np.int64), np.zeros(2, np.int64), np.zeros(15, np.int64)
    buf = np.zeros(2, np.int32)
    rc = _lib.lib().rf_moe_ep_plan(cnt.ctypes.data, 2, 2, 0, flat.ctypes.data, offs.ctypes.data, 128, 4,
                                   send.ctypes.data, recv.ctypes.data, buf.ctypes.data, buf.size, lay.ctypes.data)
    assert rc == 1 and lay[14] > 2 and "needs" in _lib.lib().rf_moe_last_error().decode()


def test_place_experts_and_split_rows_balance():
    """On the C2-like skew over 8 ranks, 2 replica slots per rank bring the
    busiest rank within ~15 % of the mean (contiguous sharding alone: 2.3x)."""
    load = np.array([1041, 959, 1817, 1128, 2319, 518, 149, 261]) * 8
    R = 8
    shards = [shard_range(8, R, r) for r in range(R)]
    base = load.max() / (load.sum() / R)
    assert base > 2.0
    pl = place_experts(load, shards, redundant=2)
    assert all(len(set(s)) == len(s) for s in pl.slots)
    assert all(s[0] == shards[r][0] for r, s in enumerate(pl.slots))  # primaries first
    cnt = np.tile(load // R, (R, 1))
    q = split_rows(cnt, pl)
    assert np.array_equal(q.sum(axis=1), cnt.sum(axis=0))  # every row assigned once
    holders = pl.holders(8)
    for e in range(8):
        assert all(q[e, h] == 0 for h in range(R) if h not in holders[e])
    ratio = q.sum(axis=0).max() / (cnt.sum() / R)
    assert ratio < 1.15, ratio


def _ctx_worker(rank, ctx):
    assert ctx.ep_rank == rank and ctx.world_size == 2 and D.get_rank() == rank
    t = torch.tensor([rank + 1.0])
    D.all_reduce_sum(t)
    assert float(t) == 3.0
    chunks = D.all_to_all(torch.tensor([10.0 * rank, 10.0 * rank + 1]))
    assert chunks.tolist() == [rank, 10 + rank]


def test_dist_context_and_collectives_gloo():
    D.run(_ctx_worker, world_size=2, backend="gloo", init_method=f"tcp://127.0.0.1:{_free_port()}", ep_size=2)


def _failing_worker(rank, ctx):
    if rank == 1:
        raise SystemExit(3)


def test_run_reports_failed_rank():
    with pytest.raises(RuntimeError, match="exit codes"):
        D.run(_failing_worker, world_size=2, backend="gloo", init_method=f"tcp://127.0.0.1:{_free_port()}")


def test_current_without_group_raises():
    D.destroy()
    with pytest.raises(RuntimeError, match="No process group"):
        D.current()


# ------------------------------------------------ device planner, run on the host
def _aligned_bytes(n):
    buf = np.zeros(n + 16, np.uint8)
    off = (-buf.ctypes.data) % 16
    return buf[off:off + n]


def _devplan_host(cnt, flat, offs, R, E, me, align, recv_cap, back_cap, rows_cap, S=None):
    """rf_moe_ep_devplan's planner (same source) on the host: (status, ws, layout)."""
    import ctypes
    from reframework_b200 import _lib
    L = _lib.lib()
    S = int(offs[me + 1] - offs[me]) if S is None else S
    nslots = int(flat.size)
    nb = L.rf_moe_ep_devplan_workspace_size(R, E, S, nslots)
    ws = _aligned_bytes(nb)
    ws[:] = 0x55  # stale bytes: every table the row kernels read must be written
    lay = np.zeros(_lib.EP_DEVPLAN_LAYOUT_N, np.int64)
    assert L.rf_moe_ep_devplan_layout(R, E, S, nslots, lay.ctypes.data) == 0
    st = ctypes.c_int32(-1)
    assert L.rf_moe_ep_devplan_host(cnt.ctypes.data, flat.ctypes.data, offs.ctypes.data, R, E, me, S, nslots, align,
                                    4, recv_cap, back_cap, rows_cap, ws.ctypes.data, nb, ctypes.byref(st)) == 0
    return st.value, ws, lay


def _find_le(a, v):
    """Largest index k with a[k] <= v (a ascending, a[0] <= v) — the row kernels' lookup."""
    return np.searchsorted(a, v, side="right") - 1


def _random_case(rng, max_r):
    R = int(rng.integers(1, max_r + 1))
    E = int(rng.integers(R, 3 * R + 4))
    K = int(rng.integers(1, min(E, 4) + 1))
    shards = [shard_range(E, R, r) for r in range(R)]
    Ts = [int(rng.integers(0, 120)) if rng.random() > 0.1 else 0 for _ in range(R)]
    cnt = np.zeros((R, E), np.int32)
    for r in range(R):  # each token routes to K distinct experts, skewed
        p = rng.dirichlet(np.full(E, 0.4))
        for _ in range(Ts[r]):
            cnt[r, rng.choice(E, size=K, replace=False, p=p)] += 1
    pl = place_experts(cnt.sum(0) + 1, shards, int(rng.integers(0, 4)))
    flat = np.ascontiguousarray([e for s in pl.slots for e in s], dtype=np.int32)
    offs = np.ascontiguousarray(np.cumsum([0] + [len(s) for s in pl.slots]), dtype=np.int32)
    return R, E, K, Ts, cnt, pl, flat, offs


@pytest.mark.parametrize("seed", range(40))
def test_device_planner_on_host_matches_host_plan_and_round_trips(seed):
    """The device planner's own code (compiled for the host) against the host
    planner for every rank, then the dispatch / regroup / return index math of
    the row kernels replayed over its tables: every (token, slot) row comes back
    to its own permuted row on its own rank, each exactly once, and every GEMM
    segment holds only rows of its slot's expert."""
    from reframework_b200 import _lib
    L = _lib.lib()
    rng = np.random.default_rng(1000 + seed)
    R, E, K, Ts, cnt, pl, flat, offs = _random_case(rng, 64 if seed % 10 == 9 else 12)
    align = 128 if seed % 2 else 1
    recv_cap = max(int(cnt.sum()), 1)
    back_cap = max(max(Ts) * K, 1)
    M = np.zeros(R * R, np.int64)
    assert L.rf_moe_ep_pair_rows(cnt.ctypes.data, R, E, flat.ctypes.data, offs.ctypes.data, 4, M.ctypes.data) == 0
    M = M.reshape(R, R)
    cpre = np.concatenate([np.zeros((R, 1), np.int64), np.cumsum(cnt, axis=1)], axis=1)
    plans = []
    for me in range(R):
        S = int(offs[me + 1] - offs[me])
        st, wb, lo = _devplan_host(cnt, flat, offs, R, E, me, align, recv_cap, back_cap, recv_cap + S * align)
        assert st == 0, f"rank {me}: status {st}"
        i64 = lambda off, n: wb[off:off + 8 * n].view(np.int64)
        i32 = lambda off, n: wb[off:off + 4 * n].view(np.int32)
        send = np.zeros(R, np.int64)
        recvs = np.zeros(R, np.int64)
        hl = np.zeros(15, np.int64)
        buf = np.zeros(4 * int(cnt.sum()) + 4096, np.int32)
        assert L.rf_moe_ep_plan(cnt.ctypes.data, R, E, me, flat.ctypes.data, offs.ctypes.data, align, 4,
                                send.ctypes.data, recvs.ctypes.data, buf.ctypes.data, buf.size, hl.ctypes.data) == 0
        assert i32(lo[2], 1)[0] == 0
        send_off, recv_off = i64(lo[6], R + 1), i64(lo[8], R + 1)
        assert np.array_equal(send_off, np.concatenate([[0], np.cumsum(send)]))
        assert np.array_equal(recv_off, np.concatenate([[0], np.cumsum(recvs)]))
        assert np.array_equal(i64(lo[7], R), M[:me].sum(0) if me else np.zeros(R))
        assert np.array_equal(i64(lo[9], R), M[:, :me].sum(1) if me else np.zeros(R))
        seg = lambda i: buf[hl[2 * i]:hl[2 * i] + hl[2 * i + 1]]
        assert np.array_equal(i32(lo[0], S + 1), seg(2)) and np.array_equal(i32(lo[1], S), seg(3))
        assert i32(lo[10], 1)[0] == hl[13] and i64(lo[11], 1)[0] == hl[12]
        npc = int(i32(lo[17], 1)[0])
        plans.append(dict(S=S, send_off=send_off, recv_off=recv_off, dst_row0=i64(lo[7], R),
                          loff=i32(lo[0], S + 1).astype(np.int64), lcount=i32(lo[1], S).astype(np.int64),
                          cs=i64(lo[12], R * (S + 1)).reshape(R, S + 1), cj=i64(lo[13], S * (R + 1)).reshape(S, R + 1),
                          ps=i64(lo[14], R * S).reshape(R, S), piece_pos=i64(lo[15], npc + 1),
                          piece_src=i64(lo[16], npc), n_send=int(i64(lo[4], 1)[0]),
                          piece_slot=i32(lo[20], npc).astype(np.int64), loc=i32(lo[18], 2 * S).astype(np.int64),
                          rem=i32(lo[19], 4 * S).astype(np.int64)))
    # dispatch: tag = source * 2^20 + its permuted row
    recv = [np.full(max(int(recv_off_d[-1]), 1), -1, np.int64) for recv_off_d in (p["recv_off"] for p in plans)]
    for s, p in enumerate(plans):
        assert p["n_send"] == Ts[s] * K
        i = np.arange(p["n_send"])
        if not i.size:
            continue
        k = _find_le(p["piece_pos"][:-1], i)
        src_row = p["piece_src"][k] + i - p["piece_pos"][k]
        d = _find_le(p["send_off"][:R], i)
        drow = p["dst_row0"][d] + i - p["send_off"][d]
        assert np.array_equal(np.sort(src_row), np.arange(Ts[s] * K)), "every routed row is sent once"
        for dd in np.unique(d):
            recv[dd][drow[d == dd]] = (s << 20) + src_row[d == dd]
    back = [np.full(max(T * K, 1), -1, np.int64) for T in Ts]
    for me, p in enumerate(plans):
        assert (recv[me][:p["recv_off"][-1]] >= 0).all(), f"rank {me}: receive rows left unwritten"
        for j in range(p["S"]):
            e = int(flat[offs[me] + j])
            k = np.arange(p["lcount"][j])
            if not k.size:
                continue
            s = _find_le(p["cj"][j, :R], k)
            q = p["recv_off"][s] + p["cs"][s, j] + k - p["cj"][j, s]
            rows = recv[me][q]  # regroup: GEMM rows of slot j
            src, prow = rows >> 20, rows & ((1 << 20) - 1)
            assert np.array_equal(src, s)
            assert ((cpre[src, e] <= prow) & (prow < cpre[src, e + 1])).all(), f"slot {j} holds another expert's rows"
            drow = p["ps"][s, j] + k - p["cj"][j, s]  # fused return: the source's permuted row
            for ss in np.unique(s):
                assert (back[ss][drow[s == ss]] == -1).all(), "a return row written twice"
                back[ss][drow[s == ss]] = rows[s == ss]
    for s in range(R):
        assert np.array_equal(back[s][:Ts[s] * K], (s << 20) + np.arange(Ts[s] * K)), f"rank {s}: round trip"
    # the overlapped dispatch: dir 3 puts this rank's own rows straight into its
    # GEMM rows, the remote-only regroup fills the rest; together they give the
    # GEMM rows of the plain regroup, and the group tables split each slot's
    # segment into the rows below / of / above this rank
    for me, p in enumerate(plans):
        S, loff, lcount = p["S"], p["loff"], p["lcount"]
        xl = np.full(max(int(loff[-1]), 1), -1, np.int64)
        i = np.arange(p["send_off"][me], p["send_off"][me + 1])
        if i.size:
            k = _find_le(p["piece_pos"][:-1], i)
            src_row = p["piece_src"][k] + i - p["piece_pos"][k]
            js = p["piece_slot"][k]
            drow = loff[js] + p["cj"][js, me] + i - p["piece_pos"][k]
            assert (xl[drow] == -1).all(), "an own row placed twice"
            xl[drow] = (me << 20) + src_row
        for j in range(S):
            k = np.arange(lcount[j])
            s = _find_le(p["cj"][j, :R], k)
            q = p["recv_off"][s] + p["cs"][s, j] + k - p["cj"][j, s]
            rem = s != me
            assert (xl[loff[j] + k[rem]] == -1).all()
            xl[loff[j] + k[rem]] = recv[me][q[rem]]
            want = recv[me][q]
            assert np.array_equal(xl[loff[j]:loff[j] + lcount[j]], want), f"rank {me} slot {j}: overlapped rows"
            lo_, own, hi = p["cj"][j, me], p["cj"][j, me + 1] - p["cj"][j, me], lcount[j] - p["cj"][j, me + 1]
            assert (p["rem"][2 * j], p["rem"][2 * S + 2 * j]) == (loff[j], lo_)
            assert (p["loc"][j], p["loc"][S + j]) == (loff[j] + lo_, own)
            assert (p["rem"][2 * j + 1], p["rem"][2 * S + 2 * j + 1]) == (loff[j] + lo_ + own, hi)


def test_device_planner_on_host_rejects_bad_placements_and_small_buffers():
    """Status codes of the planner's own checks (host build of the same source):
    a plan that needs more rows than the buffers hold fails on every rank with
    RF_DEV_PLAN_OVERFLOW and empty segments; a broken placement fails with
    RF_DEV_BAD_EXPERT_ID."""
    R, E = 2, 4
    cnt = np.array([[20, 20, 20, 20], [12, 12, 12, 12]], np.int32)
    flat = np.array([0, 1, 2, 3], np.int32)
    offs = np.array([0, 2, 4], np.int32)
    for me in range(R):  # rank 0 receives 64 rows, capacity 50: both ranks' plans fail
        st, wb, lo = _devplan_host(cnt, flat, offs, R, E, me, 1, 50, 80, 400)
        assert st == 3
        assert wb[lo[2]:lo[2] + 4].view(np.int32)[0] == 1
        assert not wb[lo[0]:lo[0] + 12].view(np.int32).any() and not wb[lo[1]:lo[1] + 8].view(np.int32).any()
        assert wb[lo[4]:lo[4] + 8].view(np.int64)[0] == 0
        assert not wb[lo[18]:lo[18] + 16].view(np.int32).any() and not wb[lo[19]:lo[19] + 32].view(np.int32).any()
    st, *_ = _devplan_host(cnt, flat, offs, R, E, 0, 1, 64, 79, 400)  # rank 0's 80 return rows, capacity 79
    assert st == 3
    st, *_ = _devplan_host(cnt, flat, offs, R, E, 0, 128, 64, 80, 64 + 127)  # GEMM rows: 2 x 128 > 191
    assert st == 3
    st, *_ = _devplan_host(cnt, flat, offs, R, E, 0, 1, 64, 80, 400)
    assert st == 0
    bad = [
        (np.array([0, 1, 2, 7], np.int32), offs, None),          # expert id out of range
        (np.array([0, 0, 2, 3], np.int32), offs, None),          # expert 0 twice on rank 0, expert 1 nowhere
        (np.array([0, 1, 2, 2, 3], np.int32), np.array([0, 2, 5], np.int32), None),  # rank 1 holds expert 2 twice
        (flat, np.array([0, 2, 3], np.int32), None),             # offsets end before n_slots
        (flat, offs, 3),                                         # S differs from the placement
    ]
    for fl, of, S in bad:
        st, wb, lo = _devplan_host(cnt, fl, of, R, E, 0, 1, 64, 80, 400, S=S)
        assert st == 1, (fl, of, S)
        assert wb[lo[2]:lo[2] + 4].view(np.int32)[0] == 1


def _waterfill_scalar(n, base):
    """The planner's split of n rows over holders with current loads `base`
    (waterfill_dev in csrc/ep_devplan.cu, the host planner's steps)."""
    m = len(base)
    order = sorted(range(m), key=lambda i: (base[i], i))
    loads = [base[o] for o in order]
    k = m
    while k > 1 and n + sum(loads[:k]) <= loads[k - 1] * k:
        k -= 1
    level = (n + sum(loads[:k])) // k
    give = [max(level - loads[i], 0) if i < k else 0 for i in range(m)]
    rem = n - sum(give)
    i = 0
    while rem > 0:
        give[i % k] += 1
        i += 1
        rem -= 1
    out = [0] * m
    for pos in range(m):
        out[order[pos]] = give[pos]
    return out


def _waterfill_by_rank(n, base):
    """The same split in the per-holder form the device planner's warp uses
    (waterfill_warp): each holder's stable rank and the sorted-load prefix up
    to it, the cut-off as the largest position whose holder still takes rows,
    then the level and the remainder for the first sorted positions."""
    m = len(base)
    rank = [sum(1 for j in range(m) if base[j] < base[i] or (base[j] == base[i] and j < i)) for i in range(m)]
    upto = [sum(base[j] for j in range(m) if rank[j] <= rank[i]) for i in range(m)]
    k = max([rank[i] + 1 for i in range(m) if rank[i] >= 1 and not (n + upto[i] <= base[i] * (rank[i] + 1))],
            default=1)
    pk = next(upto[i] for i in range(m) if rank[i] == k - 1)
    level = (n + pk) // k
    give = [max(level - base[i], 0) if rank[i] < k else 0 for i in range(m)]
    rem = n - sum(give)
    if rem > 0:
        give = [g + (rem // k + (1 if rank[i] < rem % k else 0)) if rank[i] < k else g for i, g in enumerate(give)]
    return give


def test_warp_split_formulation_equals_the_scalar_water_filling():
    """The device planner splits a replicated expert's rows with one warp lane
    per holder; its per-holder formulation gives the scalar split's rows on
    random loads with ties, zeros and large values (the GPU tests then compare
    the device plans with the host planner's)."""
    rng = np.random.default_rng(5)
    for _ in range(20000):
        m = int(rng.integers(1, 33))
        hi = int(rng.choice([3, 10, 1000, 10 ** 9]))
        base = [int(v) for v in rng.integers(0, hi + 1, size=m)]
        n = int(rng.integers(0, int(rng.choice([5, 100, 10 ** 6, 10 ** 10])) + 1))
        assert _waterfill_by_rank(n, base) == _waterfill_scalar(n, base), (n, base)
