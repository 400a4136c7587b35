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
