"""Expert parallelism: experts sharded across ranks, tokens exchanged all-to-all.

Drop-in for reframework/parallel/ep.py (``shard_range``, ``EPFusedMoE``,
``ep_enabled``).  The reference replicates every token on every rank, masks
non-local slots to weight 0 and SUM-all-reduces the full ``[T, H]`` output
(ep.py:120-150).  Here each rank routes only its own tokens and the rows move
to the rank that owns their expert:

  1. router + stable permute of this rank's (token, slot) pairs by global
     expert (compact layout: rows for rank r are one contiguous range, since
     experts are sharded contiguously);
  2. counts exchange (all_gather of the per-expert counts [E]) — the one host
     synchronisation, needed for the all-to-all split sizes;
  3. dispatch: NCCL all_to_all_single of the permuted rows;
  4. regroup the received rows by local expert (128-row aligned segments, one
     gather kernel), grouped gated GEMM, grouped down GEMM;
  5. return the expert rows with the inverse gather and the reverse
     all_to_all_single; the combine (weights, shared experts, residual) runs on
     the tokens' own rank.

Two calling conventions:
  * ``token_sharded=False`` (default; the reference's contract): every rank is
    given the same ``x`` and returns the full output.  Each rank takes a
    contiguous slice of the tokens, runs the exchange above, and the slices are
    all-gathered.
  * ``token_sharded=True``: each rank passes and receives only its own tokens
    (no all-gather) — the data-parallel-attention layout.
Routing is computed with the same kernel and replicated gate on every rank, so
per token it is bit-identical to the single-process ``FusedMoE``.
"""

from __future__ import annotations

import time
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np
import torch
import torch.distributed as tdist
import torch.nn as nn

from .. import kernels as K
from .. import _lib as _lib_mod
from .._lib import ACTIVATIONS, RfMoeError, check, dtype_code, lib, stream_of
from ..moe.keys import expert_tensor
from ..moe.moe_layer import FusedMoE, _bank_view, adjacent_router_weights, reference_output
from . import dist as _dist
from .eplb import Placement, place_experts, split_rows

__all__ = ["shard_range", "EPFusedMoE", "ep_enabled", "DispatchPlan", "plan_dispatch", "plan_exchange"]


def ep_enabled() -> bool:
    """True when a live process group has ``ep_size > 1`` (ep.py:40-42)."""
    return _dist.is_initialized() and _dist.current().ep_size > 1


def shard_range(num_experts: int, ep_size: int, ep_rank: int) -> Tuple[int, int]:
    """Contiguous ``[start, end)`` expert block of ``ep_rank``; the first
    ``num_experts % ep_size`` ranks take one extra expert (ep.py:45-55)."""
    base, rem = divmod(num_experts, ep_size)
    size = base + (1 if ep_rank < rem else 0)
    start = ep_rank * base + min(ep_rank, rem)
    return start, start + size


@dataclass
class DispatchPlan:
    """Host-side bookkeeping of one exchange, from the [R, E] routed-row counts."""

    send_splits: List[int]       # rows this rank sends to each rank
    recv_splits: List[int]       # rows this rank receives from each rank
    local_counts: np.ndarray     # [slots] rows per local expert slot (all sources)
    local_offsets: np.ndarray    # [slots + 1] aligned segment starts
    rows_capacity: int           # rows of the regrouped GEMM buffer
    gather_index: np.ndarray     # [rows_capacity] GEMM row -> received row (-1 = pad)
    inverse_index: np.ndarray    # [recv_total] received row -> GEMM row
    send_index: Optional[np.ndarray] = None  # send position -> permuted row (None = identity)

    @property
    def recv_total(self) -> int:
        return int(sum(self.recv_splits))

    @property
    def send_total(self) -> int:
        return int(sum(self.send_splits))


def plan_exchange(counts_all: np.ndarray, rank: int, placement: Placement,
                  quota: Optional[np.ndarray] = None, align: int = K.ALIGN) -> DispatchPlan:
    """Split sizes and index maps of one exchange, for rank ``rank``.

    ``counts_all[r, e]``: rows rank r routes to expert e (its compact permuted
    rows are expert-major).  ``placement.slots[d]`` lists the experts rank d
    computes; ``quota[e, d]`` how many of expert e's rows rank d takes (default:
    every expert's rows go to its only holder).  An expert's rows are enumerated
    source-major, and holders (by ascending rank) take consecutive runs.
    Rank r sends, to each destination d in turn, its runs for d's slots in d's
    slot order; rank d receives source-major, slot-minor, and regroups them
    slot-major with each slot's segment starting on an ``align`` boundary.
    """
    cnt = np.asarray(counts_all, dtype=np.int64)
    R, E = cnt.shape
    if quota is None:
        quota = np.zeros((E, R), dtype=np.int64)
        for r, ss in enumerate(placement.slots):
            quota[list(ss), r] = cnt[:, list(ss)].sum(axis=0)
        if np.any(quota.sum(axis=1) != cnt.sum(axis=0)):
            raise ValueError("replicated experts need an explicit quota")
    quota = np.asarray(quota, dtype=np.int64)
    # expert e's holders take consecutive runs in rank order: holder h covers
    # global rows [lo[e,h], lo[e,h] + quota[e,h]) (empty for non-holders)
    lo = np.cumsum(quota, axis=1) - quota             # [E, R]
    hi = lo + quota
    src_base = (np.cumsum(cnt, axis=0) - cnt).T       # [E, R] first global row of source r's rows of e
    src_end = src_base + cnt.T
    # run length / offset of expert e's rows that source r sends holder h: [E, R(src), R(holder)]
    a = np.maximum(lo[:, None, :], src_base[:, :, None])
    b = np.minimum(hi[:, None, :], src_end[:, :, None])
    length = np.maximum(0, b - a)
    offset = a - src_base[:, :, None]
    seg_start = np.cumsum(cnt[rank]) - cnt[rank]      # my compact segment starts
    slot_e = [np.asarray(ss, dtype=np.int64) for ss in placement.slots]
    starts = np.concatenate([seg_start[ss] + offset[ss, rank, d] for d, ss in enumerate(slot_e)])
    lens = np.concatenate([length[ss, rank, d] for d, ss in enumerate(slot_e)])
    send_splits = [int(length[ss, rank, d].sum()) for d, ss in enumerate(slot_e)]
    keep = lens > 0
    starts, lens = starts[keep], lens[keep]
    pos = np.cumsum(lens) - lens
    send_index = None
    if np.any(starts != pos):
        send_index = (np.repeat(starts - pos, lens) + np.arange(int(lens.sum()))).astype(np.int32)
    my = placement.slots[rank]
    c = length[slot_e[rank], :, rank].T.reshape(R, len(my))  # [R(src), slots]
    recv_splits = [int(x) for x in c.sum(axis=1)]
    local_counts = c.sum(axis=0) if my else np.zeros(0, dtype=np.int64)
    padded = (local_counts + align - 1) // align * align
    local_offsets = np.concatenate([[0], np.cumsum(padded)]).astype(np.int64)
    total = int(c.sum())
    rows_cap = int(local_offsets[-1]) if my else 0
    sizes = c.reshape(-1)                            # receive order: source-major, slot-minor
    recv_block_start = np.concatenate([[0], np.cumsum(sizes)[:-1]]) if sizes.size else sizes
    dst_block_start = (local_offsets[:-1][None, :] + np.cumsum(c, axis=0) - c).reshape(-1)
    blk = np.repeat(np.arange(sizes.size), sizes)
    within = np.arange(total) - np.repeat(recv_block_start, sizes)
    inverse = (dst_block_start[blk] + within).astype(np.int32)
    gather = np.full(max(rows_cap, 1), -1, dtype=np.int32)
    gather[inverse] = np.arange(total, dtype=np.int32)
    return DispatchPlan(send_splits, recv_splits, local_counts, local_offsets, rows_cap, gather, inverse,
                        send_index)


def plan_dispatch(counts_all: np.ndarray, rank: int, shards: Sequence[Tuple[int, int]],
                  align: int = K.ALIGN) -> DispatchPlan:
    """Exchange plan for plain contiguous sharding (each expert on one rank)."""
    placement = Placement(tuple(tuple(range(a, b)) for a, b in shards))
    return plan_exchange(counts_all, rank, placement, None, align)


class EPFusedMoE(nn.Module):
    """Expert-sharded MoE layer with the same forward / state-dict contract as
    the reference ``EPFusedMoE`` (ep.py:58-179)."""

    def __init__(self, cfg, ep_size: int, ep_rank: int, *, token_sharded: bool = False,
                 router_dtype: Optional[torch.dtype] = None, device: Optional[torch.device] = None,
                 group=None) -> None:
        super().__init__()
        self.cfg = cfg
        self.ep_size = ep_size
        self.ep_rank = ep_rank
        self.token_sharded = token_sharded
        self.num_experts = cfg.num_experts
        self.top_k = cfg.num_experts_per_tok
        self.hidden_size = cfg.hidden_size
        self.intermediate_size = cfg.moe_inter
        self.activation = getattr(cfg, "moe_activation", "silu")
        self.renormalize = getattr(cfg, "moe_renormalize", True)
        self.dtype = cfg.dtype
        self.router_dtype = router_dtype
        self.group = group
        if self.activation not in ACTIVATIONS:
            raise ValueError(f"unknown gated activation {self.activation!r}")
        E, H, I = self.num_experts, self.hidden_size, self.intermediate_size
        fk = {"dtype": self.dtype, "device": device}
        self.gate = nn.Parameter(torch.empty(E, H, **fk))
        self.shards = [shard_range(E, ep_size, r) for r in range(ep_size)]
        self.local_start, self.local_end = self.shards[ep_rank]
        self.local_count = self.local_end - self.local_start
        n = self.local_count
        w1 = torch.empty(n, 2 * I, H, **fk)
        w2 = torch.empty(n, H, I, **fk)
        self.experts_w1 = nn.ParameterList([nn.Parameter(w1[j]) for j in range(n)])
        self.experts_w2 = nn.ParameterList([nn.Parameter(w2[j]) for j in range(n)])
        self.register_buffer("router_bias", None, persistent=False)
        self.entropy_adaptive_k = False
        self.entropy_k_min = 2
        self.precise_combine = False
        self.num_shared_experts = 0
        self._shared: Optional[Tuple[torch.Tensor, torch.Tensor]] = None
        self._shared_gate: Optional[torch.Tensor] = None
        self._bank_cache = None
        self.last_plan: Optional[DispatchPlan] = None
        self.last_counts: Optional[np.ndarray] = None   # [R, E] rows routed last step
        # experts held per rank: the contiguous shard, plus replicas after rebalance()
        self.placement = Placement(tuple(tuple(range(a, b)) for a, b in self.shards))
        self._slot_bank: Optional[Tuple[torch.Tensor, torch.Tensor]] = None
        # set to [] to record per-phase CUDA events / host times (see phase_times)
        self.trace: Optional[list] = None
        self._pin_ring = [[None, None] for _ in range(3)]
        self._pin_next = 0
        self._slot_arrays = None
        self.split_rounds = 4         # water-filling passes of the per-step row split
        self.native_planner = True    # False: the numpy planner (same result, slower)
        # rows cross NVLink as one-sided stores into peer buffers (one push
        # kernel + a bounded flag wait per direction); False: NCCL all-to-alls
        self.p2p = True
        self._px = None
        # with p2p: plan the exchange on the device (no host synchronisation
        # per step); False: the native host planner
        self.device_plan = True
        # device plan: buffers hold max_tokens_per_rank tokens from every rank
        # (None: the largest first-step token count over the ranks)
        self.max_tokens_per_rank: Optional[int] = None
        self._dp = None
        # device plan: push the rows bound for the other ranks on a side stream
        # while the gated GEMM runs over the rows this rank routed to itself;
        # False: push everything, wait, then one gated GEMM (same result)
        self.overlap_dispatch = False
        self._side_stream = None
        self.last_counts_dev: Optional[torch.Tensor] = None

    # --------------------------------------------------------------- build
    @classmethod
    def from_full(cls, base: FusedMoE, ep_size: int, ep_rank: int, *, token_sharded: bool = False,
                  group=None) -> "EPFusedMoE":
        """Shard a fully loaded :class:`FusedMoE` (ep.py:98-117)."""
        cfg = _LayerCfg(base.num_experts, base.top_k, base.hidden_size, base.intermediate_size,
                        base.activation, base.renormalize, base.dtype)
        ep = cls(cfg, ep_size, ep_rank, token_sharded=token_sharded, router_dtype=base.router_dtype,
                 device=base.gate.device, group=group)
        with torch.no_grad():
            ep.gate.copy_(base.gate)
            if ep.local_count:
                w1b, w2b = base._resident_banks()
                b1, b2 = ep._banks()
                b1.copy_(w1b[ep.local_start:ep.local_end])
                b2.copy_(w2b[ep.local_start:ep.local_end])
        ep.router_bias = base.router_bias
        ep.entropy_adaptive_k = base.entropy_adaptive_k
        ep.entropy_k_min = base.entropy_k_min
        ep.precise_combine = base.precise_combine
        if base.num_shared_experts:
            ep.num_shared_experts = base.num_shared_experts
            ep._shared = base._shared_banks()
            ep._shared_gate = None if base.shared_gate is None else base.shared_gate.detach()
        return ep

    def set_router_bias(self, bias: Optional[torch.Tensor]) -> None:
        self.router_bias = None if bias is None else bias.detach().float().to(self.gate.device)

    def _apply(self, fn, recurse=True):
        self._bank_cache = None
        if self._slot_bank is not None:
            self._slot_bank = tuple(fn(b) for b in self._slot_bank)
            for j, p in enumerate(self.experts_w1):
                p.data = self._slot_bank[0][j]
            for j, p in enumerate(self.experts_w2):
                p.data = self._slot_bank[1][j]
        return super()._apply(fn, recurse)

    @property
    def num_replicas(self) -> int:
        return len(self.placement.slots[self.ep_rank]) - self.local_count

    def _gemm_banks(self) -> Tuple[torch.Tensor, torch.Tensor]:
        """Weights of every local slot: primaries first, then replicas."""
        return self._slot_bank if self.num_replicas else self._banks()

    def rebalance(self, load: Optional[Sequence[float]] = None, redundant: int = 1) -> Placement:
        """Give every rank ``redundant`` replica slots of the busiest experts.

        ``load`` (per-expert rows, identical on every rank) defaults to the
        global counts of the last forward.  Collective: every rank must call it.
        Replica weights come from each expert's primary owner over NCCL/gloo
        point-to-point; afterwards each step splits an expert's rows among its
        holders so that the ranks' row counts even out.
        """
        if load is None:
            if self.last_counts is None and self.last_counts_dev is not None:
                self.last_counts = self.last_counts_dev.cpu().numpy()
            if self.last_counts is None:
                raise RuntimeError("rebalance() needs a load estimate or a previous forward")
            load = self.last_counts.sum(axis=0)
        placement = place_experts(load, self.shards, redundant)
        R, me, n = self.ep_size, self.ep_rank, self.local_count
        owner = np.zeros(self.num_experts, dtype=np.int64)
        for r, (a, b) in enumerate(self.shards):
            owner[a:b] = r
        w1b, w2b = self._banks()
        mine = placement.slots[me]
        dev = self.gate.device
        nw1 = torch.empty((len(mine),) + tuple(w1b.shape[1:]), dtype=w1b.dtype, device=dev)
        nw2 = torch.empty((len(mine),) + tuple(w2b.shape[1:]), dtype=w2b.dtype, device=dev)
        with torch.no_grad():
            nw1[:n].copy_(w1b)
            nw2[:n].copy_(w2b)
        ops = []
        for d in range(R):
            nd = self.shards[d][1] - self.shards[d][0]
            for j, e in enumerate(placement.slots[d][nd:]):
                o = int(owner[e])
                if o == me:
                    loc = e - self.local_start
                    ops += [tdist.P2POp(tdist.isend, w1b[loc].contiguous(), d, group=self._pg()),
                            tdist.P2POp(tdist.isend, w2b[loc].contiguous(), d, group=self._pg())]
                if d == me:
                    ops += [tdist.P2POp(tdist.irecv, nw1[n + j], o, group=self._pg()),
                            tdist.P2POp(tdist.irecv, nw2[n + j], o, group=self._pg())]
        if ops:
            for req in tdist.batch_isend_irecv(ops):
                req.wait()
        for j, p in enumerate(self.experts_w1):
            p.data = nw1[j]
        for j, p in enumerate(self.experts_w2):
            p.data = nw2[j]
        self._slot_bank = (nw1, nw2)
        self._bank_cache = None
        self.placement = placement
        return placement

    def _banks(self) -> Tuple[torch.Tensor, torch.Tensor]:
        if self._bank_cache is None:
            out = []
            for plist in (self.experts_w1, self.experts_w2):
                params = list(plist)
                bank = _bank_view(params)
                if bank is None:
                    bank = torch.stack([p.detach() for p in params]).contiguous()
                    for j, p in enumerate(params):
                        p.data = bank[j]
                out.append(bank.detach())
            self._bank_cache = (out[0], out[1])
        return self._bank_cache

    # ---------------------------------------------------------------- forward
    def _pg(self):
        if self.group is not None:
            return self.group
        return _dist.current().group if _dist.is_initialized() else None

    def forward(self, x: torch.Tensor, residual: Optional[torch.Tensor] = None) -> torch.Tensor:
        if not x.is_cuda:
            raise RfMoeError("EPFusedMoE runs on the B200 kernels and needs CUDA inputs")
        x2 = x.reshape(-1, self.hidden_size)
        if x2.dtype != self.dtype:
            x2 = x2.to(self.dtype)
        x2 = x2.contiguous()
        res2 = None if residual is None else residual.reshape(-1, self.hidden_size).to(self.dtype).contiguous()
        if self.token_sharded or self.ep_size == 1:
            out = self._forward_shard(x2, res2)
        else:
            T = x2.shape[0]
            lo = T * self.ep_rank // self.ep_size
            hi = T * (self.ep_rank + 1) // self.ep_size
            part = self._forward_shard(x2[lo:hi], None if res2 is None else res2[lo:hi])
            out = self._all_gather_rows(part, T)
        return reference_output(out, x, self.hidden_size)

    def _all_gather_rows(self, part: torch.Tensor, T: int) -> torch.Tensor:
        R = self.ep_size
        mx = (T + R - 1) // R
        buf = torch.zeros(mx, part.shape[1], dtype=part.dtype, device=part.device)
        buf[:part.shape[0]] = part
        outs = [torch.empty_like(buf) for _ in range(R)]
        tdist.all_gather(outs, buf, group=self._pg())
        pieces = []
        for r in range(R):
            lo, hi = T * r // R, T * (r + 1) // R
            pieces.append(outs[r][:hi - lo])
        return torch.cat(pieces, 0)

    def _pinned(self, n: int):
        """A reusable pinned int32 host buffer of >= n words from a small ring;
        a buffer is handed out again only after the copy that last read it has
        completed (no pinned allocation per step)."""
        slot = self._pin_ring[self._pin_next % len(self._pin_ring)]
        self._pin_next += 1
        if slot[1] is not None:
            slot[1].synchronize()
            slot[1] = None
        if slot[0] is None or slot[0].numel() < n:
            slot[0] = torch.empty(max(n, 1 << 16), dtype=torch.int32).pin_memory()
        return slot

    def _upload(self, slot, n: int, dev: torch.device) -> torch.Tensor:
        out = torch.empty(n, dtype=torch.int32, device=dev)
        out.copy_(slot[0][:n], non_blocking=True)
        slot[1] = torch.cuda.Event()
        slot[1].record()
        return out

    def _pair_rows(self, cnt: np.ndarray) -> np.ndarray:
        """The step's all-to-all matrix M[s, d] (rows s sends d), native."""
        R, E = cnt.shape
        cnt32 = np.ascontiguousarray(cnt, dtype=np.int32)
        if self._slot_arrays is None or self._slot_arrays[0] is not self.placement:
            flat = np.ascontiguousarray([e for s in self.placement.slots for e in s], dtype=np.int32)
            offs = np.ascontiguousarray(np.cumsum([0] + [len(s) for s in self.placement.slots]), dtype=np.int32)
            self._slot_arrays = (self.placement, flat, offs)
        _, flat, offs = self._slot_arrays
        M = np.zeros(R * R, dtype=np.int64)
        check(lib().rf_moe_ep_pair_rows(cnt32.ctypes.data, R, E, flat.ctypes.data, offs.ctypes.data,
                                        self.split_rounds, M.ctypes.data), "rf_moe_ep_pair_rows")
        return M.reshape(R, R)

    def _exchange(self):
        if self._px is None:
            from .p2p import PeerExchange
            self._px = PeerExchange(self.ep_rank, self.ep_size, self.gate.device, self._pg(),
                                    num_experts=self.num_experts)
        return self._px

    def close(self) -> None:
        """Release the peer buffers (collective: every rank, after its last forward)."""
        if self._px is not None:
            self._px.close()
            self._px = None

    def _native_plan(self, cnt: np.ndarray, n_mine: int):
        """Exchange plan from the native planner (rf_moe_ep_plan), written
        straight into a pinned buffer.  Returns (plan, pinned slot, layout)."""
        R, E = cnt.shape
        cnt32 = np.ascontiguousarray(cnt, dtype=np.int32)
        if self._slot_arrays is None or self._slot_arrays[0] is not self.placement:
            flat = np.ascontiguousarray([e for s in self.placement.slots for e in s], dtype=np.int32)
            offs = np.ascontiguousarray(np.cumsum([0] + [len(s) for s in self.placement.slots]), dtype=np.int32)
            self._slot_arrays = (self.placement, flat, offs)
        _, flat, offs = self._slot_arrays
        S = len(self.placement.slots[self.ep_rank])
        n_all = int(cnt32.sum())
        cap = 2 * n_all + S * K.ALIGN + 2 * S + 2 * n_mine + 16
        slot = self._pinned(cap)
        send = np.zeros(R, dtype=np.int64)
        recv = np.zeros(R, dtype=np.int64)
        layout = np.zeros(15, dtype=np.int64)
        rc = lib().rf_moe_ep_plan(cnt32.ctypes.data, R, E, self.ep_rank, flat.ctypes.data, offs.ctypes.data,
                                  K.ALIGN, self.split_rounds, send.ctypes.data, recv.ctypes.data,
                                  slot[0].data_ptr(), slot[0].numel(), layout.ctypes.data)
        check(rc, "rf_moe_ep_plan")
        host = slot[0].numpy()

        def arr(i):
            return host[layout[2 * i]:layout[2 * i] + layout[2 * i + 1]]
        plan = DispatchPlan([int(v) for v in send], [int(v) for v in recv], arr(3).astype(np.int64),
                            arr(2).astype(np.int64), int(layout[12]), arr(0), arr(1),
                            None if layout[13] else arr(4))
        return plan, slot, layout

    def _mark(self, name: str) -> None:
        """Record a phase boundary (CUDA event + host time) when tracing is on."""
        if self.trace is not None:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            self.trace.append((name, ev, time.perf_counter()))

    def phase_times(self) -> Dict[str, Tuple[float, float]]:
        """Per-phase (device ms, host ms) of the last traced forward."""
        tr = self.trace or []
        torch.cuda.synchronize()
        return {b[0]: (a[1].elapsed_time(b[1]), 1e3 * (b[2] - a[2])) for a, b in zip(tr, tr[1:])}

    def _forward_shard(self, x2: torch.Tensor, res2: Optional[torch.Tensor]) -> torch.Tensor:
        dev = x2.device
        T, H = x2.shape
        E, Kk, I = self.num_experts, self.top_k, self.intermediate_size
        ek = self.entropy_k_min if self.entropy_adaptive_k else 0
        rdt = None if (self.router_dtype == torch.float32 or self.dtype == torch.float32) else self.dtype
        pg = self._pg()
        if self.trace is not None:
            self.trace = []
        self._mark("start")
        use_p2p = self.p2p and dev.type == "cuda"
        if T > 0:
            gate, sg = adjacent_router_weights(self, self.gate, self._shared_gate)
            w, ids32, _, _, sscale = K.router_topk(x2, gate, Kk, renormalize=self.renormalize,
                                                   bias=self.router_bias, round_dtype=rdt, entropy_k_min=ek,
                                                   shared_gate=sg)
            # the peer push reads token rows through src_slot: no permuted copy
            p = K.permute(ids32, E, align=1, x=None if use_p2p else x2)
            counts = p.counts
        else:
            counts = torch.zeros(E, dtype=torch.int32, device=dev)
        self._mark("route+permute")
        if use_p2p and self.device_plan:
            return self._forward_devplan(x2, res2, p if T > 0 else None, w if T > 0 else None,
                                         sscale if T > 0 else None, counts)
        # (2) counts exchange -> the same plan on every rank
        gathered = [torch.empty_like(counts) for _ in range(self.ep_size)]
        tdist.all_gather(gathered, counts, group=pg)
        self._mark("counts all_gather")
        cnt = torch.stack(gathered).cpu().numpy()
        self.last_counts = cnt
        self._mark("counts to host")
        if self.native_planner:
            # native planner writes every index map into one pinned buffer -> one copy
            plan, slot, lay = self._native_plan(cnt, T * Kk)
            dev_ix = self._upload(slot, int(lay[14]), dev)
            views = [dev_ix[lay[2 * i]:lay[2 * i] + lay[2 * i + 1]] for i in range(6)]
        else:
            quota = split_rows(cnt, self.placement, rounds=self.split_rounds) if any(
                len(s) > b - a for s, (a, b) in zip(self.placement.slots, self.shards)) else None
            plan = plan_exchange(cnt, self.ep_rank, self.placement, quota)
            parts = [plan.gather_index, plan.inverse_index, plan.local_offsets.astype(np.int32),
                     plan.local_counts.astype(np.int32)]
            if plan.send_index is not None:
                pos_of_row = np.empty(T * Kk, dtype=np.int32)
                pos_of_row[plan.send_index] = np.arange(T * Kk, dtype=np.int32)
                parts += [plan.send_index, pos_of_row]
            host = np.concatenate(parts).astype(np.int32)
            slot = self._pinned(host.size)
            slot[0][:host.size].numpy()[:] = host
            dev_ix = self._upload(slot, host.size, dev)
            views, o = [], 0
            for a in parts:
                views.append(dev_ix[o:o + a.size])
                o += a.size
        self.last_plan = plan
        gidx, inv, off, lc = views[:4]
        self._mark("plan+index copy")
        if use_p2p:
            return self._exchange_p2p(x2, res2, p if T > 0 else None, plan, views,
                                      w if T > 0 else None, sscale if T > 0 else None, cnt)
        # (3) dispatch (rows reordered by destination only when replicas split an expert)
        if T == 0:
            send_rows = torch.empty(0, H, dtype=x2.dtype, device=dev)
        elif plan.send_index is None:
            send_rows = p.x_perm[:T * Kk]
        else:
            send_rows = K.gather_rows(p.x_perm, views[4], torch.empty(T * Kk, H, dtype=x2.dtype, device=dev))
        recv = torch.empty(plan.recv_total, H, dtype=x2.dtype, device=dev)
        self._mark("send gather")
        _dist.all_to_all_v(recv, send_rows, plan.recv_splits, plan.send_splits, group=pg)
        self._mark("dispatch all_to_all")
        # (4) regroup by local slot + expert GEMMs
        y_send = torch.empty(plan.recv_total, H, dtype=x2.dtype, device=dev)
        if plan.recv_total > 0:
            xl = torch.empty(plan.rows_capacity, H, dtype=x2.dtype, device=dev)
            K.gather_rows(recv, gidx, xl)
            self._mark("regroup gather")
            y = self._expert_gemms(xl, plan, off, lc)
            K.gather_rows(y, inv, y_send)
        self._mark("return gather")
        # (5) return trip + combine on the token's rank
        y_back = torch.empty(T * Kk, H, dtype=x2.dtype, device=dev)
        _dist.all_to_all_v(y_back, y_send, plan.send_splits, plan.recv_splits, group=pg)
        self._mark("combine all_to_all")
        out = torch.empty(T, H, dtype=x2.dtype, device=dev)
        if T == 0:
            return out
        if plan.send_index is not None:  # back to the expert-major permuted order
            y_back = K.gather_rows(y_back, views[5], torch.empty_like(y_back))
        shared_y = None
        if self._shared is not None:
            shared_y = K.shared_experts(x2, self._shared[0], self._shared[1], self.activation)
        out = K.combine(y_back, p.row_of_slot, w, out, shared_y=shared_y, shared_scale=sscale, residual=res2,
                        precise=self.precise_combine)
        self._mark("unpermute+shared+combine")
        return out

    def _expert_gemms(self, xl: torch.Tensor, plan, off: torch.Tensor, lc: torch.Tensor) -> torch.Tensor:
        """Grouped gated + down GEMMs over this rank's slot-major rows."""
        I, H = self.intermediate_size, xl.shape[1]
        rows = xl.shape[0]
        w1b, w2b = self._gemm_banks()
        h = torch.empty(rows, I, dtype=xl.dtype, device=xl.device)
        K.grouped_gemm_gated(xl, w1b, off, lc, h, activation=self.activation)
        self._mark("gated GEMM")
        y = torch.empty(rows, H, dtype=xl.dtype, device=xl.device)
        K.grouped_gemm_down(h, w2b, off, lc, y)
        self._mark("down GEMM")
        return y

    def _devplan_state(self, T: int, row_bytes: int):
        """Device slot arrays, plan workspace and peer buffers for the device
        plan (rebuilt when the placement changes).  The first call agrees on the
        per-rank token bound (collective)."""
        import ctypes
        dev = self.gate.device
        R, E, Kk = self.ep_size, self.num_experts, self.top_k
        if self.max_tokens_per_rank is None:
            t = torch.tensor([T], dtype=torch.int64, device=dev)
            tdist.all_reduce(t, op=tdist.ReduceOp.MAX, group=self._pg())
            self.max_tokens_per_rank = max(int(t.item()), 1)
        if T > self.max_tokens_per_rank:
            raise RfMoeError(f"EPFusedMoE: {T} tokens on this rank exceed max_tokens_per_rank="
                             f"{self.max_tokens_per_rank}; set it (on every rank) before the first forward")
        st = self._dp
        if st is None or st["placement"] is not self.placement:
            flat = np.ascontiguousarray([e for s_ in self.placement.slots for e in s_], dtype=np.int32)
            offs = np.ascontiguousarray(np.cumsum([0] + [len(s_) for s_ in self.placement.slots]), dtype=np.int32)
            S, nslots = len(self.placement.slots[self.ep_rank]), int(flat.size)
            nb = int(lib().rf_moe_ep_devplan_workspace_size(R, E, S, nslots))
            lay = np.zeros(_lib_mod.EP_DEVPLAN_LAYOUT_N, dtype=np.int64)
            check(lib().rf_moe_ep_devplan_layout(R, E, S, nslots, lay.ctypes.data), "rf_moe_ep_devplan_layout")
            ws = torch.zeros(nb, dtype=torch.uint8, device=dev)
            i32 = lambda o, n: ws[o:o + 4 * n].view(torch.int32)  # noqa: E731
            st = self._dp = {
                "placement": self.placement, "S": S, "nslots": nslots, "ws": ws,
                "flat": torch.from_numpy(flat).to(dev), "offs": torch.from_numpy(offs).to(dev),
                "seg_off": i32(lay[0], S + 1),
                "seg_cnt": i32(lay[1], max(S, 1))[:S],
                # groups of the overlapped dispatch: own rows per slot, then the
                # other sources' rows (below / above this rank) per slot
                "loc_off": i32(lay[18], 2 * S)[:S], "loc_cnt": i32(lay[18], 2 * S)[S:],
                "rem_off": i32(lay[19], 4 * S)[:2 * S], "rem_cnt": i32(lay[19], 4 * S)[2 * S:],
                "rem_slot": torch.arange(S, dtype=torch.int32, device=dev).repeat_interleave(2),
            }
        recv_cap = R * self.max_tokens_per_rank * Kk
        st["recv_cap"] = recv_cap
        st["back_cap"] = self.max_tokens_per_rank * Kk
        st["rows_cap"] = recv_cap + st["S"] * (K.ALIGN - 1)
        px = self._exchange()
        px.ensure(recv_cap, self.max_tokens_per_rank * Kk, row_bytes)
        return st, px

    def _forward_devplan(self, x2, res2, p, w, sscale, counts) -> torch.Tensor:
        """The EP forward with the exchange planned on the device: counts
        exchange over peer memory, planner kernel, peer pushes, bounded waits —
        no collective and no host synchronisation in the step."""
        import ctypes
        from .p2p import DISPATCH, RETURN
        dev = x2.device
        T, H = x2.shape
        R, E, Kk = self.ep_size, self.num_experts, self.top_k
        row_bytes = H * x2.element_size()
        stt, px = self._devplan_state(T, row_bytes)
        S, nslots, ws = stt["S"], stt["nslots"], stt["ws"]
        epoch = px.next_epoch()
        # counts all-gather as peer stores + a bounded flag wait (no collective)
        cnt = px.exchange_counts(counts.contiguous(), epoch)
        self.last_counts_dev, self.last_counts, self.last_plan = cnt, None, None
        self._mark("counts exchange")
        st = stream_of(dev)
        check(lib().rf_moe_ep_devplan(cnt.data_ptr(), stt["flat"].data_ptr(), stt["offs"].data_ptr(), R, E,
                                      self.ep_rank, S, nslots, K.ALIGN, self.split_rounds, stt["recv_cap"],
                                      stt["back_cap"], stt["rows_cap"], ws.data_ptr(), ws.numel(), st),
              "rf_moe_ep_devplan")
        self._mark("device plan")
        ctrl = px.peer[2]
        flags0 = (ctypes.c_void_p * R)(*[ctrl[d] + 4 * (DISPATCH * R + self.ep_rank) for d in range(R)])
        flags1 = (ctypes.c_void_p * R)(*[ctrl[d] + 4 * (RETURN * R + self.ep_rank) for d in range(R)])
        done = px.own[2].ptr + 2 * R * 4
        xsrc = x2.data_ptr() if T else None
        ssrc = p.src_slot.data_ptr() if p is not None else None
        peers_recv = (ctypes.c_void_p * R)(*px.peer[0])
        y = None
        back = (ctypes.c_void_p * R)(*px.peer[1])
        returned = False
        rows = stt["rows_cap"]
        I = self.intermediate_size
        overlap = self.overlap_dispatch and S > 0
        if overlap:
            # this rank's own rows go straight into their GEMM rows; then the
            # rows for the other ranks cross NVLink on a side stream while the
            # gated GEMM runs over the own rows; the other sources' rows follow
            cur = torch.cuda.current_stream(dev)
            if self._side_stream is None:
                self._side_stream = torch.cuda.Stream(device=dev)
            side = self._side_stream
            xl = torch.empty(rows, H, dtype=x2.dtype, device=dev)
            own = (ctypes.c_void_p * R)(*([xl.data_ptr()] * R))
            check(lib().rf_moe_ep_devplan_push(ws.data_ptr(), R, E, S, nslots, 3, xsrc, ssrc, Kk, row_bytes,
                                               own, flags0, epoch, done, st), "rf_moe_ep_devplan_push")
            self._mark("own rows")
            side.wait_stream(cur)
            check(lib().rf_moe_ep_devplan_push(ws.data_ptr(), R, E, S, nslots, 2, xsrc, ssrc, Kk, row_bytes,
                                               peers_recv, flags0, epoch, done, side.cuda_stream),
                  "rf_moe_ep_devplan_push")
            w1b, w2b = self._gemm_banks()
            h = torch.empty(rows, I, dtype=x2.dtype, device=dev)
            K.grouped_gemm_gated(xl, w1b, stt["loc_off"], stt["loc_cnt"], h, activation=self.activation)
            self._mark("gated GEMM (own rows)")
            cur.wait_stream(side)  # every tensor the side stream read outlives this join
            px.wait(DISPATCH)
            self._mark("dispatch wait")
            check(lib().rf_moe_ep_devplan_regroup_remote(ws.data_ptr(), R, E, S, nslots, px.recv_ptr(),
                                                         xl.data_ptr(), row_bytes, st),
                  "rf_moe_ep_devplan_regroup_remote")
            self._mark("regroup gather")
            K.grouped_gemm_gated(xl, w1b, stt["rem_off"], stt["rem_cnt"], h, slot=stt["rem_slot"],
                                 activation=self.activation)
            self._mark("gated GEMM")
        else:
            check(lib().rf_moe_ep_devplan_push(ws.data_ptr(), R, E, S, nslots, 0, xsrc, ssrc, Kk, row_bytes,
                                               peers_recv, flags0, epoch, done, st), "rf_moe_ep_devplan_push")
            self._mark("dispatch push")
            px.wait(DISPATCH)
            self._mark("dispatch wait")
        if S > 0:
            if not overlap:
                xl = torch.empty(rows, H, dtype=x2.dtype, device=dev)
                check(lib().rf_moe_ep_devplan_regroup(ws.data_ptr(), R, E, S, nslots, px.recv_ptr(),
                                                      xl.data_ptr(), row_bytes, st), "rf_moe_ep_devplan_regroup")
                self._mark("regroup gather")
                w1b, w2b = self._gemm_banks()
                h = torch.empty(rows, I, dtype=x2.dtype, device=dev)
                K.grouped_gemm_gated(xl, w1b, stt["seg_off"], stt["seg_cnt"], h, activation=self.activation)
                self._mark("gated GEMM")
            # the down GEMM's epilogue stores every row into its token rank's
            # return buffer (the exchange overlaps the GEMM tile by tile)
            rc = lib().rf_moe_ep_devplan_down_return(ws.data_ptr(), R, E, S, nslots, h.data_ptr(), w2b.data_ptr(),
                                                     rows, H, I, dtype_code(x2.dtype), back, flags1, epoch, done, st)
            if rc == _lib_mod.RF_ERR_UNSUPPORTED:  # no tensor-core path: down GEMM, then the push
                y = torch.empty(rows, H, dtype=x2.dtype, device=dev)
                K.grouped_gemm_down(h, w2b, stt["seg_off"], stt["seg_cnt"], y)
            else:
                check(rc, "rf_moe_ep_devplan_down_return")
                returned = True
            self._mark("down GEMM + return")
        if not returned:
            check(lib().rf_moe_ep_devplan_push(ws.data_ptr(), R, E, S, nslots, 1,
                                               y.data_ptr() if y is not None else None, None, 1, row_bytes, back,
                                               flags1, epoch, done, st), "rf_moe_ep_devplan_push")
            self._mark("return push")
        px.wait(RETURN)
        self._mark("return wait")
        out = torch.empty(T, H, dtype=x2.dtype, device=dev)
        if T == 0:
            return out
        # the return push left every result at its permuted row: the combine
        # reads them through the permute's own row_of_slot (expert order)
        shared_y = None
        if self._shared is not None:
            shared_y = K.shared_experts(x2, self._shared[0], self._shared[1], self.activation)
        wf = w.contiguous()
        mode = _lib_mod.COMBINE_FP32 if self.precise_combine else _lib_mod.COMBINE_REFERENCE
        check(lib().rf_moe_combine(px.back_ptr(), p.row_of_slot.data_ptr(), wf.data_ptr(), T, Kk, H,
                                   dtype_code(x2.dtype), None if shared_y is None else shared_y.data_ptr(),
                                   None if sscale is None else sscale.data_ptr(),
                                   None if res2 is None else res2.data_ptr(), 0, mode, out.data_ptr(), st),
              "rf_moe_combine")
        self._mark("shared+combine")
        return out

    def _exchange_p2p(self, x2, res2, p, plan, views, w, sscale, cnt) -> torch.Tensor:
        """Steps 3-5 over peer memory: push token rows into the experts' ranks,
        compute, push results back into the tokens' ranks, combine."""
        from .p2p import DISPATCH, RETURN, matrix_offsets
        dev = x2.device
        T, H = x2.shape
        Kk = self.top_k
        gidx, inv, off, lc = views[:4]
        row_bytes = H * x2.element_size()
        M = self._pair_rows(cnt)
        px = self._exchange()
        px.ensure(int(M.sum(0).max()), int(M.sum(1).max()), row_bytes)
        send_off, dst_row0, recv_off, back_row0 = matrix_offsets(M, self.ep_rank)
        px.next_epoch()
        px.push(DISPATCH, x2, send_off, dst_row0,
                idx1=views[4] if (p is not None and plan.send_index is not None) else None,
                idx2=None if p is None else p.src_slot, div=Kk)
        self._mark("dispatch push")
        px.wait(DISPATCH)
        self._mark("dispatch wait")
        st = stream_of(dev)
        y = None
        if plan.recv_total > 0:
            xl = torch.empty(plan.rows_capacity, H, dtype=x2.dtype, device=dev)
            check(lib().rf_moe_gather_rows(px.recv_ptr(), gidx.data_ptr(), 1, plan.rows_capacity, None, row_bytes,
                                           xl.data_ptr(), st), "rf_moe_gather_rows")
            self._mark("regroup gather")
            y = self._expert_gemms(xl, plan, off, lc)
        px.push(RETURN, y if y is not None else x2[:0], recv_off, back_row0,
                idx1=inv if plan.recv_total > 0 else None)
        self._mark("return push")
        px.wait(RETURN)
        self._mark("return wait")
        out = torch.empty(T, H, dtype=x2.dtype, device=dev)
        if T == 0:
            return out
        y_back = px.back_ptr()  # T*K rows in this rank's send order
        keep = None
        if plan.send_index is not None:  # back to the expert-major permuted order
            keep = torch.empty(T * Kk, H, dtype=x2.dtype, device=dev)
            check(lib().rf_moe_gather_rows(y_back, views[5].data_ptr(), 1, T * Kk, None, row_bytes,
                                           keep.data_ptr(), st), "rf_moe_gather_rows")
            y_back = keep.data_ptr()
        shared_y = None
        if self._shared is not None:
            shared_y = K.shared_experts(x2, self._shared[0], self._shared[1], self.activation)
        wf = w.contiguous()
        mode = _lib_mod.COMBINE_FP32 if self.precise_combine else _lib_mod.COMBINE_REFERENCE
        check(lib().rf_moe_combine(y_back, p.row_of_slot.data_ptr(), wf.data_ptr(), T, Kk, H,
                                   dtype_code(x2.dtype), None if shared_y is None else shared_y.data_ptr(),
                                   None if sscale is None else sscale.data_ptr(),
                                   None if res2 is None else res2.data_ptr(), 0, mode, out.data_ptr(), st),
              "rf_moe_combine")
        self._mark("unpermute+shared+combine")
        return out

    # ------------------------------------------------------------- (de)serial
    def state_dict(self, *args, prefix: str = "", result: Optional[dict] = None, **kwargs) -> Dict[str, torch.Tensor]:
        """Per-rank HF names with *global* expert ids (ep.py:153-162)."""
        result = {} if result is None else result
        pre = f"{prefix}." if prefix else ""
        result[f"{pre}gate.weight"] = self.gate
        I = self.intermediate_size
        for j, g in enumerate(range(self.local_start, self.local_end)):
            p = f"{pre}experts.{g}"
            result[f"{p}.gate_proj.weight"] = self.experts_w1[j][:I]
            result[f"{p}.up_proj.weight"] = self.experts_w1[j][I:]
            result[f"{p}.down_proj.weight"] = self.experts_w2[j]
        return result

    def load_state_dict(self, state_dict: Dict[str, torch.Tensor], *args, prefix: str = "", **kwargs) -> None:
        pre = f"{prefix}." if prefix else ""
        with torch.no_grad():
            g = f"{pre}gate.weight"
            if g in state_dict:
                self.gate.copy_(state_dict[g].detach().to(dtype=self.dtype))
            I = self.intermediate_size
            for j, gg in enumerate(range(self.local_start, self.local_end)):
                p = f"{pre}experts.{gg}"
                for half, param in (("gate_proj", self.experts_w1[j][:I]), ("up_proj", self.experts_w1[j][I:]),
                                    ("down_proj", self.experts_w2[j])):
                    t = expert_tensor(state_dict, p, half)
                    if t is not None:
                        param.copy_(t.detach().to(dtype=self.dtype))


@dataclass
class _LayerCfg:
    num_experts: int
    num_experts_per_tok: int
    hidden_size: int
    moe_inter: int
    moe_activation: str
    moe_renormalize: bool
    dtype: torch.dtype
