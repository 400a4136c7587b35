"""Expert offload cache: pinned host pool + a fixed pool of device expert slots.

Drop-in for reframework/moe/offload_cache.py (``ExpertOffloadCache``,
``Prediction``, ``OffloadStats``).  The residency *policy* is the reference's:
  * ``prefetch`` (offload_cache.py:478-507): requested experts become the most
    recently used; misses are loaded; eviction protects the request (hard) and
    the lookahead set (soft) — ``_evict`` (654-711) with ``RE_CACHE_POLICY``
    ``lru`` or ``least_stale``.
  * ``reserve`` (569-643): lookahead loads bounded by a PCIe byte budget
    (``bw * forward_ms * headroom - inflight``) and by the evictable room.
  * ``Prediction`` (108-223): decode-step routed-set window, score
    ``freq * 1000 + (window - age)``.
The *mechanism* is B200-shaped:
  * experts live in one contiguous pinned host buffer (offload_cache.py:304-347);
  * the device side is a fixed pool ``[S, 2I, H]`` / ``[S, H, I]`` of slots
    (S = ``lru_capacity``), so a resident expert is a slot index, never a
    separate allocation, and the grouped GEMM reads experts through an
    expert -> slot table (no per-step ``torch.stack`` repack, 734-742);
  * host->device copies run on a dedicated copy stream; each slot carries a
    "ready" event (copy done) that compute waits on, and a "free" event
    (recorded on the compute stream when the slot is evicted) that the copy
    stream waits on before overwriting the slot.
A slot is acquired *before* a miss is copied: when none is free, one victim is
evicted with the same two-tier policy first.  This evicts the same experts the
reference's fill-then-evict order does (victims never come from the request),
without ever holding more than S experts.  Only when every resident expert is
hard-protected does the pool grow (the reference then exceeds its capacity).

``prefetch`` returns ``(pool_w1, pool_w2, local_index)``: the banks are the slot
pool itself and ``local_index`` maps each requested global id to its slot
(the reference returns freshly stacked N-row banks and row indices; code that
indexes the banks through ``local_index`` works unchanged).
"""

from __future__ import annotations

import logging
import time
from collections import OrderedDict, deque
from dataclasses import dataclass, field
from typing import Deque, Dict, List, Optional, Sequence, Tuple

import torch

from .. import env

logger = logging.getLogger(__name__)

__all__ = ["ExpertOffloadCache", "OffloadStats", "Prediction"]


@dataclass
class OffloadStats:
    """Counters (field names and ``as_dict`` keys of offload_cache.py:75-105)."""

    hits: int = 0
    misses: int = 0
    evictions: int = 0
    transfers_bytes: int = 0
    subs: int = 0
    predicts: int = 0
    inflight_bytes: int = 0

    def reset(self) -> None:
        self.hits = self.misses = self.evictions = self.transfers_bytes = 0
        self.subs = self.predicts = self.inflight_bytes = 0

    def as_dict(self) -> dict:
        return {
            "hits": self.hits,
            "misses": self.misses,
            "evictions": self.evictions,
            "subs": self.subs,
            "predicts": self.predicts,
            "inflight_bytes": self.inflight_bytes,
            "transfer_mb": self.transfers_bytes / (1024 * 1024),
        }


class Prediction:
    """Rolling decode-step routing history of one layer (offload_cache.py:108-223).

    ``record_step`` resets on prefill, otherwise ages every seen expert, stamps
    the routed ones with age 0, appends the routed set to the window and asks
    the cache to ``reserve`` the predicted next set.  ``predict_next`` ranks
    non-resident experts by ``freq * 1000 + (window - age)`` (ties: lower id).
    """

    def __init__(self, cache: "ExpertOffloadCache", window: int = 32) -> None:
        self.cache = cache
        self.window = max(1, int(window))
        self._history: Deque[frozenset] = deque(maxlen=self.window)
        self._age: Dict[int, int] = {}

    def reset(self) -> None:
        self._history.clear()
        self._age.clear()

    def record_step(self, routed: Sequence[int], *, is_prefill: bool, forward_ms: float,
                    inflight_bytes: float = 0.0) -> None:
        routed_set = frozenset(int(i) for i in routed)
        if is_prefill:
            self.reset()
            return
        for e in self._age:
            self._age[e] += 1
        for e in routed_set:
            self._age[e] = 0
        self._history.append(routed_set)
        predicted = self.predict_next()
        if predicted:
            self.cache.reserve(predicted, forward_ms=forward_ms, protect_current=routed,
                               inflight_bytes=inflight_bytes)

    def predict_next(self, limit: Optional[int] = None) -> List[int]:
        freq: Dict[int, int] = {}
        for s in self._history:
            for e in s:
                freq[e] = freq.get(e, 0) + 1
        if not freq:
            return []
        ranked = sorted(freq, key=lambda e: (-(freq[e] * 1000 + self.window - self._age.get(e, self.window)), e))
        out: List[int] = []
        for e in ranked:
            if e in self.cache._lru:
                continue
            out.append(e)
            if limit is not None and len(out) >= limit:
                break
        return out


def sym_int8_quantize(w: torch.Tensor) -> Tuple[torch.Tensor, float]:
    """Symmetric per-tensor int8 (offload_cache.py:58-72): scale = max|w| / 127
    in fp32, codes = round(w / scale) clamped to +-127; an all-zero tensor gets
    scale 1.0.  Runs once per expert when the split is armed (host setup)."""
    amax = w.detach().abs().max().float()
    if amax <= 0:
        return torch.zeros_like(w, dtype=torch.int8), 1.0
    scale = amax / 127.0
    wq = (w.detach().float() / scale).round().clamp(-127, 127).to(torch.int8).contiguous()
    return wq, float(scale)


def _pin(t: torch.Tensor) -> Tuple[torch.Tensor, bool]:
    if not torch.cuda.is_available():
        return t, False
    try:
        return t.pin_memory(), True
    except RuntimeError:
        return t, False


@dataclass
class ExpertOffloadCache:
    """Pinned host expert pool + a fixed pool of device slots (see module doc)."""

    device: torch.device
    lru_capacity: int
    dtype: torch.dtype = torch.float16
    _host: List[Tuple[torch.Tensor, torch.Tensor]] = field(default_factory=list, repr=False)
    _host_buf: Optional[torch.Tensor] = field(default=None, repr=False)
    _pinned: bool = field(default=False, repr=False)
    # expert id -> slot index, in LRU order (oldest first)
    _lru: "OrderedDict[int, int]" = field(default_factory=OrderedDict, repr=False)
    stats: OffloadStats = field(default_factory=OffloadStats, repr=False)
    _next_reserve: frozenset = field(default_factory=frozenset, repr=False, compare=False)
    sim_table: Optional[torch.Tensor] = field(default=None, repr=False, compare=False)
    _predictor: Optional[Prediction] = field(default=None, repr=False, compare=False)
    _bw_gb_s: Optional[float] = field(default=None, repr=False, compare=False)
    _bw_headroom: float = field(default=0.9, repr=False, compare=False)
    # device slot pool
    pool_w1: Optional[torch.Tensor] = field(default=None, repr=False, compare=False)
    pool_w2: Optional[torch.Tensor] = field(default=None, repr=False, compare=False)
    _free: List[int] = field(default_factory=list, repr=False, compare=False)
    _slot_refs: List[int] = field(default_factory=list, repr=False, compare=False)
    _slot_ready: List[Optional[object]] = field(default_factory=list, repr=False, compare=False)
    _slot_free_evt: List[Optional[object]] = field(default_factory=list, repr=False, compare=False)
    _copy_stream: Optional[object] = field(default=None, repr=False, compare=False)
    h2d_seconds: float = field(default=0.0, repr=False, compare=False)
    # expert split: int8 copies of the host pool (one pinned buffer), their
    # scales [E, 2] (host and device) and a device pool the step's misses are
    # staged in
    _cpu_split: bool = field(default=False, repr=False, compare=False)
    _int8_host: List[Tuple[torch.Tensor, torch.Tensor, float, float]] = field(default_factory=list, repr=False,
                                                                               compare=False)
    _int8_buf: Optional[torch.Tensor] = field(default=None, repr=False, compare=False)
    _int8_scales: Optional[torch.Tensor] = field(default=None, repr=False, compare=False)
    _int8_scales_dev: Optional[torch.Tensor] = field(default=None, repr=False, compare=False)
    pool_q1: Optional[torch.Tensor] = field(default=None, repr=False, compare=False)
    pool_q2: Optional[torch.Tensor] = field(default=None, repr=False, compare=False)
    _int8_free_evt: Optional[object] = field(default=None, repr=False, compare=False)
    int8_transfer_bytes: int = field(default=0, repr=False, compare=False)  # outside OffloadStats (reference keys)

    def __post_init__(self) -> None:
        self.device = torch.device(self.device)

    # ----------------------------------------------------------------- factory
    @classmethod
    def from_config(cls, cfg, *, device=None, lru_capacity: Optional[int] = None) -> "ExpertOffloadCache":
        return cls(device=torch.device(device or cfg.device),
                   lru_capacity=lru_capacity if lru_capacity is not None else env.get_moe_cache_size(),
                   dtype=cfg.dtype)

    # ------------------------------------------------------------------- setup
    @property
    def _cuda(self) -> bool:
        return self.device.type == "cuda"

    def load(self, experts: Sequence[Dict[str, torch.Tensor]]) -> None:
        """Stage per-expert ``{"w1": [2I,H], "w2": [H,I]}`` in one pinned host buffer
        and allocate the device slot pool (offload_cache.py:304-347)."""
        n1 = sum(e["w1"].numel() for e in experts)
        n2 = sum(e["w2"].numel() for e in experts)
        buf = None
        if self._cuda and torch.cuda.is_available():
            try:  # allocate the pool pinned directly (no pageable copy of every expert first)
                buf = torch.empty(n1 + n2, dtype=self.dtype, pin_memory=True)
                self._pinned = True
            except RuntimeError:
                buf = None
        if buf is None:
            buf = torch.empty(n1 + n2, dtype=self.dtype)
            self._pinned = False
        self._host_buf = buf
        self._host = []
        off = 0
        for e in experts:
            w1, w2 = e["w1"].detach(), e["w2"].detach()
            v1 = buf[off:off + w1.numel()].view(tuple(w1.shape))
            v1.copy_(w1.to(dtype=self.dtype))
            off += w1.numel()
            v2 = buf[off:off + w2.numel()].view(tuple(w2.shape))
            v2.copy_(w2.to(dtype=self.dtype))
            off += w2.numel()
            self._host.append((v1, v2))
        if self._cuda and torch.cuda.is_available():
            torch.cuda.synchronize(self.device)  # device-to-host copies into the pool are complete
        self._lru = OrderedDict()
        self.stats.reset()
        self._alloc_pool(max(1, int(self.lru_capacity)))
        logger.info("ExpertOffloadCache staged %d experts (%s) in %s host pool; %d device slots",
                    len(self._host), self.dtype, "pinned" if self._pinned else "pageable",
                    self.num_slots)

    def _alloc_pool(self, slots: int) -> None:
        w1, w2 = self._host[0]
        old1, old2 = self.pool_w1, self.pool_w2
        n_old = 0 if old1 is None else old1.shape[0]
        self.pool_w1 = torch.empty((slots,) + tuple(w1.shape), dtype=self.dtype, device=self.device)
        self.pool_w2 = torch.empty((slots,) + tuple(w2.shape), dtype=self.dtype, device=self.device)
        if n_old:
            if self._cuda:
                torch.cuda.current_stream(self.device).wait_stream(self.copy_stream())
            self.pool_w1[:n_old].copy_(old1)
            self.pool_w2[:n_old].copy_(old2)
        self._free.extend(range(n_old, slots))
        self._slot_refs.extend([0] * (slots - n_old))
        self._slot_ready.extend([None] * (slots - n_old))
        self._slot_free_evt.extend([None] * (slots - n_old))

    @property
    def num_slots(self) -> int:
        return 0 if self.pool_w1 is None else self.pool_w1.shape[0]

    @property
    def num_experts(self) -> int:
        return len(self._host)

    @property
    def cpu_split(self) -> bool:
        """True once the int8 copies are built and the split is armed."""
        return self._cpu_split

    def copy_stream(self):
        if self._copy_stream is None and self._cuda:
            self._copy_stream = torch.cuda.Stream(device=self.device)
        return self._copy_stream

    def expert_bytes(self, idx: int = 0) -> int:
        w1, w2 = self._host[idx]
        return (w1.numel() + w2.numel()) * w1.element_size()

    def resident_set(self) -> frozenset:
        return frozenset(self._lru.keys())

    def slot_of(self, idx: int) -> int:
        return self._lru[idx]

    def set_sim_table(self, sim: torch.Tensor) -> None:
        E = len(self._host)
        sim = torch.as_tensor(sim, dtype=torch.float32)
        if tuple(sim.shape) != (E, E):
            raise ValueError(f"sim_table shape {tuple(sim.shape)} != [E,E]=[{E},{E}]")
        self.sim_table = sim

    def attach_predictor(self, window: int = 32) -> None:
        self._predictor = Prediction(self, window=window)
        self._bw_headroom = max(0.05, min(1.0, env.get_moe_predict_headroom()))
        self.measure_bandwidth()

    def measure_bandwidth(self) -> Optional[float]:
        """Pinned host->device copy rate in GB/s on the copy stream (offload_cache.py:436-467)."""
        if not (self._cuda and torch.cuda.is_available()):
            return None
        try:
            n = 1 << 27  # 256 MB of 16-bit elements: long enough to reach the link's steady rate
            src, _ = _pin(torch.empty(n, dtype=self.dtype))
            dst = torch.empty(n, dtype=self.dtype, device=self.device)
            cs = self.copy_stream()
            with torch.cuda.stream(cs):
                dst.copy_(src, non_blocking=True)
                t0 = torch.cuda.Event(enable_timing=True)
                t1 = torch.cuda.Event(enable_timing=True)
                t0.record(cs)
                for _ in range(3):
                    dst.copy_(src, non_blocking=True)
                t1.record(cs)
            t1.synchronize()
            ms = t0.elapsed_time(t1)
            if ms > 0:
                self._bw_gb_s = 3 * n * src.element_size() / (ms * 1e-3) / 1e9
            return self._bw_gb_s
        except Exception as exc:  # pragma: no cover - best effort, as in the reference
            logger.warning("host->device bandwidth measure failed: %s", exc)
            return None

    def reset_lru(self) -> None:
        for idx in list(self._lru):
            self._release(idx)
        self._lru = OrderedDict()
        self._next_reserve = frozenset()
        if self._predictor is not None:
            self._predictor.reset()

    # ------------------------------------------------------------------ access
    def prefetch(self, indices: Sequence[int]) -> Tuple[torch.Tensor, torch.Tensor, Dict[int, int]]:
        """Make ``indices`` resident; returns (pool_w1, pool_w2, {global id: slot})."""
        uniq = sorted(set(int(i) for i in indices if int(i) >= 0))
        hard = set(uniq)
        soft = set(self._next_reserve) - hard
        for idx in uniq:
            if idx not in self._lru:
                if self._substitute(idx) is None:
                    self._fill(idx, hard, soft)
            else:
                self.stats.hits += 1
            self._lru.move_to_end(idx)
        self._evict(uniq, soft)
        return self._pack(uniq)

    def reserve(self, predicted: Sequence[int], *, forward_ms: float = 0.0,
                bandwidth_gb_s: Optional[float] = None, protect_current: Sequence[int] = (),
                inflight_bytes: float = 0.0) -> int:
        """Lookahead load of the ranked ``predicted`` experts (offload_cache.py:569-643)."""
        if not predicted or self.lru_capacity <= 0:
            return 0
        protect = set(int(i) for i in protect_current) | set(int(i) for i in predicted)
        bw = bandwidth_gb_s if bandwidth_gb_s is not None else self._bw_gb_s
        budget = None
        if forward_ms > 0 and bw and bw > 0:
            budget = bw * 1e9 * (forward_ms / 1000.0) * self._bw_headroom
            if inflight_bytes and inflight_bytes > 0:
                budget = max(0.0, budget - inflight_bytes)
                self.stats.inflight_bytes += int(inflight_bytes)
        loaded: List[int] = []
        for idx in (int(i) for i in predicted):
            if idx in self._lru:
                continue
            b = self.expert_bytes(idx)
            if budget is not None:
                if b > budget and loaded:
                    break
                budget -= b
            self._fill(idx, protect, set())
            self.stats.predicts += 1
            loaded.append(idx)
            self._evict(protect)
            if len(self._lru) > self.lru_capacity:
                break
        self._next_reserve = frozenset(loaded)
        return len(loaded)

    # ---------------------------------------------------------- slot machinery
    def _victim(self, hard: set, soft: set) -> Optional[int]:
        """Next eviction victim under RE_CACHE_POLICY (offload_cache.py:654-711)."""
        pred = self._predictor
        if env.get_moe_cache_policy() == "least_stale" and pred is not None:
            age, window = pred._age, pred.window

            def pick(cands: List[int]) -> Optional[int]:
                best, best_age = None, -1
                for i in cands:  # LRU order: the first maximum (oldest) wins ties
                    a = age.get(i, window)
                    if a > best_age:
                        best, best_age = i, a
                return best
        else:
            def pick(cands: List[int]) -> Optional[int]:
                return cands[0] if cands else None
        v = pick([i for i in self._lru if i not in hard and i not in soft])
        if v is None:
            v = pick([i for i in self._lru if i in soft])
        return v

    def _evict(self, hard_protect: Sequence[int], soft_protect: Sequence[int] = ()) -> None:
        hard = set(int(i) for i in hard_protect)
        soft = set(int(i) for i in soft_protect) - hard
        while len(self._lru) > self.lru_capacity:
            v = self._victim(hard, soft)
            if v is None:
                return
            self._release(v)
            self.stats.evictions += 1

    def _release(self, idx: int) -> None:
        slot = self._lru.pop(idx)
        self._slot_refs[slot] -= 1
        if self._slot_refs[slot] == 0:
            if self._cuda:
                # the slot may be overwritten once the work queued so far has run
                evt = torch.cuda.Event()
                evt.record(torch.cuda.current_stream(self.device))
                self._slot_free_evt[slot] = evt
            self._free.append(slot)

    def _acquire_slot(self, hard: set, soft: set) -> int:
        if not self._free and len(self._lru) >= self.lru_capacity:
            v = self._victim(hard, soft)
            if v is not None:
                self._release(v)
                self.stats.evictions += 1
        if not self._free:
            self._alloc_pool(self.num_slots + 1)
        return self._free.pop(0)

    def _fill(self, idx: int, hard: Optional[set] = None, soft: Optional[set] = None) -> None:
        """Copy expert ``idx`` host -> a device slot (copy stream when on CUDA)."""
        hard = set(hard or ()) | {idx}
        slot = self._acquire_slot(hard, set(soft or ()) - hard)
        w1, w2 = self._host[idx]
        if self._cuda:
            cs = self.copy_stream()
            with torch.cuda.stream(cs):
                free_evt = self._slot_free_evt[slot]
                if free_evt is not None:
                    cs.wait_event(free_evt)
                self.pool_w1[slot].copy_(w1, non_blocking=self._pinned)
                self.pool_w2[slot].copy_(w2, non_blocking=self._pinned)
                ready = torch.cuda.Event()
                ready.record(cs)
            self._slot_ready[slot] = ready
        else:
            self.pool_w1[slot].copy_(w1)
            self.pool_w2[slot].copy_(w2)
        self._slot_refs[slot] += 1
        self.stats.transfers_bytes += self.expert_bytes(idx)
        self.stats.misses += 1
        self._lru[idx] = slot

    def _substitute(self, idx: int) -> Optional[int]:
        """Serve a miss with the most similar resident expert (offload_cache.py:713-732)."""
        if self.sim_table is None or idx in self._lru:
            return None
        residents = [i for i in self._lru if i != idx]
        if not residents:
            return None
        row = self.sim_table[idx]
        best = max(residents, key=lambda i: (float(row[i]), -i))
        self.stats.subs += 1
        slot = self._lru[best]
        self._slot_refs[slot] += 1
        self._lru[idx] = slot
        return best

    def wait_ready(self, experts: Sequence[int], stream=None) -> None:
        """Make ``stream`` (default: current) wait for the copies of these experts."""
        if not self._cuda:
            return
        st = stream or torch.cuda.current_stream(self.device)
        for e in experts:
            ev = self._slot_ready[self._lru[e]]
            if ev is not None:
                st.wait_event(ev)

    def _pack(self, uniq: Sequence[int]) -> Tuple[torch.Tensor, torch.Tensor, Dict[int, int]]:
        self.wait_ready(uniq)
        return self.pool_w1, self.pool_w2, {i: self._lru[i] for i in uniq}

    # ------------------------------------------------------------ expert split
    def quantize_int8_host(self) -> None:
        """Per-expert symmetric int8 copies of the host pool for the expert
        split (offload_cache.py:386-408), in one pinned buffer (half the bytes
        of a 16-bit pool): a step's non-resident experts cross PCIe as int8."""
        if not self._host:
            return
        n = sum(w1.numel() + w2.numel() for w1, w2 in self._host)
        buf = None
        if self._cuda and torch.cuda.is_available():
            try:
                buf = torch.empty(n, dtype=torch.int8, pin_memory=True)
            except RuntimeError:
                buf = None
        if buf is None:
            buf = torch.empty(n, dtype=torch.int8)
        scales = torch.empty(len(self._host), 2, dtype=torch.float32)
        self._int8_host = []
        off = 0
        for i, (w1, w2) in enumerate(self._host):
            q1, s1 = sym_int8_quantize(w1)
            q2, s2 = sym_int8_quantize(w2)
            v1 = buf[off:off + q1.numel()].view(tuple(q1.shape))
            v1.copy_(q1)
            off += q1.numel()
            v2 = buf[off:off + q2.numel()].view(tuple(q2.shape))
            v2.copy_(q2)
            off += q2.numel()
            self._int8_host.append((v1, v2, s1, s2))
            scales[i, 0], scales[i, 1] = s1, s2
        self._int8_buf = buf
        self._int8_scales = scales
        self._int8_scales_dev = scales.to(self.device)
        self._cpu_split = True
        logger.info("expert split: int8 copies of %d experts (symmetric per-tensor)", len(self._int8_host))

    def split_prefetch(self, indices: Sequence[int]) -> Tuple[Tuple[torch.Tensor, torch.Tensor, Dict[int, int]],
                                                               List[int]]:
        """Dispatch the routed set by residency (offload_cache.py:509-552):
        ``((pool_w1, pool_w2, {hit: slot}), misses)``, both ascending; hits
        count as hits and move to the LRU's recent end; misses are not loaded
        here (``reactive_load`` brings them resident after the step)."""
        uniq = sorted(set(int(i) for i in indices if int(i) >= 0))
        hits = [i for i in uniq if i in self._lru]
        misses = [i for i in uniq if i not in self._lru]
        for i in hits:
            self._lru.move_to_end(i)
            self.stats.hits += 1
        return self._pack(hits), misses

    def cpu_banks(self, indices: Sequence[int]) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor,
                                                          Dict[int, int]]:
        """The int8 copies of ``indices`` (ascending) on the host:
        ``(w1q [N,2I,H], w2q [N,H,I], scales1 [N], scales2 [N], {id: row})``
        (offload_cache.py:410-434; every index is packed)."""
        uniq = sorted(set(int(i) for i in indices))
        local = {e: k for k, e in enumerate(uniq)}
        if not uniq:
            w1, w2 = self._host[0]
            return (torch.empty((0,) + tuple(w1.shape), dtype=torch.int8),
                    torch.empty((0,) + tuple(w2.shape), dtype=torch.int8),
                    torch.empty(0), torch.empty(0), local)
        return (torch.stack([self._int8_host[e][0] for e in uniq]), torch.stack([self._int8_host[e][1] for e in uniq]),
                self._int8_scales[uniq, 0].clone(), self._int8_scales[uniq, 1].clone(), local)

    def int8_banks(self, indices: Sequence[int]) -> Tuple[torch.Tensor, torch.Tensor, Dict[int, int]]:
        """Stage the int8 copies of ``indices`` in the device int8 pool (one
        H2D copy per matrix on the copy stream, after the previous step's int8
        GEMMs released the pool; the current stream waits for the copies).
        Returns ``(pool_q1, pool_q2, {id: pool row})``; the scales of every
        expert are ``_int8_scales_dev`` [E, 2]."""
        uniq = sorted(set(int(i) for i in indices))
        if not uniq:
            return self.pool_q1, self.pool_q2, {}
        w1, w2 = self._int8_host[0][0], self._int8_host[0][1]
        if self.pool_q1 is None or self.pool_q1.shape[0] < len(uniq):
            # a larger pool; its memory may be the old pool's, so the copies
            # below still wait for the last release of the old one
            self.pool_q1 = torch.empty((len(uniq),) + tuple(w1.shape), dtype=torch.int8, device=self.device)
            self.pool_q2 = torch.empty((len(uniq),) + tuple(w2.shape), dtype=torch.int8, device=self.device)
        pinned = self._int8_buf is not None and self._int8_buf.is_pinned()
        if self._cuda:
            cs = self.copy_stream()
            self.pool_q1.record_stream(cs)
            self.pool_q2.record_stream(cs)
            with torch.cuda.stream(cs):
                if self._int8_free_evt is not None:
                    cs.wait_event(self._int8_free_evt)
                for k, e in enumerate(uniq):
                    self.pool_q1[k].copy_(self._int8_host[e][0], non_blocking=pinned)
                    self.pool_q2[k].copy_(self._int8_host[e][1], non_blocking=pinned)
                ready = torch.cuda.Event()
                ready.record(cs)
            torch.cuda.current_stream(self.device).wait_event(ready)
        else:
            for k, e in enumerate(uniq):
                self.pool_q1[k].copy_(self._int8_host[e][0])
                self.pool_q2[k].copy_(self._int8_host[e][1])
        self.int8_transfer_bytes += sum(self._int8_host[e][0].numel() + self._int8_host[e][1].numel()
                                        for e in uniq)
        return self.pool_q1, self.pool_q2, {e: k for k, e in enumerate(uniq)}

    def int8_release(self) -> None:
        """The int8 pool may be overwritten once the work queued so far has run."""
        if self._cuda:
            evt = torch.cuda.Event()
            evt.record(torch.cuda.current_stream(self.device))
            self._int8_free_evt = evt

    def reactive_load(self, indices: Sequence[int]) -> None:
        """Bring this step's misses resident for the next step
        (offload_cache.py:554-567): every miss is loaded (no substitution) with
        all of them protected, then the LRU is trimmed with the next-step
        reserve as the soft tier."""
        uniq = sorted(set(int(i) for i in indices))
        hard = set(uniq)
        soft = set(self._next_reserve) - hard
        for i in uniq:
            if i not in self._lru:
                self._fill(i, hard, soft)
        self._evict(uniq, soft)

    def slot_table(self) -> torch.Tensor:
        """int32 [E] expert -> slot (-1 when not resident), on the device."""
        t = torch.full((self.num_experts,), -1, dtype=torch.int32)
        for e, s in self._lru.items():
            t[e] = s
        return t.to(self.device, non_blocking=True)

    # ------------------------------------------------------------------- stats
    def report(self) -> str:
        s = self.stats.as_dict()
        return (f"offload: hit={s['hits']} miss={s['misses']} sub={s['subs']} "
                f"pred={s['predicts']} evict={s['evictions']} transfer={s['transfer_mb']:.1f}MB")
