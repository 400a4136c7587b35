"""FusedMoE: the routed MoE block, drop-in for reframework/moe/moe_layer.py.

Same constructor, parameters (``gate`` [E,H], ``experts_w1[e]`` [2I,H] gate|up,
``experts_w2[e]`` [H,I]), HF state-dict names and methods (``route``,
``forward``, ``prefetch_ids``, ``build_offload_cache``, ``attach_predictor``,
``enable_cpu_split``, ``set_shuttle``, ``state_dict``, ``load_state_dict``,
``from_config``) as the reference ``FusedMoE`` (moe_layer.py:132-663).

What differs is where the work runs:
  * the expert parameters are views into one contiguous ``[E,2I,H]`` /
    ``[E,H,I]`` bank, so ``forward`` never restacks the weights (the
    reference stacks every expert on every call, moe_layer.py:444-445);
  * one forward is router -> permute -> grouped gated GEMM -> grouped down
    GEMM -> combine, each a CUDA kernel of ``reframework_b200._rf_moe.so``;
    there is no host synchronisation in resident mode;
  * offload mode is always exact (every routed expert is computed): experts
    stream through the cache's fixed device slots, copies on a side stream
    overlapping the grouped GEMMs of already-resident experts.  The
    reference's default offload path keeps only ``RE_MAX_PACK`` experts per
    step (moe_layer.py:430-441), which changes the output; that truncation is
    not reproduced (a set ``RE_MAX_PACK`` is logged once and ignored).

Opt-in extensions (default off, reference behaviour unchanged):
  ``router_dtype=torch.float32`` keeps fp32 logits (the reference rounds them to
  the layer dtype); ``router_bias`` [E] is added to the logits;
  ``num_shared_experts`` / ``shared_intermediate_size`` / ``shared_expert_gate``
  add always-on shared SwiGLU experts (optionally scaled by sigmoid(x.w_s));
  ``forward(x, residual=r)`` fuses ``+ r`` into the combine; ``device=``
  allocates the parameters directly on a device.
"""

from __future__ import annotations

import logging
import time
from collections import deque
from typing import Deque, Dict, List, Optional, Sequence, Tuple

import torch
import torch.nn as nn

from .. import env
from .. import kernels as K
from .._lib import ACTIVATIONS, RfMoeError
from .keys import expert_tensor
from .offload_cache import ExpertOffloadCache, Prediction

logger = logging.getLogger(__name__)

__all__ = ["FusedMoE", "CpuShuttle"]

_warned_max_pack = False


class CpuShuttle:
    """Byte-accounting mock of a device shuttle (moe_layer.py:58-129).

    ``send`` ages the in-flight transfers by one step and records the new
    transfer's bytes, each transfer decaying linearly over ``n_steps`` steps;
    ``inflight_bytes`` is the sum still on the link (read by ``reserve``)."""

    def __init__(self, n_steps: int = 2) -> None:
        self.n_steps = max(1, int(n_steps))
        self._transfers: Deque[Tuple[float, float]] = deque()

    def send(self, hidden: torch.Tensor, to: str = "") -> torch.Tensor:
        self.advance_step()
        if hidden is not None and hidden.numel() > 0:
            b = float(hidden.numel() * hidden.element_size())
            self._transfers.append((b, b / self.n_steps))
        return hidden.clone() if hidden is not None else hidden

    def advance_step(self) -> None:
        self._transfers = deque((r - per, per) for r, per in self._transfers if r - per > 0.0)

    def inflight_bytes(self) -> float:
        return float(sum(r for r, _ in self._transfers))

    def sync(self) -> None:
        self._transfers.clear()


def _bank_view(params: Sequence[torch.Tensor]) -> Optional[torch.Tensor]:
    """A [E, ...] tensor aliasing ``params`` when they are consecutive slices of
    one contiguous storage, else None."""
    p0 = params[0]
    if not p0.is_contiguous():
        return None
    st = p0.untyped_storage()
    step = p0.numel()
    off0 = p0.storage_offset()
    for e, p in enumerate(params):
        if (p.untyped_storage().data_ptr() != st.data_ptr() or not p.is_contiguous()
                or p.storage_offset() != off0 + e * step or p.shape != p0.shape or p.dtype != p0.dtype):
            return None
    bank = torch.empty(0, dtype=p0.dtype, device=p0.device)
    bank.set_(st, off0, (len(params),) + tuple(p0.shape),
              (step,) + tuple(p0.stride()))
    return bank


def adjacent_router_weights(owner, gate: torch.Tensor,
                            shared_gate: Optional[torch.Tensor]) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """The router gate and, with a gated shared expert, its gate vector as the
    row right after the gate's E rows of one [E+1, H] tensor cached on
    ``owner._router_cat`` (the router then computes all E+1 logits in one
    tensor-core GEMM).  Rebuilt when either parameter is edited or moved."""
    g = gate.detach()
    if shared_gate is None:
        return g, None
    sg = shared_gate.detach()
    key = (g.data_ptr(), g._version, sg.data_ptr(), sg._version, g.dtype)
    cached = getattr(owner, "_router_cat", None)
    if cached is None or cached[0] != key:
        cached = (key, torch.cat([g, sg.reshape(1, -1).to(g.dtype)], 0).contiguous())
        owner._router_cat = cached
    cat = cached[1]
    return cat[:-1], cat[-1]


def reference_output(out: torch.Tensor, x: torch.Tensor, hidden: int) -> torch.Tensor:
    """The layer output in the input's dtype and the reference's shape
    (moe_layer.py:519, ep.py:150): ``[x.shape[0], hidden]`` for an input of two
    or more dimensions (``[B, 1, H]`` gives ``[B, H]``; like the reference's
    reshape, ``[B, S > 1, H]`` is rejected), ``[1, hidden]`` for one ``[H]``
    token."""
    if out.dtype != x.dtype:
        out = out.to(x.dtype)
    return out.reshape(x.shape[:1] + (hidden,)) if x.dim() > 1 else out


class FusedMoE(nn.Module):
    """A routed MoE block: ``gate`` -> top-k -> grouped expert GEMMs -> combine."""

    def __init__(self, num_experts: int, top_k: int, hidden_size: int, intermediate_size: int,
                 activation: str = "silu", renormalize: bool = True, dtype: torch.dtype = torch.float16,
                 *, router_dtype: Optional[torch.dtype] = None, num_shared_experts: int = 0,
                 shared_intermediate_size: int = 0, shared_expert_gate: bool = False,
                 device: Optional[torch.device] = None) -> None:
        super().__init__()
        if activation not in ACTIVATIONS:
            raise ValueError(f"unknown gated activation {activation!r}; known: {tuple(ACTIVATIONS)}")
        self.num_experts = num_experts
        self.top_k = top_k
        self.hidden_size = hidden_size
        self.intermediate_size = intermediate_size
        self.activation = activation
        self.renormalize = renormalize
        self.dtype = dtype
        self.router_dtype = router_dtype
        E, H, I = num_experts, hidden_size, intermediate_size
        fk = {"dtype": dtype, "device": device}
        self.gate = nn.Parameter(torch.empty(E, H, **fk))
        w1 = torch.empty(E, 2 * I, H, **fk)
        w2 = torch.empty(E, H, I, **fk)
        self.experts_w1 = nn.ParameterList([nn.Parameter(w1[e]) for e in range(E)])
        self.experts_w2 = nn.ParameterList([nn.Parameter(w2[e]) for e in range(E)])
        self.register_buffer("router_bias", None, persistent=False)
        self.num_shared_experts = num_shared_experts
        self.shared_intermediate_size = shared_intermediate_size
        if num_shared_experts:
            Is = shared_intermediate_size
            self.shared_w1 = nn.Parameter(torch.empty(num_shared_experts, 2 * Is, H, **fk))
            self.shared_w2 = nn.Parameter(torch.empty(num_shared_experts, H, Is, **fk))
            self.shared_gate = nn.Parameter(torch.empty(H, **fk)) if shared_expert_gate else None
        else:
            self.shared_w1 = self.shared_w2 = self.shared_gate = None
        self._bank_cache: Optional[Tuple[torch.Tensor, torch.Tensor]] = None
        self._router_cat: Optional[Tuple[tuple, torch.Tensor]] = None
        self._cache: Optional[ExpertOffloadCache] = None
        self._cpu_split_enabled = False
        self._predictor: Optional[Prediction] = None
        self._shuttle: Optional[CpuShuttle] = None
        self._last_step_t: Optional[float] = None
        self.entropy_adaptive_k = False
        self.entropy_k_min = 2
        # False: the combine keeps the reference's rounding points and order
        # (outputs match the reference bit for bit wherever the expert GEMMs
        # round identically); True: fp32 accumulation, one rounding.
        self.precise_combine = False

    # ---------------------------------------------------------------- factories
    @classmethod
    def from_config(cls, cfg, dtype: Optional[torch.dtype] = None) -> "FusedMoE":
        """Build from a ModelConfig-like object (moe_layer.py:196-225)."""
        moe = cls(num_experts=cfg.num_experts, top_k=cfg.num_experts_per_tok,
                  hidden_size=cfg.hidden_size, intermediate_size=cfg.moe_inter,
                  activation=getattr(cfg, "moe_activation", "silu"),
                  renormalize=getattr(cfg, "moe_renormalize", True), dtype=dtype or cfg.dtype)
        moe.entropy_adaptive_k = bool(getattr(cfg, "entropy_adaptive_k", False)) or env.get_entropy_k()
        moe.entropy_k_min = env.get_entropy_k_min(int(getattr(cfg, "entropy_k_min", 2)))
        return moe

    def set_router_bias(self, bias: Optional[torch.Tensor]) -> None:
        """Add a fixed per-expert bias [E] to the router logits (None clears it)."""
        self.router_bias = None if bias is None else bias.detach().float().to(self.gate.device)

    # ------------------------------------------------------------ weight banks
    def _apply(self, fn, recurse=True):
        self._bank_cache = None
        self._router_cat = None
        return super()._apply(fn, recurse)

    def invalidate_banks(self) -> None:
        """Call after replacing an expert parameter's ``.data`` directly."""
        self._bank_cache = None
        self._router_cat = None

    def _resident_banks(self) -> Tuple[torch.Tensor, torch.Tensor]:
        c = self._bank_cache
        if c is not None:
            return c
        banks = []
        for plist in (self.experts_w1, self.experts_w2):
            params = list(plist)
            bank = _bank_view(params)
            if bank is None:  # params moved one by one (e.g. .to(device)): repack once, re-point
                bank = torch.stack([p.detach() for p in params]).contiguous()
                for e, p in enumerate(params):
                    p.data = bank[e]
            banks.append(bank.detach())
        self._bank_cache = (banks[0], banks[1])
        return self._bank_cache

    def _shared_banks(self) -> Optional[Tuple[torch.Tensor, torch.Tensor]]:
        """The shared experts' weights, (w1 [S,2Is,H], w2 [S,H,Is]); the layer
        computes sum_s MLP_s(x) with K.shared_experts (each expert's output
        rounded, then summed in order, as the reference harness composes it)."""
        if not self.num_shared_experts:
            return None
        return self.shared_w1.detach(), self.shared_w2.detach()

    # ------------------------------------------------------------ offload setup
    def build_offload_cache(self, device: torch.device, lru_capacity: int) -> ExpertOffloadCache:
        """Stage the experts in a pinned host pool with ``lru_capacity`` device slots."""
        self._cache = ExpertOffloadCache(device=torch.device(device), lru_capacity=lru_capacity,
                                         dtype=self.dtype)
        self._cache.load([{"w1": self.experts_w1[e], "w2": self.experts_w2[e]}
                          for e in range(self.num_experts)])
        self.experts_w1 = nn.ParameterList()
        self.experts_w2 = nn.ParameterList()
        self._bank_cache = None
        return self._cache

    def attach_predictor(self, window: int = 32) -> None:
        if self._cache is None:
            return
        self._cache.attach_predictor(window=window)
        self._predictor = self._cache._predictor

    def enable_cpu_split(self) -> None:
        """Arm the expert split (moe_layer.py:263-282): build the int8 copies of
        the offloaded experts and, from the next forward on, compute every step's
        non-resident experts on them (``_forward_split``).  No-op without an
        offload cache."""
        if self._cache is None:
            return
        self._cache.quantize_int8_host()
        self._cpu_split_enabled = True

    def set_shuttle(self, shuttle: Optional[CpuShuttle]) -> None:
        self._shuttle = shuttle

    @property
    def cpu_split(self) -> bool:
        return self._cpu_split_enabled and self.uses_offload and self._cache.cpu_split

    @property
    def uses_offload(self) -> bool:
        return self._cache is not None

    def _since_last_step_ms(self) -> float:
        """Inter-forward window handed to the predictor (moe_layer.py:303-312).

        Mirrors the reference exactly: ``_last_step_t`` starts as None and this
        method only updates it once it is set, so unless a caller sets it the
        window is 0.0 and ``reserve`` is bounded by slot room alone."""
        t = time.perf_counter()
        if self._last_step_t is None:
            return 0.0
        dt = max(0.0, (t - self._last_step_t) * 1000.0)
        self._last_step_t = t
        return dt

    # ------------------------------------------------------------------ routing
    def _round_dtype(self) -> Optional[torch.dtype]:
        if self.router_dtype == torch.float32 or self.dtype == torch.float32:
            return None
        return self.dtype

    def _router_weights(self) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
        sg = self.shared_gate if self.num_shared_experts else None
        return adjacent_router_weights(self, self.gate, sg)

    def _router(self, x2: torch.Tensor, *, ids32: bool, ids64: bool):
        ek = self.entropy_k_min if self.entropy_adaptive_k else 0
        gate, sg = self._router_weights()
        return K.router_topk(x2, gate, self.top_k, renormalize=self.renormalize,
                             bias=self.router_bias, round_dtype=self._round_dtype(), entropy_k_min=ek,
                             shared_gate=sg, ids32=ids32, ids64=ids64)

    def _prep(self, x: torch.Tensor) -> torch.Tensor:
        if not x.is_cuda:
            raise RfMoeError("FusedMoE runs on the B200 kernels and needs a CUDA input "
                             f"(got {x.device}); there is no CPU path")
        x2 = x.reshape(-1, self.hidden_size)
        if x2.dtype != self.dtype:
            x2 = x2.to(self.dtype)
        return x2.contiguous()

    def route(self, x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """(topk_weights [M,K] fp32, topk_ids [M,K] int64) — moe_layer.py:320-344."""
        w, _, ids64, _, _ = self._router(self._prep(x), ids32=False, ids64=True)
        return w, ids64

    def prefetch_ids(self, x: torch.Tensor) -> torch.Tensor:
        return self.route(x)[1]

    # ------------------------------------------------------------------ forward
    def forward(self, x: torch.Tensor, residual: Optional[torch.Tensor] = None) -> torch.Tensor:
        out, _ = self._forward_impl(x, residual, None)
        return self._shape_like(out, x)

    def forward_add_residual(self, x: torch.Tensor, residual: torch.Tensor,
                             norm) -> Tuple[torch.Tensor, torch.Tensor]:
        """The layer with the decoder's next ``RMSNorm.forward_add_residual``
        fused into its combine (reframework/layers/norm.py:43-53):
        ``residual = moe(x) + residual; x = norm(residual)``; returns
        ``(normed, residual)``.  ``norm`` is an RMSNorm (``weight`` [H],
        ``eps``, optional ``bias``), applied in fp32 as norm.py:27-35 does."""
        bias = getattr(norm, "bias", None)
        spec = (norm.weight.detach(), None if bias is None else bias.detach(), float(norm.eps))
        res, normed = self._forward_impl(x, residual, spec)
        return self._shape_like(normed, x), self._shape_like(res, x)

    def _shape_like(self, out: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
        return reference_output(out, x, self.hidden_size)

    def _forward_impl(self, x: torch.Tensor, residual: Optional[torch.Tensor], norm):
        x2 = self._prep(x)
        res2 = None
        if residual is not None:
            res2 = residual.reshape(-1, self.hidden_size).to(self.dtype).contiguous()
        normed = None if norm is None else torch.empty_like(x2)
        shared_y = None
        shared_done = None
        sb = self._shared_banks()
        if sb is not None and not self.uses_offload:
            # The shared experts depend only on x: run them on a side stream so
            # they overlap the router, permute and gather (a few small kernels),
            # and join before the combine.  (Decode: the shared down projection
            # has few tiles and would otherwise leave most SMs idle.)
            cur = torch.cuda.current_stream(x2.device)
            side = self._side_stream(x2.device)
            side.wait_stream(cur)
            with torch.cuda.stream(side):
                shared_y = K.shared_experts(x2, sb[0], sb[1], self.activation)
                shared_done = torch.cuda.Event()
                shared_done.record(side)
            x2.record_stream(side)
            shared_y.record_stream(cur)
        w, ids32, _, _, sscale = self._router(x2, ids32=True, ids64=False)
        if sb is not None and self.uses_offload:
            shared_y = K.shared_experts(x2, sb[0], sb[1], self.activation)
        if self.cpu_split:
            if shared_y is not None or res2 is not None or norm is not None:
                raise RfMoeError("the expert split computes the routed experts only (no shared experts, "
                                 "residual or fused norm)")
            out = self._forward_split(x2, w, ids32)
        elif self.uses_offload:
            out = self._forward_offload(x2, w, ids32, shared_y, sscale, res2, norm, normed)
        else:
            w1b, w2b = self._resident_banks()
            out = K.moe_experts(x2, w1b, w2b, w, ids32, activation=self.activation,
                                shared_y=shared_y, shared_scale=sscale, residual=res2,
                                precise=self.precise_combine, norm=norm, norm_out=normed,
                                before_combine=shared_done)
        return out, normed

    def _side_stream(self, device: torch.device) -> torch.cuda.Stream:
        s = getattr(self, "_side", None)
        if s is None or s.device != device:
            s = self._side = torch.cuda.Stream(device=device)
        return s

    def _forward_offload(self, x2, w, ids32, shared_y, sscale, res2, norm=None, normed=None):
        """Exact streaming forward through the cache's device slots.

        Resident routed experts run first (one grouped launch); each missing
        expert is copied into a slot on the copy stream (evicting per policy,
        never an expert still to be computed this step) and computed as soon
        as its copy lands, so copies overlap the GEMMs.  Restates the exact
        chunked path of moe_layer.py:354-420 without its chunk barriers.
        """
        global _warned_max_pack
        if env.get_max_pack() is not None and not _warned_max_pack:
            logger.warning("RE_MAX_PACK is ignored: the offload forward is always exact")
            _warned_max_pack = True
        cache = self._cache
        dev = x2.device
        T, H = x2.shape
        E, I = self.num_experts, self.intermediate_size
        p = K.permute(ids32, E, x=x2)
        counts = p.counts.to("cpu").tolist()  # host sync: which experts this step needs
        active = [e for e in range(E) if counts[e] > 0]
        resident = [e for e in active if e in cache._lru]
        missing = [e for e in active if e not in cache._lru]
        h = torch.empty(p.rows_cap, I, dtype=x2.dtype, device=dev)
        y = torch.empty(p.rows_cap, H, dtype=x2.dtype, device=dev)

        def run(experts: List[int]) -> None:
            cache.wait_ready(experts)
            slots = torch.full((E,), -1, dtype=torch.int32)
            for e in experts:
                slots[e] = cache.slot_of(e)
            slot_t = slots.pin_memory().to(dev, non_blocking=True)
            grp = torch.tensor(experts, dtype=torch.int32).pin_memory().to(dev, non_blocking=True)
            K.grouped_gemm_gated(p.x_perm, cache.pool_w1, p.offsets, p.counts, h, slot=slot_t,
                                 groups=grp, activation=self.activation)
            K.grouped_gemm_down(h, cache.pool_w2, p.offsets, p.counts, y, slot=slot_t, groups=grp)

        for e in resident:
            cache.stats.hits += 1
            cache._lru.move_to_end(e)
        if resident:
            run(resident)
        pending = set(missing)
        soft = set(cache._next_reserve) - set(active)
        for e in missing:
            cache._fill(e, hard=set(pending), soft=soft)
            cache._lru.move_to_end(e)
            run([e])
            pending.discard(e)
        cache._evict((), soft)  # only trims a pool that had to grow past capacity
        out = torch.empty(T, H, dtype=x2.dtype, device=dev)
        K.combine(y, p.row_of_slot, w, out, shared_y=shared_y, shared_scale=sscale, residual=res2,
                  precise=self.precise_combine, norm=norm, norm_out=normed)
        if self._predictor is not None:
            self._predictor.record_step(active, is_prefill=(T > 1), forward_ms=self._since_last_step_ms(),
                                        inflight_bytes=(self._shuttle.inflight_bytes()
                                                        if self._shuttle is not None else 0.0))
        return out

    def _forward_split(self, x2, w, ids32):
        """The CPU/GPU expert split (moe_layer.py:523-627), B200 form.

        The routed experts resident in the device slots ("hits") run in the
        layer dtype on the grouped tensor-core GEMMs; the others ("misses") run
        on their int8 copies (fused.py:140-197), which cross PCIe at half the
        bytes of the 16-bit weights and are computed on the GPU with exact int8
        GEMMs; the halves meet in fp32 per token (rf_moe_split_combine).  The
        misses are then loaded resident for the next step (``reactive_load``).
        Every miss is computed (no RE_MAX_PACK cap) and slot (t, k) belongs to
        token t (the reference's ``repeat(K)`` mapping, fused.py:118,175, is
        wrong for K > 1).
        """
        cache = self._cache
        dev = x2.device
        T, H = x2.shape
        E, I = self.num_experts, self.intermediate_size
        p = K.permute(ids32, E, x=x2)
        counts = p.counts.to("cpu").tolist()  # host sync: which experts this step routes to
        routed = [e for e in range(E) if counts[e] > 0]
        (pool_w1, pool_w2, hit_slots), misses = cache.split_prefetch(routed)
        hits = sorted(hit_slots)
        if self._shuttle is not None:
            self._shuttle.send(x2)
        y = torch.empty(p.rows_cap, H, dtype=x2.dtype, device=dev)
        if hits:
            slots = torch.full((E,), -1, dtype=torch.int32)
            for e in hits:
                slots[e] = hit_slots[e]
            slot_t = slots.pin_memory().to(dev, non_blocking=True)
            grp = torch.tensor(hits, dtype=torch.int32).pin_memory().to(dev, non_blocking=True)
            h = torch.empty(p.rows_cap, I, dtype=x2.dtype, device=dev)
            K.grouped_gemm_gated(p.x_perm, pool_w1, p.offsets, p.counts, h, slot=slot_t, groups=grp,
                                 activation=self.activation)
            K.grouped_gemm_down(h, pool_w2, p.offsets, p.counts, y, slot=slot_t, groups=grp)
        y8 = torch.empty(p.rows_cap, H, dtype=torch.float32, device=dev)
        miss_mask = torch.zeros(E, dtype=torch.uint8)
        if misses:
            miss_mask[misses] = 1
            q1, q2, rows8 = cache.int8_banks(misses)
            n = len(misses)
            slot8 = torch.full((E,), -1, dtype=torch.int32)
            for e, k in rows8.items():
                slot8[e] = k
            slot8 = slot8.pin_memory().to(dev, non_blocking=True)
            grp8 = torch.tensor(misses, dtype=torch.int32).pin_memory().to(dev, non_blocking=True)
            f32 = dict(dtype=torch.float32, device=dev)
            xq = torch.empty(p.rows_cap, H, dtype=torch.int8, device=dev)
            amax, xs = torch.empty(n, **f32), torch.empty(n, **f32)
            K.int8_quantize(p.x_perm, p.offsets, p.counts, grp8, xq, xs, amax)
            scales = cache._int8_scales_dev  # [E, 2]: w1, w2
            inter = torch.empty(p.rows_cap, I, **f32)
            amax2, iscale = torch.empty(n, **f32), torch.empty(n, **f32)
            K.int8_grouped_gemm(xq, q1, p.offsets, p.counts, grp8, slot8, xs, scales[:, 0], 2, inter, gated=True,
                                activation=self.activation, amax_out=amax2)
            iq = torch.empty(p.rows_cap, I, dtype=torch.int8, device=dev)
            K.int8_quantize(inter, p.offsets, p.counts, grp8, iq, iscale, amax2, compute_amax=False)
            K.int8_grouped_gemm(iq, q2, p.offsets, p.counts, grp8, slot8, iscale, scales[:, 1], 2, y8, gated=False,
                                row_weights=w.float().contiguous().reshape(-1), src_slot=p.src_slot)
            cache.int8_release()
        out = torch.empty(T, H, dtype=x2.dtype, device=dev)
        K.split_combine(y, y8, p.row_of_slot, ids32, miss_mask.pin_memory().to(dev, non_blocking=True), w, out)
        cache.reactive_load(misses)
        if self._predictor is not None:
            self._predictor.record_step(routed, is_prefill=(T > 1), forward_ms=self._since_last_step_ms(),
                                        inflight_bytes=(self._shuttle.inflight_bytes()
                                                        if self._shuttle is not None else 0.0))
        return out

    # --------------------------------------------------------------- (de)serial
    def state_dict(self, *args, prefix: str = "", result: Optional[dict] = None, **kwargs) -> Dict[str, torch.Tensor]:
        """HF names: ``gate.weight``, ``experts.{e}.{gate,up,down}_proj.weight`` (moe_layer.py:631-642)."""
        result = {} if result is None else result
        pre = f"{prefix}." if prefix else ""
        result[f"{pre}gate.weight"] = self.gate
        I = self.intermediate_size
        for e in range(len(self.experts_w1)):
            p = f"{pre}experts.{e}"
            result[f"{p}.gate_proj.weight"] = self.experts_w1[e][:I]
            result[f"{p}.up_proj.weight"] = self.experts_w1[e][I:]
            result[f"{p}.down_proj.weight"] = self.experts_w2[e]
        if self.num_shared_experts:
            Is = self.shared_intermediate_size
            for s in range(self.num_shared_experts):
                p = f"{pre}shared_experts.{s}"
                result[f"{p}.gate_proj.weight"] = self.shared_w1[s][:Is]
                result[f"{p}.up_proj.weight"] = self.shared_w1[s][Is:]
                result[f"{p}.down_proj.weight"] = self.shared_w2[s]
            if self.shared_gate is not None:
                result[f"{pre}shared_expert_gate.weight"] = self.shared_gate
        return result

    def load_state_dict(self, state_dict: Dict[str, torch.Tensor], *args, prefix: str = "", **kwargs) -> None:
        """Copy HF-named tensors into the (bank-backed) parameters (moe_layer.py:644-660).
        Expert weights may also use the PhiMoE / Mixtral names ``w1`` / ``w3`` /
        ``w2`` (checkpoint/loader.py:83-103)."""
        pre = f"{prefix}." if prefix else ""
        with torch.no_grad():
            g = f"{pre}gate.weight"
            if g in state_dict:
                self.gate.copy_(state_dict[g].detach().to(dtype=self.dtype))
            I = self.intermediate_size
            for e in range(len(self.experts_w1)):
                p = f"{pre}experts.{e}"
                for half, param in (("gate_proj", self.experts_w1[e][:I]), ("up_proj", self.experts_w1[e][I:]),
                                    ("down_proj", self.experts_w2[e])):
                    t = expert_tensor(state_dict, p, half)
                    if t is not None:
                        param.copy_(t.detach().to(dtype=self.dtype))
            if self.num_shared_experts:
                Is = self.shared_intermediate_size
                for s in range(self.num_shared_experts):
                    p = f"{pre}shared_experts.{s}"
                    for half, param in (("gate_proj", self.shared_w1[s][:Is]), ("up_proj", self.shared_w1[s][Is:]),
                                        ("down_proj", self.shared_w2[s])):
                        key = f"{p}.{half}.weight"
                        if key in state_dict:
                            param.copy_(state_dict[key].detach().to(dtype=self.dtype))
                key = f"{pre}shared_expert_gate.weight"
                if self.shared_gate is not None and key in state_dict:
                    self.shared_gate.copy_(state_dict[key].detach().reshape(-1).to(dtype=self.dtype))
