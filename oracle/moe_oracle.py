"""CPU oracle for the MoE-layer forward — TEST INFRASTRUCTURE ONLY.

This module restates, on the CPU, the algorithm of Reframework's torch MoE
layer so the CUDA path can be checked against it.  It is imported only by
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
``--impl reference`` leg; the product package never imports it.

Each function cites the reference line it restates (paths relative to the
reference project root).  The arithmetic deliberately uses the same torch CPU
operators in the same dtypes and the same order as the reference, so that on
the same inputs the oracle reproduces the reference's outputs bit for bit
(pinned by ``tests/test_oracle_golden.py`` against fixtures produced by running
the reference itself, ``tests/golden/make_golden.py``).

The integer part (grouping (token, slot) pairs by expert) is restated in numpy
as a stable counting sort (``permutation``).

Harness adaptations (not in the reference; both are opt-in):
  * fp32 router with a per-expert bias: ``logits = x.float() @ gate.float().T
    + bias``, then ``torch_fused_topk``.  The reference's ``FusedMoE.route``
    runs the router GEMM in the layer dtype (reframework/moe/moe_layer.py:324).
  * shared experts: ``out += sigmoid(x.w_s) * MLP(x)`` (gated) or
    ``out += sum_s MLP_s(x)``; the MLP restates reframework/layers/mlp.py:35-39
    with the dtype rule of reframework/layers/linear.py:41-49.
"""

from __future__ import annotations

import math
from typing import Dict, Optional, Tuple

import numpy as np
import torch
import torch.nn.functional as F

__all__ = [
    "gated_act_and_mul",
    "torch_fused_topk",
    "router_logits",
    "route",
    "route_entropy_k",
    "permutation",
    "fused_experts",
    "dense_mlp",
    "moe_forward",
    "forward_streaming",
    "sym_int8_quantize",
    "masked_experts",
    "int8_experts",
    "split_forward",
    "shard_range",
]


def gated_act_and_mul(activation: str, x: torch.Tensor) -> torch.Tensor:
    """``act(x[..., :I]) * x[..., I:]`` — reframework/layers/activation.py:15-24,52-59."""
    d = x.shape[-1] // 2
    g, u = x[..., :d], x[..., d:]
    if activation == "silu":
        return F.silu(g) * u
    if activation == "gelu":
        return F.gelu(g) * u
    if activation == "gelu_tanh":
        return F.gelu(g, approximate="tanh") * u
    raise ValueError(f"unknown gated activation {activation!r}")


def torch_fused_topk(logits: torch.Tensor, topk: int, renormalize: bool) -> Tuple[torch.Tensor, torch.Tensor]:
    """softmax(float32) -> topk (sorted, descending) -> optional renorm.

    Restates reframework/moe/fused.py:32-46.  Returns (fp32 weights [T,K],
    int64 ids [T,K]).
    """
    probs = torch.softmax(logits.float(), dim=-1)
    w, ids = torch.topk(probs, topk, dim=-1)
    if renormalize:
        w = w / w.sum(dim=-1, keepdim=True)
    return w.contiguous(), ids.contiguous()


def router_logits(x: torch.Tensor, gate: torch.Tensor, *, bias: Optional[torch.Tensor] = None,
                  fp32: bool = True, layer_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    """Router logits [T,E].

    ``fp32=False`` restates reframework/moe/moe_layer.py:324 (``F.linear`` in
    the layer dtype).  ``fp32=True`` is the harness's fp32 router (x and the
    gate upcast, plus the optional bias).
    """
    if fp32:
        lg = x.float() @ gate.float().t()
        if bias is not None:
            lg = lg + bias.float()
        return lg
    dt = layer_dtype or gate.dtype
    lg = F.linear(x.to(dt), gate.to(dt))
    if bias is not None:
        lg = lg + bias.to(lg.dtype)
    return lg


def route(x: torch.Tensor, gate: torch.Tensor, top_k: int, renormalize: bool, *,
          bias: Optional[torch.Tensor] = None, fp32: bool = True,
          layer_dtype: Optional[torch.dtype] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """``FusedMoE.route`` — reframework/moe/moe_layer.py:320-344 (default branch)."""
    return torch_fused_topk(router_logits(x, gate, bias=bias, fp32=fp32, layer_dtype=layer_dtype),
                            top_k, renormalize)


def route_entropy_k(logits: torch.Tensor, top_k: int, k_min: int, num_experts: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """Entropy-adaptive top-k branch — reframework/moe/moe_layer.py:327-342."""
    probs = F.softmax(logits.float(), dim=-1)
    Hn = -(probs * probs.clamp_min(1e-9).log()).sum(-1) / math.log(num_experts)
    k_dyn = (k_min + (top_k - k_min) * Hn).round().long().clamp(min=k_min, max=top_k)
    top_w, top_idx = torch.topk(probs, top_k, dim=-1)
    mask = torch.arange(top_k).unsqueeze(0) < k_dyn.unsqueeze(1)
    top_w = torch.where(mask, top_w, torch.zeros_like(top_w))
    top_w = top_w / top_w.sum(-1, keepdim=True).clamp_min(1e-9)
    return top_w, top_idx


def permutation(ids: np.ndarray, num_experts: int) -> Tuple[np.ndarray, np.ndarray]:
    """Group flattened (token, slot) pairs by expert — stable counting sort.

    Restates the grouping of reframework/moe/fused.py:71-80: ``flat_token =
    arange(M).repeat_interleave(K)`` and, for each active expert in ascending
    order, the rows ``flat_expert == e`` in ascending flat index t*K+k.

    Returns ``(counts [E] int64, order [T*K] int64)``: ``order`` lists the flat
    indices t*K+k expert by expert (expert-major, ascending within an expert).
    """
    flat = np.asarray(ids, dtype=np.int64).reshape(-1)
    counts = np.bincount(flat, minlength=num_experts).astype(np.int64)
    starts = np.concatenate([[0], np.cumsum(counts)[:-1]])
    order = np.empty(flat.size, dtype=np.int64)
    cursor = starts.copy()
    # counting-sort scatter; a python loop is fine for oracle sizes, numpy's
    # stable argsort gives the same answer and is used for large inputs
    if flat.size <= 4096:
        for i, e in enumerate(flat):
            order[cursor[e]] = i
            cursor[e] += 1
    else:
        order = np.argsort(flat, kind="stable").astype(np.int64)
    return counts, order


def fused_experts(hidden_states: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor,
                  topk_weights: torch.Tensor, topk_ids: torch.Tensor,
                  activation: str = "silu") -> torch.Tensor:
    """Routed experts, summed — reframework/moe/fused.py:49-87.

    Per active expert e (ascending): gather its rows, ``x @ w1[e].T`` in the
    weight dtype, gated activation, ``@ w2[e].T``, scale by the routing weight
    cast to the activation dtype, ``index_add_`` into an output of the
    activation dtype.
    """
    M, H = hidden_states.shape
    K = topk_ids.shape[1]
    E = w1.shape[0]
    out = torch.zeros((M, H), dtype=hidden_states.dtype)
    flat_expert = topk_ids.reshape(-1)
    flat_weight = topk_weights.reshape(-1)
    flat_token = torch.arange(M).repeat_interleave(K)
    counts = torch.bincount(flat_expert, minlength=E)
    for e in torch.nonzero(counts, as_tuple=False).flatten().tolist():
        sel = flat_expert == e
        tok = flat_token[sel]
        w = flat_weight[sel].to(hidden_states.dtype)
        x = hidden_states[tok]
        gu = x.to(w1.dtype) @ w1[e].t()
        inter = gated_act_and_mul(activation, gu)
        y = inter @ w2[e].t()
        y = y * w.unsqueeze(-1)
        out.index_add_(0, tok, y)
    return out


def dense_mlp(x: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor, activation: str = "silu") -> torch.Tensor:
    """Dense gated MLP — reframework/layers/mlp.py:35-39 with the Linear dtype
    rule of reframework/layers/linear.py:41-49 (fp16 computes in fp32)."""
    def linear(a, w):
        compute = torch.float32 if (a.dtype == torch.float16 or w.dtype == torch.float16) else a.dtype
        return F.linear(a.to(compute), w.to(compute)).to(a.dtype)
    return linear(gated_act_and_mul(activation, linear(x, w1)), w2)


def moe_forward(x: torch.Tensor, gate: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor, *,
                top_k: int, renormalize: bool = True, bias: Optional[torch.Tensor] = None,
                router_fp32: bool = True, activation: str = "silu",
                shared_w1: Optional[torch.Tensor] = None, shared_w2: Optional[torch.Tensor] = None,
                shared_gate: Optional[torch.Tensor] = None,
                entropy_k_min: Optional[int] = None) -> Dict[str, torch.Tensor]:
    """Resident-mode ``FusedMoE.forward`` — reframework/moe/moe_layer.py:451-519.

    Returns ``{"out", "weights", "ids", "logits"}``.  With shared experts the
    output adds the harness composition described in the module docstring.
    """
    logits = router_logits(x, gate, bias=bias, fp32=router_fp32, layer_dtype=w1.dtype)
    if entropy_k_min is not None:
        w, ids = route_entropy_k(logits, top_k, entropy_k_min, gate.shape[0])
    else:
        w, ids = torch_fused_topk(logits, top_k, renormalize)
    out = fused_experts(x, w1, w2, w, ids, activation)
    if shared_w1 is not None:
        sh = None
        for s in range(shared_w1.shape[0]):
            y = dense_mlp(x, shared_w1[s], shared_w2[s], activation)
            sh = y if sh is None else sh + y
        if shared_gate is not None:
            sg = torch.sigmoid(x.float() @ shared_gate.float())
            sh = (sh.float() * sg.unsqueeze(-1)).to(x.dtype)
        out = out + sh
    return {"out": out, "weights": w, "ids": ids, "logits": logits}


def forward_streaming(x: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor,
                      topk_weights: torch.Tensor, topk_ids: torch.Tensor,
                      chunk_size: int, activation: str = "silu") -> torch.Tensor:
    """Exact offload forward — reframework/moe/moe_layer.py:354-420.

    Unique routed experts are processed ``chunk_size`` at a time; each chunk's
    (token, slot) pairs run through ``fused_experts`` with K=1 and are
    accumulated into an fp32 buffer with ``index_add_``.
    """
    uniq = sorted(set(int(i) for i in topk_ids.reshape(-1).tolist() if i >= 0))
    out = torch.zeros(x.shape, dtype=torch.float32)
    E = w1.shape[0]
    for i in range(0, len(uniq), chunk_size):
        chunk = uniq[i:i + chunk_size]
        local = {g: k for k, g in enumerate(chunk)}
        remap = torch.full((E,), -1, dtype=torch.long)
        for g, loc in local.items():
            remap[g] = loc
        mask = torch.isin(topk_ids, torch.tensor(chunk, dtype=topk_ids.dtype))
        if not mask.any():
            continue
        t_idx, k_idx = mask.nonzero(as_tuple=True)
        sel_w = topk_weights[t_idx, k_idx]
        loc_ids = remap[topk_ids[t_idx, k_idx]]
        valid = (loc_ids >= 0) & (sel_w > 0)
        if not valid.any():
            continue
        bank1 = torch.stack([w1[g] for g in chunk])
        bank2 = torch.stack([w2[g] for g in chunk])
        part = fused_experts(x[t_idx][valid], bank1, bank2, sel_w[valid].unsqueeze(-1),
                             loc_ids[valid].unsqueeze(-1), activation)
        out.index_add_(0, t_idx[valid], part.to(torch.float32))
    return out.to(x.dtype)


def sym_int8_quantize(w: torch.Tensor) -> Tuple[torch.Tensor, float]:
    """Symmetric per-tensor int8 — reframework/moe/offload_cache.py:58-72:
    scale = max|w| / 127 (fp32), codes = round(w / scale) clamped to +-127;
    an all-zero tensor gets scale 1.0 and zero codes."""
    amax = w.abs().max().float()
    if amax <= 0:
        return torch.zeros_like(w, dtype=torch.int8), 1.0
    scale = amax / 127.0
    wq = (w.float() / scale).round().clamp(-127, 127).to(torch.int8).contiguous()
    return wq, float(scale)


def masked_experts(hidden_states: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor,
                   topk_weights: torch.Tensor, topk_ids: torch.Tensor, active: torch.Tensor,
                   activation: str = "silu") -> torch.Tensor:
    """The GPU half of the CPU/GPU split — reframework/moe/fused.py:89-137:
    ``fused_experts`` over the slots with ``active`` set only (``topk_ids``
    local rows of ``w1``/``w2``).  Slot (t, k) belongs to token t; the
    reference's ``arange(M).repeat(K)`` (fused.py:118) maps it to token
    (t*K + k) % M instead, which differs for K > 1, so this restatement uses
    ``repeat_interleave`` (the two agree for K = 1)."""
    M, H = hidden_states.shape
    K = topk_ids.shape[1]
    E = w1.shape[0]
    out = torch.zeros((M, H), dtype=hidden_states.dtype)
    flat_expert = topk_ids.reshape(-1)
    flat_weight = topk_weights.reshape(-1)
    flat_active = active.reshape(-1)
    flat_token = torch.arange(M).repeat_interleave(K)
    active_ids = torch.where(flat_active, flat_expert, torch.full_like(flat_expert, -1))
    counts = torch.bincount(active_ids[flat_active], minlength=E)
    for e in torch.nonzero(counts, as_tuple=False).flatten().tolist():
        sel = (flat_expert == e) & flat_active
        tok = flat_token[sel]
        w = flat_weight[sel].to(hidden_states.dtype)
        x = hidden_states[tok]
        gu = x.to(w1.dtype) @ w1[e].t()
        inter = gated_act_and_mul(activation, gu)
        y = inter @ w2[e].t()
        y = y * w.unsqueeze(-1)
        out.index_add_(0, tok, y)
    return out


def int8_experts(hidden_states: torch.Tensor, w1q: torch.Tensor, w2q: torch.Tensor, scales1: torch.Tensor,
                 scales2: torch.Tensor, topk_weights: torch.Tensor, topk_ids: torch.Tensor,
                 active: torch.Tensor, activation: str = "silu") -> torch.Tensor:
    """The int8 half of the CPU/GPU split — reframework/moe/fused.py:140-197
    (same token mapping fix as ``masked_experts``).  Per active expert e
    (ascending): its rows in fp32 quantized to int8 with one scale for the
    whole block, ``int8 x int8 -> int32`` GEMM against ``w1q[e]``, dequantized
    by ``block scale * scales1[e]``, gated activation in fp32, the result
    quantized again per block, a second int8 GEMM against ``w2q[e]``,
    dequantized, scaled by the fp32 routing weight and ``index_add_``-ed into an
    fp32 output."""
    M, H = hidden_states.shape
    K = topk_ids.shape[1]
    E = w1q.shape[0]
    x2 = hidden_states.float()
    out = torch.zeros((M, H), dtype=torch.float32)
    flat_expert = topk_ids.reshape(-1)
    flat_weight = topk_weights.float().reshape(-1)
    flat_active = active.reshape(-1)
    flat_token = torch.arange(M).repeat_interleave(K)
    active_ids = torch.where(flat_active, flat_expert, torch.full_like(flat_expert, -1))
    counts = torch.bincount(active_ids[flat_active], minlength=E)
    for e in torch.nonzero(counts, as_tuple=False).flatten().tolist():
        sel = (flat_expert == e) & flat_active
        tok = flat_token[sel]
        w = flat_weight[sel]
        x = x2[tok]
        xq, xs = sym_int8_quantize(x)
        gu = torch._int_mm(xq, w1q[e].t().contiguous()).float() * (xs * float(scales1[e]))
        inter = gated_act_and_mul(activation, gu)
        iq, iscale = sym_int8_quantize(inter)
        y = torch._int_mm(iq, w2q[e].t().contiguous()).float() * (iscale * float(scales2[e]))
        y = y * w.unsqueeze(-1)
        out.index_add_(0, tok, y)
    return out


def split_forward(x: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor, topk_weights: torch.Tensor,
                  topk_ids: torch.Tensor, resident, activation: str = "silu") -> Dict[str, torch.Tensor]:
    """One step of the CPU/GPU split forward — reframework/moe/moe_layer.py:523-627
    with the host int8 bank of offload_cache.py:386-434.  The routed experts
    resident before the step ("hits", ascending) run in the layer dtype
    (``masked_experts``); the others ("misses", ascending) run on their int8
    copies (``int8_experts``); out = (hits.float() + misses).to(x.dtype).
    Every miss is computed (the reference packs at most RE_MAX_PACK of them,
    offload_cache.py:417-421)."""
    E = w1.shape[0]
    routed = sorted(set(int(i) for i in topk_ids.reshape(-1).tolist()))
    hits = [e for e in routed if e in resident]
    misses = [e for e in routed if e not in resident]
    out = torch.zeros(x.shape, dtype=x.dtype)
    if hits:
        remap = torch.full((E,), -1, dtype=torch.long)
        for k, e in enumerate(hits):
            remap[e] = k
        loc = remap[topk_ids]
        out = masked_experts(x, w1[hits], w2[hits], topk_weights, loc.clamp_min(0), loc >= 0, activation)
    half = torch.zeros(x.shape, dtype=torch.float32)
    if misses:
        remap = torch.full((E,), -1, dtype=torch.long)
        for k, e in enumerate(misses):
            remap[e] = k
        loc = remap[topk_ids]
        q = [sym_int8_quantize(w1[e]) for e in misses], [sym_int8_quantize(w2[e]) for e in misses]
        w1q = torch.stack([a for a, _ in q[0]])
        w2q = torch.stack([a for a, _ in q[1]])
        s1 = torch.tensor([b for _, b in q[0]], dtype=torch.float32)
        s2 = torch.tensor([b for _, b in q[1]], dtype=torch.float32)
        half = int8_experts(x, w1q, w2q, s1, s2, topk_weights, loc.clamp_min(0), loc >= 0, activation)
    return {"out": (out.float() + half).to(x.dtype), "hits": hits, "misses": misses, "gpu_half": out,
            "int8_half": half}


def shard_range(num_experts: int, ep_size: int, ep_rank: int) -> Tuple[int, int]:
    """Contiguous expert block of one EP rank — reframework/parallel/ep.py:45-55."""
    base, rem = divmod(num_experts, ep_size)
    size = base + (1 if ep_rank < rem else 0)
    start = ep_rank * base + min(ep_rank, rem)
    return start, start + size
