"""Thin torch-facing wrappers over the rf_moe C ABI, one per stage.

Tensors are CUDA tensors (the library launches on the current torch stream
of their device); scratch buffers come from torch's caching allocator.
Nothing here falls back to torch math: a missing library or an unsupported
case raises :class:`reframework_b200._lib.RfMoeError`.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, Optional, Tuple

import torch

from . import _lib
from ._lib import check, dtype_code, lib, ptr, stream_of

ALIGN = 128  # expert segment alignment of the permuted row layout (one GEMM m-tile)


def _require_cuda(*ts: Optional[torch.Tensor]) -> torch.device:
    dev = None
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise _lib.RfMoeError("reframework_b200 kernels need CUDA tensors "
                                  f"(got a tensor on {t.device}); there is no CPU path")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise _lib.RfMoeError(f"tensors on different devices: {dev} vs {t.device}")
    return dev


def rows_capacity(n_pairs: int, num_experts: int, align: int = ALIGN) -> int:
    return int(lib().rf_moe_rows_capacity(n_pairs, num_experts, align))


# ----------------------------------------------------------------------- K1
def router_topk(x: torch.Tensor, gate: Optional[torch.Tensor], top_k: int, *, renormalize: bool = True,
                bias: Optional[torch.Tensor] = None, round_dtype: Optional[torch.dtype] = None,
                entropy_k_min: int = 0, shared_gate: Optional[torch.Tensor] = None,
                want_logits: bool = False, ids64: bool = False, ids32: bool = True):
    """Router logits + softmax + top-k (+ renorm).  ``gate=None``: ``x`` holds logits.

    Returns ``(weights fp32 [T,K], ids32 or None, ids64 or None, logits or None,
    shared_scale or None)``.
    """
    dev = _require_cuda(x, gate, bias, shared_gate)
    x = x.contiguous()
    T, H = x.shape
    E = gate.shape[0] if gate is not None else H
    if gate is not None:
        gate = gate.contiguous()
    w = torch.empty(T, top_k, dtype=torch.float32, device=dev)
    i32 = torch.empty(T, top_k, dtype=torch.int32, device=dev) if ids32 else None
    i64 = torch.empty(T, top_k, dtype=torch.int64, device=dev) if ids64 else None
    lg = torch.empty(T, E, dtype=torch.float32, device=dev) if want_logits else None
    ss = torch.empty(T, dtype=torch.float32, device=dev) if shared_gate is not None else None
    if bias is not None:
        bias = bias.to(device=dev, dtype=torch.float32).contiguous()
    if shared_gate is not None:
        shared_gate = shared_gate.to(dtype=gate.dtype).contiguous()
    ws_bytes = 0
    ws = None
    if gate is not None and T > 0:
        ws_bytes = int(lib().rf_moe_router_workspace_size(T, H, E, int(shared_gate is not None)))
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    rc = lib().rf_moe_router_topk(
        ptr(x), dtype_code(x.dtype), ptr(gate), dtype_code(gate.dtype if gate is not None else x.dtype),
        ptr(bias), T, H, E, top_k, int(bool(renormalize)),
        -1 if round_dtype is None else dtype_code(round_dtype), int(entropy_k_min),
        ptr(shared_gate), ptr(ss), ptr(w), ptr(i32), ptr(i64), ptr(lg), ptr(ws), ws_bytes,
        stream_of(dev))
    check(rc, "rf_moe_router_topk")
    return w, i32, i64, lg, ss


# ----------------------------------------------------------------------- K2
@dataclass
class Permutation:
    offsets: torch.Tensor       # [E+1] int32, padded row starts (offsets[E] = rows used)
    counts: torch.Tensor        # [E] int32
    row_of_slot: torch.Tensor   # [T*K] int32
    src_slot: torch.Tensor      # [rows_cap] int32 (-1 on pad rows)
    x_perm: Optional[torch.Tensor]  # [rows_cap, H]
    rows_cap: int
    align: int


def permute(ids32: torch.Tensor, num_experts: int, *, align: int = ALIGN,
            x: Optional[torch.Tensor] = None) -> Permutation:
    dev = _require_cuda(ids32, x)
    if ids32.dtype != torch.int32:
        raise _lib.RfMoeError("permute: ids must be int32")
    ids32 = ids32.contiguous()
    T, K = ids32.shape
    E = int(num_experts)
    cap = rows_capacity(T * K, E, align)
    offsets = torch.empty(E + 1, dtype=torch.int32, device=dev)
    counts = torch.empty(E, dtype=torch.int32, device=dev)
    row_of_slot = torch.empty(T * K, dtype=torch.int32, device=dev)
    src_slot = torch.empty(max(cap, 1), dtype=torch.int32, device=dev)
    ws_bytes = int(lib().rf_moe_permute_workspace_size(T * K, E))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    x_perm = None
    H = 0
    if x is not None:
        x = x.contiguous()
        H = x.shape[1]
        x_perm = torch.empty(max(cap, 1), H, dtype=x.dtype, device=dev)
    rc = lib().rf_moe_permute(ptr(ids32), T, K, E, align, ptr(x), dtype_code(x.dtype) if x is not None else 0,
                              H, ptr(offsets), ptr(counts), ptr(row_of_slot), ptr(src_slot), ptr(x_perm),
                              ptr(ws), ws_bytes, stream_of(dev))
    check(rc, "rf_moe_permute")
    return Permutation(offsets, counts, row_of_slot, src_slot, x_perm, cap, align)


def gather_rows(src: torch.Tensor, index: torch.Tensor, out: torch.Tensor, *, index_div: int = 1,
                n_rows_dev: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``out[r] = src[index[r] // index_div]`` (zero where index < 0)."""
    dev = _require_cuda(src, index, out, n_rows_dev)
    row_bytes = src.shape[1] * src.element_size()
    rc = lib().rf_moe_gather_rows(ptr(src), ptr(index), index_div, out.shape[0], ptr(n_rows_dev),
                                  row_bytes, ptr(out), stream_of(dev))
    check(rc, "rf_moe_gather_rows")
    return out


# -------------------------------------------------------------------- K3/K4
def grouped_gemm_gated(a: torch.Tensor, w1: torch.Tensor, offsets: torch.Tensor, counts: torch.Tensor,
                       out: torch.Tensor, *, slot: Optional[torch.Tensor] = None,
                       groups: Optional[torch.Tensor] = None, activation: str = "silu") -> torch.Tensor:
    """``out[r] = act(a[r] . w1[s, :I]^T) * (a[r] . w1[s, I:]^T)`` per expert segment."""
    dev = _require_cuda(a, w1, offsets, counts, out, slot, groups)
    S, I2, H = w1.shape
    E = counts.shape[0]
    if activation not in _lib.ACTIVATIONS:
        raise ValueError(f"unknown gated activation {activation!r}; known: {tuple(_lib.ACTIVATIONS)}")
    rc = lib().rf_moe_grouped_gemm_gated(
        ptr(a), ptr(w1), ptr(out), ptr(offsets), ptr(counts), ptr(slot), ptr(groups),
        0 if groups is None else groups.numel(), E, S, a.shape[0], H, I2 // 2,
        dtype_code(a.dtype), _lib.ACTIVATIONS[activation], stream_of(dev))
    check(rc, "rf_moe_grouped_gemm_gated")
    return out


def grouped_gemm_gated_gather(x: torch.Tensor, src_slot: torch.Tensor, topk: int, w1: torch.Tensor,
                              offsets: torch.Tensor, counts: torch.Tensor, out: torch.Tensor, *,
                              slot: Optional[torch.Tensor] = None, groups: Optional[torch.Tensor] = None,
                              activation: str = "silu") -> bool:
    """``out[r] = act(x[src_slot[r] // topk] . w1[s, :I]^T) * (...)`` with the row
    gather fused into the tensor-core operand load.  Returns False (nothing
    launched) when the shape or dtype needs the explicit gather instead."""
    dev = _require_cuda(x, src_slot, w1, offsets, counts, out, slot, groups)
    if activation not in _lib.ACTIVATIONS:
        raise ValueError(f"unknown gated activation {activation!r}; known: {tuple(_lib.ACTIVATIONS)}")
    x = x.contiguous()
    S, I2, H = w1.shape
    E = counts.shape[0]
    rc = lib().rf_moe_grouped_gemm_gated_gather(
        ptr(x), x.shape[0], ptr(src_slot), int(topk), ptr(w1), ptr(out), ptr(offsets), ptr(counts), ptr(slot),
        ptr(groups), 0 if groups is None else groups.numel(), E, S, out.shape[0], H, I2 // 2,
        dtype_code(x.dtype), _lib.ACTIVATIONS[activation], stream_of(dev))
    if rc == _lib.RF_ERR_UNSUPPORTED:
        return False
    check(rc, "rf_moe_grouped_gemm_gated_gather")
    return True


def grouped_gemm_down(h: torch.Tensor, w2: torch.Tensor, offsets: torch.Tensor, counts: torch.Tensor,
                      out: torch.Tensor, *, slot: Optional[torch.Tensor] = None,
                      groups: Optional[torch.Tensor] = None, addend: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``out[r] = h[r] . w2[s]^T`` per expert segment; with ``addend`` (out's
    shape and dtype, may be ``out``): ``out[r] = addend[r] + round(h[r] . w2[s]^T)``
    rounded in the layer dtype."""
    dev = _require_cuda(h, w2, offsets, counts, out, slot, groups, addend)
    S, H, I = w2.shape
    E = counts.shape[0]
    ng = 0 if groups is None else groups.numel()
    if addend is None:
        rc = lib().rf_moe_grouped_gemm_down(
            ptr(h), ptr(w2), ptr(out), ptr(offsets), ptr(counts), ptr(slot), ptr(groups),
            ng, E, S, h.shape[0], H, I, dtype_code(h.dtype), stream_of(dev))
        check(rc, "rf_moe_grouped_gemm_down")
        return out
    if addend.shape != out.shape or addend.dtype != out.dtype or not addend.is_contiguous():
        raise _lib.RfMoeError("grouped_gemm_down: addend must be contiguous with out's shape and dtype")
    rc = lib().rf_moe_grouped_gemm_down_add(
        ptr(h), ptr(w2), ptr(out), ptr(addend), ptr(offsets), ptr(counts), ptr(slot), ptr(groups),
        ng, E, S, h.shape[0], H, I, dtype_code(h.dtype), stream_of(dev))
    check(rc, "rf_moe_grouped_gemm_down_add")
    return out


# ----------------------------------------------------------------------- K5
def combine(y: torch.Tensor, row_of_slot: torch.Tensor, weights: torch.Tensor, out: torch.Tensor, *,
            shared_y: Optional[torch.Tensor] = None, shared_scale: Optional[torch.Tensor] = None,
            residual: Optional[torch.Tensor] = None, accumulate: bool = False,
            precise: bool = False, norm: Optional[Tuple[torch.Tensor, Optional[torch.Tensor], float]] = None,
            norm_out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``out[t] = sum_k w[t,k] y[row(t,k)] (+ shared, residual)``.  Default: the
    reference's rounding points and order; ``precise=True``: fp32 accumulation.
    ``norm=(weight, bias or None, eps)``: ``out`` is the new residual and
    ``norm_out`` receives its RMSNorm (reframework/layers/norm.py:43-53)."""
    dev = _require_cuda(y, row_of_slot, weights, out, shared_y, shared_scale, residual, norm_out)
    T, K = weights.shape
    H = out.shape[1]
    weights = weights.contiguous()
    if weights.dtype != torch.float32:
        weights = weights.float()
    mode = _lib.COMBINE_FP32 if precise else _lib.COMBINE_REFERENCE
    if norm is not None:
        if accumulate or norm_out is None:
            raise ValueError("combine with norm needs norm_out and no accumulate")
        nw, nb, eps = norm
        nw = nw.to(device=dev, dtype=torch.float32).contiguous()
        nb = None if nb is None else nb.to(device=dev, dtype=torch.float32).contiguous()
        rc = lib().rf_moe_combine_rmsnorm(ptr(y), ptr(row_of_slot), ptr(weights), T, K, H, dtype_code(out.dtype),
                                          ptr(shared_y), ptr(shared_scale), ptr(residual), mode, ptr(nw), ptr(nb),
                                          float(eps), ptr(out), ptr(norm_out), stream_of(dev))
        check(rc, "rf_moe_combine_rmsnorm")
        return out
    rc = lib().rf_moe_combine(ptr(y), ptr(row_of_slot), ptr(weights), T, K, H, dtype_code(out.dtype),
                              ptr(shared_y), ptr(shared_scale), ptr(residual), int(bool(accumulate)),
                              _lib.COMBINE_FP32 if precise else _lib.COMBINE_REFERENCE, ptr(out), stream_of(dev))
    check(rc, "rf_moe_combine")
    return out


# --------------------------------------------------------- composed forward
_SINGLE_GROUP: Dict[Tuple[torch.device, int], Tuple[torch.Tensor, torch.Tensor]] = {}


def dense_segment(device: torch.device, rows: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """(offsets [2], counts [1]) describing one segment of ``rows`` rows at row 0."""
    key = (device, int(rows))
    seg = _SINGLE_GROUP.get(key)
    if seg is None:
        seg = (torch.tensor([0, rows], dtype=torch.int32, device=device),
               torch.tensor([rows], dtype=torch.int32, device=device))
        if len(_SINGLE_GROUP) > 64:
            _SINGLE_GROUP.clear()
        _SINGLE_GROUP[key] = seg
    return seg


def dense_gated_mlp(x: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor, activation: str = "silu", *,
                    addend: Optional[torch.Tensor] = None) -> torch.Tensor:
    """A dense gated MLP over all rows of ``x`` (a shared expert), on the grouped kernels
    with a single segment.  w1 [2I,H], w2 [H,I].  With ``addend`` [T,H] the result
    is ``addend + MLP(x)`` with both terms rounded to the layer dtype (written
    into ``addend``)."""
    T, H = x.shape
    off, cnt = dense_segment(x.device, T)
    I = w2.shape[1]
    h = torch.empty(T, I, dtype=x.dtype, device=x.device)
    grouped_gemm_gated(x, w1.unsqueeze(0), off, cnt, h, activation=activation)
    y = addend if addend is not None else torch.empty(T, H, dtype=x.dtype, device=x.device)
    grouped_gemm_down(h, w2.unsqueeze(0), off, cnt, y, addend=addend)
    return y


def shared_experts(x: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor, activation: str = "silu") -> torch.Tensor:
    """``sum_s MLP_s(x)`` over the shared experts w1 [S,2I,H], w2 [S,H,I] in the
    reference harness's arithmetic: each expert's output rounded to the layer
    dtype, then added in order in the layer dtype (the second and later
    experts' down GEMMs add onto the running sum in their epilogue)."""
    y = None
    for s in range(w1.shape[0]):
        y = dense_gated_mlp(x, w1[s], w2[s], activation, addend=y)
    return y


def moe_experts(x: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor, weights: torch.Tensor,
                ids32: torch.Tensor, *, activation: str = "silu", shared_y: Optional[torch.Tensor] = None,
                shared_scale: Optional[torch.Tensor] = None, residual: Optional[torch.Tensor] = None,
                out: Optional[torch.Tensor] = None, slot: Optional[torch.Tensor] = None,
                num_experts: Optional[int] = None, precise: bool = False,
                norm: Optional[Tuple[torch.Tensor, Optional[torch.Tensor], float]] = None,
                norm_out: Optional[torch.Tensor] = None,
                before_combine: Optional[torch.cuda.Event] = None) -> torch.Tensor:
    """Permute -> grouped gated GEMM -> grouped down GEMM -> combine (routing given).
    With ``norm`` the combine also writes the RMSNorm of its output to ``norm_out``.
    ``before_combine``: an event (e.g. the shared experts on a side stream)
    the combine waits for; everything before it does not."""
    T, H = x.shape
    E = num_experts if num_experts is not None else w1.shape[0]
    I = w2.shape[2]
    # The explicit gather + gated GEMM is faster on B200 than fetching the
    # token rows inside the GEMM with TMA gather4 (grouped_gemm_gated_gather;
    # measured: C4 routed gated GEMM 0.30 -> 1.41 ms, C2 1.39 -> 1.44 ms).
    p = permute(ids32, E, x=x)
    h = torch.empty(p.rows_cap, I, dtype=x.dtype, device=x.device)
    grouped_gemm_gated(p.x_perm, w1, p.offsets, p.counts, h, slot=slot, activation=activation)
    y = torch.empty(p.rows_cap, H, dtype=x.dtype, device=x.device)
    grouped_gemm_down(h, w2, p.offsets, p.counts, y, slot=slot)
    if out is None:
        out = torch.empty(T, H, dtype=x.dtype, device=x.device)
    if before_combine is not None:
        torch.cuda.current_stream(x.device).wait_event(before_combine)
    return combine(y, p.row_of_slot, weights, out, shared_y=shared_y, shared_scale=shared_scale,
                   residual=residual, precise=precise, norm=norm, norm_out=norm_out)


# ------------------------------------------------------- expert split, int8 half
def int8_quantize(src: torch.Tensor, offsets: torch.Tensor, counts: torch.Tensor, groups: torch.Tensor,
                  q: torch.Tensor, scales: torch.Tensor, amax: torch.Tensor, *, compute_amax: bool = True) -> None:
    """Per listed expert (``groups``), its rows of ``src`` [rows_cap, cols] to
    int8 ``q`` with one symmetric scale (``scales``); ``amax`` [n] fp32 holds
    (or, with ``compute_amax``, receives) each block's max|src|."""
    dev = _require_cuda(src, offsets, counts, groups, q, scales, amax)
    rc = lib().rf_moe_int8_quantize(ptr(src), dtype_code(src.dtype), ptr(offsets), ptr(counts), ptr(groups),
                                    groups.numel(), counts.shape[0], src.shape[0], src.shape[1], ptr(amax),
                                    1 if compute_amax else 0, ptr(scales), ptr(q), stream_of(dev))
    check(rc, "rf_moe_int8_quantize")


def int8_grouped_gemm(a: torch.Tensor, w: torch.Tensor, offsets: torch.Tensor, counts: torch.Tensor,
                      groups: torch.Tensor, slot: torch.Tensor, a_scales: torch.Tensor, w_scales: torch.Tensor,
                      w_scale_stride: int, out: torch.Tensor, *, gated: bool, activation: str = "silu",
                      amax_out: Optional[torch.Tensor] = None, row_weights: Optional[torch.Tensor] = None,
                      src_slot: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Exact int8 grouped GEMM with the split's dequantizing epilogues
    (gated: fp32 ``act(g) * u`` and max|.| per expert; down: fp32 rows times
    the routing weight).  ``w_scales`` points at expert 0's scale, stride
    ``w_scale_stride`` elements."""
    dev = _require_cuda(a, w, offsets, counts, groups, slot, a_scales, w_scales, out, amax_out, row_weights, src_slot)
    if activation not in _lib.ACTIVATIONS:
        raise ValueError(f"unknown gated activation {activation!r}; known: {tuple(_lib.ACTIVATIONS)}")
    rc = lib().rf_moe_int8_grouped_gemm(ptr(a), ptr(w), ptr(offsets), ptr(counts), ptr(groups), ptr(slot),
                                        groups.numel(), counts.shape[0], w.shape[0], a.shape[0], a.shape[1],
                                        out.shape[1], ptr(a_scales), ptr(w_scales), int(w_scale_stride),
                                        1 if gated else 0, _lib.ACTIVATIONS[activation], ptr(out), ptr(amax_out),
                                        ptr(row_weights), ptr(src_slot), stream_of(dev))
    check(rc, "rf_moe_int8_grouped_gemm")
    return out


def split_combine(y_hit: torch.Tensor, y_int8: torch.Tensor, row_of_slot: torch.Tensor, ids32: torch.Tensor,
                  is_miss: torch.Tensor, weights: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """Merge of the split's halves per token (rf_moe_split_combine)."""
    dev = _require_cuda(y_hit, y_int8, row_of_slot, ids32, is_miss, weights, out)
    T, K = weights.shape
    wf = weights.float().contiguous()
    rc = lib().rf_moe_split_combine(ptr(y_hit), ptr(y_int8), ptr(row_of_slot), ptr(ids32), ptr(is_miss), ptr(wf),
                                    T, K, out.shape[1], is_miss.numel(), dtype_code(out.dtype), ptr(out),
                                    stream_of(dev))
    check(rc, "rf_moe_split_combine")
    return out
