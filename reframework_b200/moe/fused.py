"""Functional MoE API: routing and routed-expert compute on the B200 kernels.

Drop-in for reframework/moe/fused.py:
  * ``torch_fused_topk``  (fused.py:32-46)  softmax -> top-k -> renormalise
  * ``fused_experts``     (fused.py:49-87)  routed experts, summed into [M, H]
Both run the CUDA kernels of ``reframework_b200._rf_moe.so`` and need CUDA
tensors; there is no CPU path.

Numerics: expert GEMMs accumulate in fp32 and round the gated activation to
the weight dtype once; the combine sums the K weighted expert rows in fp32 and
rounds once to the output dtype (the reference rounds after every op and
accumulates with a low-precision ``index_add_``).
"""

from __future__ import annotations

from typing import Tuple

import torch

from .. import kernels as K
from .._lib import RfMoeError

__all__ = ["torch_fused_topk", "fused_experts"]


def torch_fused_topk(gating_output: torch.Tensor, topk: int, renormalize: bool) -> Tuple[torch.Tensor, torch.Tensor]:
    """Softmax over all experts (fp32), keep the top-k (ties to the lower id),
    renormalise the kept weights.  Returns (weights fp32 [M,K], ids int64 [M,K])."""
    g = gating_output
    if g.dim() != 2:
        g = g.reshape(-1, g.shape[-1])
    w, _, ids, _, _ = K.router_topk(g.contiguous(), None, int(topk), renormalize=renormalize,
                                    ids64=True, ids32=False)
    return w, ids


def fused_experts(hidden_states: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor,
                  topk_weights: torch.Tensor, topk_ids: torch.Tensor,
                  activation: str = "silu") -> torch.Tensor:
    """Run the routed experts and return the summed output ``[M, H]``.

    ``w1`` [E, 2I, H] rows ``[gate | up]``; ``w2`` [E, H, I]; ``topk_weights``
    [M, K] (any float dtype, used in fp32); ``topk_ids`` [M, K] (int32/int64).
    The output has the dtype of ``hidden_states``; the GEMMs run in the weight
    dtype (the activations are cast, as ``x.to(w1.dtype)`` in the reference).
    """
    if hidden_states.dim() != 2:
        raise RfMoeError("fused_experts: hidden_states must be [M, H]")
    x = hidden_states
    xc = x if x.dtype == w1.dtype else x.to(w1.dtype)
    ids32 = topk_ids.to(torch.int32)
    w = topk_weights.float()
    out = K.moe_experts(xc.contiguous(), w1.contiguous(), w2.contiguous(), w, ids32, activation=activation)
    return out if out.dtype == x.dtype else out.to(x.dtype)
