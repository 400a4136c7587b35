"""MoE layer on B200 kernels — same public names as reframework.moe
(reframework/moe/__init__.py:8-18)."""

from .fused import fused_experts, torch_fused_topk
from .keys import translate_phimoe_keys
from .moe_layer import CpuShuttle, FusedMoE
from .offload_cache import ExpertOffloadCache, OffloadStats, Prediction

__all__ = [
    "torch_fused_topk",
    "fused_experts",
    "FusedMoE",
    "ExpertOffloadCache",
    "OffloadStats",
]
