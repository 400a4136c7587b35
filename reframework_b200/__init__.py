"""reframework_b200 — B200 (sm_100a) MoE-layer forward, drop-in for Reframework's
torch MoE layer (``reframework.moe``) and its expert-parallel layer
(``reframework.parallel``).

Subpackages mirror the reference's import paths:
  ``reframework_b200.moe``       FusedMoE, ExpertOffloadCache, OffloadStats,
                                 torch_fused_topk, fused_experts
  ``reframework_b200.parallel``  process-group context, collectives, EPFusedMoE
The compute runs in ``_rf_moe.so`` (C ABI in include/rf_moe.h).
"""

__version__ = "0.1.0"
