"""Process-group context, collectives and expert parallelism — same names as
reframework.parallel (reframework/parallel/__init__.py:8-44), minus pipeline
parallelism (not part of the MoE-layer path)."""

from .dist import (ParallelContext, all_gather, all_reduce_sum, all_to_all, all_to_all_v, barrier, current,
                   destroy, get_rank, get_world_size, init, is_initialized, recv, run, send)
from .ep import EPFusedMoE, ep_enabled, plan_dispatch, shard_range

__all__ = [
    "ParallelContext", "init", "run", "is_initialized", "current", "get_rank", "get_world_size",
    "all_reduce_sum", "all_gather", "all_to_all", "all_to_all_v", "send", "recv", "barrier", "destroy",
    "EPFusedMoE", "ep_enabled", "shard_range", "plan_dispatch",
]
