"""RE_* environment flags read by the MoE path (same names and defaults as
reframework/env.py:68-153 plus the flags the reference MoE code reads
directly: RE_ENTROPY_K(_MIN) moe_layer.py:214-219, RE_CHUNK_SIZE
moe_layer.py:362,465, RE_MAX_PACK moe_layer.py:430)."""

from __future__ import annotations

import os


def _get(name: str, default: str) -> str:
    return os.environ.get(name, default).strip()


def _get_bool(name: str, default: bool = False) -> bool:
    raw = os.environ.get(name)
    if raw is None:
        return default
    return raw.strip().lower() in {"1", "true", "yes", "on", "y"}


def _get_int(name: str, default: int) -> int:
    raw = os.environ.get(name)
    if raw is None:
        return default
    try:
        return int(raw)
    except ValueError:
        return default


def _get_float(name: str, default: float) -> float:
    raw = os.environ.get(name)
    if raw is None:
        return default
    try:
        return float(raw)
    except ValueError:
        return default


def get_moe_offload_enabled() -> bool:
    return _get_bool("RE_MOE_OFFLOAD", True)


def get_moe_cache_size() -> int:
    """GPU expert slots per layer; 0 = sized by the caller."""
    return _get_int("RE_MOE_CACHE_SIZE", 0)


def get_moe_cache_ratio() -> float:
    return _get_float("RE_MOE_CACHE_RATIO", 0.5)


def get_moe_substitute() -> bool:
    return _get_bool("RE_MOE_SUBSTITUTE", True)


def get_moe_predict() -> bool:
    return _get_bool("RE_MOE_PREDICT", True)


def get_moe_predict_window() -> int:
    return _get_int("RE_MOE_PREDICT_WINDOW", 32)


def get_moe_predict_headroom() -> float:
    return _get_float("RE_MOE_PREDICT_HEADROOM", 0.9)


def get_moe_prefill_overlap() -> bool:
    return _get_bool("RE_MOE_PREFILL_OVERLAP", True)


def get_moe_cache_policy() -> str:
    """``lru`` (default) or ``least_stale``; unknown values fall back to ``lru``."""
    p = _get("RE_CACHE_POLICY", "lru").lower()
    return p if p in {"lru", "least_stale"} else "lru"


def get_moe_cpu_split() -> bool:
    return _get_bool("RE_MOE_CPU_SPLIT", False)


def get_moe_shuttle_steps() -> int:
    return _get_int("RE_MOE_SHUTTLE_STEPS", 0)


def get_entropy_k() -> bool:
    return _get("RE_ENTROPY_K", "").lower() in {"1", "true", "yes", "on"}


def get_entropy_k_min(default: int = 2) -> int:
    return _get_int("RE_ENTROPY_K_MIN", default)


def get_chunk_size(default: int = 0) -> int:
    return _get_int("RE_CHUNK_SIZE", default)


def get_max_pack():
    raw = os.environ.get("RE_MAX_PACK")
    return None if raw is None else _get_int("RE_MAX_PACK", 2)
