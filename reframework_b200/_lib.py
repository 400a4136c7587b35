"""ctypes binding of the rf_moe C ABI (include/rf_moe.h).

Loads ``reframework_b200/_rf_moe.so`` (built in-tree by
``python -m reframework_b200.csrc.build``).  There is no fallback: if the
library is missing or a call fails, an :class:`RfMoeError` is raised with the
library's message.
"""

from __future__ import annotations

import ctypes
import os
import threading
from typing import Optional

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_rf_moe.so")

RF_F32, RF_F16, RF_BF16 = 0, 1, 2
ACTIVATIONS = {"silu": 0, "gelu": 1, "gelu_tanh": 2}
COMBINE_REFERENCE, COMBINE_FP32 = 0, 1
DEV_ERRORS = {0: "ok", 1: "routed expert id out of range", 2: "pipeline wait timed out",
              3: "expert-parallel plan exceeds its buffers"}

_c_void_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int

# name -> (restype, argtypes) — mirrors include/rf_moe.h
_SIGNATURES = {
    "rf_moe_last_error": (ctypes.c_char_p, []),
    "rf_moe_version": (_int, []),
    "rf_moe_device_status": (_int, [ctypes.POINTER(_int)]),
    "rf_moe_rows_capacity": (_i64, [_i64, _i64, _i64]),
    "rf_moe_permute_workspace_size": (ctypes.c_size_t, [_i64, _i64]),
    "rf_moe_router_topk": (_int, [_c_void_p, _int, _c_void_p, _int, _c_void_p, _i64, _i64, _i64, _i64,
                                  _int, _int, _int, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
                                  _c_void_p, _c_void_p, _c_void_p, ctypes.c_size_t, _c_void_p]),
    "rf_moe_router_workspace_size": (ctypes.c_size_t, [_i64, _i64, _i64, _int]),
    "rf_moe_permute": (_int, [_c_void_p, _i64, _i64, _i64, _i64, _c_void_p, _int, _i64, _c_void_p,
                              _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, ctypes.c_size_t,
                              _c_void_p]),
    "rf_moe_permute_noalloc": (_int, [_c_void_p, _i64, _i64, _i64, _i64, _c_void_p, _int, _i64, _c_void_p,
                                      _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p]),
    "rf_moe_gather_rows": (_int, [_c_void_p, _c_void_p, _i64, _i64, _c_void_p, _i64, _c_void_p,
                                  _c_void_p]),
    "rf_moe_set_gemm_impl": (_int, [_int]),
    "rf_moe_grouped_gemm_gated": (_int, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
                                         _c_void_p, _c_void_p, _i64, _i64, _i64, _i64, _i64, _i64,
                                         _int, _int, _c_void_p]),
    "rf_moe_grouped_gemm_gated_gather": (_int, [_c_void_p, _i64, _c_void_p, _i64, _c_void_p, _c_void_p, _c_void_p,
                                                _c_void_p, _c_void_p, _c_void_p, _i64, _i64, _i64, _i64, _i64,
                                                _i64, _int, _int, _c_void_p]),
    "rf_moe_grouped_gemm_down": (_int, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
                                        _c_void_p, _c_void_p, _i64, _i64, _i64, _i64, _i64, _i64,
                                        _int, _c_void_p]),
    "rf_moe_grouped_gemm_down_add": (_int, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
                                            _c_void_p, _c_void_p, _i64, _i64, _i64, _i64, _i64, _i64,
                                            _int, _c_void_p]),
    "rf_moe_combine": (_int, [_c_void_p, _c_void_p, _c_void_p, _i64, _i64, _i64, _int, _c_void_p,
                              _c_void_p, _c_void_p, _int, _int, _c_void_p, _c_void_p]),
    "rf_moe_combine_rmsnorm": (_int, [_c_void_p, _c_void_p, _c_void_p, _i64, _i64, _i64, _int, _c_void_p,
                                      _c_void_p, _c_void_p, _int, _c_void_p, _c_void_p, ctypes.c_float,
                                      _c_void_p, _c_void_p, _c_void_p]),
    "rf_moe_ep_pair_rows": (_int, [_c_void_p, ctypes.c_int32, ctypes.c_int32, _c_void_p, _c_void_p,
                                   ctypes.c_int32, _c_void_p]),
    "rf_moe_peer_alloc": (_int, [ctypes.c_size_t, ctypes.POINTER(_c_void_p), _c_void_p]),
    "rf_moe_peer_open": (_int, [_c_void_p, ctypes.POINTER(_c_void_p)]),
    "rf_moe_peer_close": (_int, [_c_void_p]),
    "rf_moe_peer_free": (_int, [_c_void_p]),
    "rf_moe_ep_push_rows": (_int, [_c_void_p, _i64, _c_void_p, _c_void_p, _i64, ctypes.c_int32, ctypes.c_int32,
                                   _c_void_p, _c_void_p, _c_void_p, _c_void_p, ctypes.c_int32, _c_void_p,
                                   _c_void_p]),
    "rf_moe_ep_wait": (_int, [_c_void_p, ctypes.c_int32, ctypes.c_int32, _c_void_p]),
    "rf_moe_ep_counts_push": (_int, [_c_void_p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, _c_void_p,
                                     _c_void_p, ctypes.c_int32, _c_void_p]),
    "rf_moe_ep_counts_collect": (_int, [_c_void_p, _c_void_p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                        _c_void_p, _c_void_p]),
    "rf_moe_ep_devplan_workspace_size": (ctypes.c_size_t, [ctypes.c_int32] * 4),
    "rf_moe_ep_devplan_layout": (_int, [ctypes.c_int32] * 4 + [_c_void_p]),
    "rf_moe_ep_devplan": (_int, [_c_void_p, _c_void_p, _c_void_p] + [ctypes.c_int32] * 7 + [_i64, _i64, _i64, _c_void_p,
                                                                                           ctypes.c_size_t, _c_void_p]),
    "rf_moe_ep_devplan_host": (_int, [_c_void_p, _c_void_p, _c_void_p] + [ctypes.c_int32] * 7 + [_i64, _i64, _i64,
                                                                                                _c_void_p,
                                                                                                ctypes.c_size_t,
                                                                                                _c_void_p]),
    "rf_moe_ep_devplan_push": (_int, [_c_void_p] + [ctypes.c_int32] * 5 + [_c_void_p, _c_void_p, _i64, _i64,
                                                                            _c_void_p, _c_void_p, ctypes.c_int32,
                                                                            _c_void_p, _c_void_p]),
    "rf_moe_ep_devplan_regroup": (_int, [_c_void_p] + [ctypes.c_int32] * 4 + [_c_void_p, _c_void_p, _i64, _c_void_p]),
    "rf_moe_ep_devplan_regroup_remote": (_int, [_c_void_p] + [ctypes.c_int32] * 4 + [_c_void_p, _c_void_p, _i64, _c_void_p]),
    "rf_moe_ep_devplan_down_return": (_int, [_c_void_p] + [ctypes.c_int32] * 4 + [_c_void_p, _c_void_p, _i64, _i64,
                                                                               _i64, ctypes.c_int32, _c_void_p,
                                                                               _c_void_p, ctypes.c_int32, _c_void_p,
                                                                               _c_void_p]),
    "rf_moe_int8_quantize": (_int, [_c_void_p, ctypes.c_int32, _c_void_p, _c_void_p, _c_void_p, ctypes.c_int32,
                                     ctypes.c_int32, _i64, _i64, _c_void_p, ctypes.c_int32, _c_void_p, _c_void_p,
                                     _c_void_p]),
    "rf_moe_int8_grouped_gemm": (_int, [_c_void_p] * 6 + [ctypes.c_int32] * 3 + [_i64, _i64, _i64, _c_void_p,
                                                                                 _c_void_p, _i64, ctypes.c_int32,
                                                                                 ctypes.c_int32] + [_c_void_p] * 5),
    "rf_moe_split_combine": (_int, [_c_void_p] * 6 + [_i64, ctypes.c_int32, _i64, ctypes.c_int32, ctypes.c_int32,
                                                       _c_void_p, _c_void_p]),
    "rf_moe_ep_plan": (_int, [_c_void_p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, _c_void_p, _c_void_p,
                              ctypes.c_int32, ctypes.c_int32, _c_void_p, _c_void_p, _c_void_p, _i64, _c_void_p]),
}


class RfMoeError(RuntimeError):
    """A call into the rf_moe CUDA library failed."""


_lib: Optional[ctypes.CDLL] = None
_lock = threading.Lock()


def lib() -> ctypes.CDLL:
    """The loaded library (raises RfMoeError if it has not been built)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise RfMoeError(
                        f"rf_moe CUDA library not found at {LIB_PATH}; build it with "
                        "`python -m reframework_b200.csrc.build` (needs nvcc)")
                h = ctypes.CDLL(LIB_PATH)
                for name, (res, args) in _SIGNATURES.items():
                    fn = getattr(h, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = h
    return _lib


def exported_symbols():
    return list(_SIGNATURES)


def check(rc: int, what: str) -> None:
    if rc != 0:
        msg = lib().rf_moe_last_error().decode(errors="replace")
        raise RfMoeError(f"{what} failed (status {rc}): {msg}")


def dtype_code(dt: torch.dtype) -> int:
    if dt == torch.float32:
        return RF_F32
    if dt == torch.float16:
        return RF_F16
    if dt == torch.bfloat16:
        return RF_BF16
    raise RfMoeError(f"unsupported dtype {dt}")


def ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def stream_of(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def device_status() -> int:
    """Read and clear the device error word (synchronises the device)."""
    code = ctypes.c_int(0)
    check(lib().rf_moe_device_status(ctypes.byref(code)), "rf_moe_device_status")
    return code.value


_gemm_impl = 0
RF_ERR_UNSUPPORTED = 2
EP_DEVPLAN_LAYOUT_N = 21  # entries of rf_moe_ep_devplan_layout's output (RF_EP_DEVPLAN_LAYOUT_N)


def set_gemm_impl(impl: int) -> None:
    global _gemm_impl
    check(lib().rf_moe_set_gemm_impl(int(impl)), "rf_moe_set_gemm_impl")
    _gemm_impl = int(impl)


def gemm_impl() -> int:
    """The grouped-GEMM implementation selected by set_gemm_impl (0 = automatic)."""
    return _gemm_impl
