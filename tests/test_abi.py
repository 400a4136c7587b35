"""The C-ABI library builds, loads and exports every symbol the header
declares; argument validation fails cleanly without touching a GPU."""

import ctypes
import os
import re

import pytest

from conftest import ROOT
from reframework_b200 import _lib

HEADER = os.path.join(ROOT, "include", "rf_moe.h")


def header_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(rf_moe_[a-z0-9_]+)\s*\(", src)))


def header_arity():
    """{function: number of parameters} from the prototypes in rf_moe.h."""
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    out = {}
    for name, params in re.findall(r"\b(rf_moe_[a-z0-9_]+)\s*\(([^)]*)\)\s*;", src):
        params = params.strip()
        out[name] = 0 if params in ("", "void") else params.count(",") + 1
    return out


def test_ctypes_bindings_match_header_arity():
    """Every binding passes exactly as many arguments as the C prototype takes."""
    arity = header_arity()
    assert arity, "no prototypes parsed"
    for name, (_, argtypes) in _lib._SIGNATURES.items():
        assert len(argtypes) == arity[name], f"{name}: ctypes {len(argtypes)} args, header {arity[name]}"


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    names = header_functions()
    assert len(names) >= 11
    for n in names:
        assert hasattr(lib, n), f"{n} declared in rf_moe.h but not exported"
    assert set(names) == set(_lib.exported_symbols()), "ctypes bindings out of sync with the header"


def test_version_and_sizes():
    lib = _lib.lib()
    assert lib.rf_moe_version() == 100
    assert lib.rf_moe_rows_capacity(8192, 8, 128) == 8192 + 8 * 127
    assert lib.rf_moe_rows_capacity(8192, 8, 1) == 8192
    assert lib.rf_moe_permute_workspace_size(8192, 8) >= 2 * 8 * 4
    # router partials: ceil(H/256) slices x T x (E + shared gate) fp32
    assert lib.rf_moe_router_workspace_size(4096, 4096, 8, 0) >= 16 * 4096 * 8 * 4
    assert lib.rf_moe_router_workspace_size(64, 2048, 60, 1) >= 8 * 64 * 61 * 4


def test_header_constants_match_bindings():
    src = open(HEADER).read()
    assert int(re.search(r"#define RF_EP_DEVPLAN_LAYOUT_N (\d+)", src).group(1)) == _lib.EP_DEVPLAN_LAYOUT_N
    codes = {int(v): k for k, v in re.findall(r"#define (RF_DEV_[A-Z_]+) (\d+)", src)}
    assert set(codes) == set(_lib.DEV_ERRORS), "every device error code has a message"


def test_fused_gather_gemm_reports_unsupported_dtype():
    """fp32 has no tensor-core path: the fused-gather GEMM declines (status 2)
    without touching a GPU, and the caller gathers explicitly."""
    lib = _lib.lib()
    rc = lib.rf_moe_grouped_gemm_gated_gather(1 << 20, 4, 1 << 20, 2, 1 << 20, 1 << 20, 1 << 20, 1 << 20, None,
                                              None, 0, 4, 4, 64, 64, 64, 0, 0, None)
    assert rc == 2 and "tensor-core" in lib.rf_moe_last_error().decode()


@pytest.mark.parametrize("call, needle", [
    (lambda L: L.rf_moe_router_topk(None, 2, None, 2, None, 4, 64, 8, 9, 1, -1, 0, None, None,
                                    None, None, None, None, None, 0, None), "K <="),
    (lambda L: L.rf_moe_router_topk(None, 7, None, 2, None, 4, 64, 8, 2, 1, -1, 0, None, None,
                                    None, None, None, None, None, 0, None), "dtype"),
    (lambda L: L.rf_moe_permute(None, 4, 2, 8, 3, None, 2, 64, None, None, None, None, None, None, 0,
                                None), "align"),
    (lambda L: L.rf_moe_combine(None, None, None, 4, 2, 60, 2, None, None, None, 0, 0, None, None),
     "multiple of 16"),
    (lambda L: L.rf_moe_combine(None, None, None, 4, 2, 64, 2, None, None, None, 0, 7, None, None),
     "unknown mode"),
    (lambda L: L.rf_moe_grouped_gemm_gated(None, None, None, None, None, None, None, 0, 8, 8, 64, 64,
                                           64, 2, 9, None), "activation"),
    (lambda L: L.rf_moe_set_gemm_impl(6), "0 to 5"),
    (lambda L: L.rf_moe_combine_rmsnorm(None, None, None, 4, 2, 64, 2, None, None, None, 0, None, None, -1.0,
                                        None, None, None), "eps"),
    (lambda L: L.rf_moe_int8_quantize(None, 9, None, None, None, 1, 4, 8, 64, None, 1, None, None, None), "dtype"),
    (lambda L: L.rf_moe_int8_grouped_gemm(None, None, None, None, None, None, 1, 4, 4, 128, 8, 64, None, None, 1,
                                          1, 0, None, None, None, None, None), "multiple of 16"),
    (lambda L: L.rf_moe_int8_grouped_gemm(None, None, None, None, None, None, 1, 4, 4, 128, 64, 64, None, None, 1,
                                          1, 7, None, None, None, None, None), "activation"),
    (lambda L: L.rf_moe_split_combine(None, None, None, None, None, None, 4, 17, 64, 8, 2, None, None), "K <= 16"),
])
def test_argument_validation(call, needle):
    lib = _lib.lib()
    rc = call(lib)
    assert rc == 1  # RF_ERR_ARG
    assert needle in lib.rf_moe_last_error().decode()


def test_errors_raise_in_python():
    with pytest.raises(_lib.RfMoeError):
        _lib.set_gemm_impl(7)


def test_no_multicast_or_batched_copy_in_sources():
    """No cluster-multicast bulk loads and no batched async memcpy anywhere in
    the CUDA sources (the patterns are assembled so this file names neither)."""
    csrc = os.path.join(ROOT, "reframework_b200", "csrc")
    bad = re.compile("|".join(["multi" + "cast::" + "cluster", "Memcpy" + "Batch", "Memcpy3D" + "Batch"]))
    for f in os.listdir(csrc):
        if f.endswith((".cu", ".cuh", ".h")):
            text = open(os.path.join(csrc, f)).read()
            assert not bad.search(text), f


def test_empty_batch_needs_no_row_buffers():
    """An empty batch (T == 0): the router, the grouped GEMMs (no rows) and the
    combine accept empty, null row buffers and return at once without a GPU
    call, as torch does for zero-row tensors in the reference layer."""
    lib = _lib.lib()
    dummy = ctypes.create_string_buffer(64)
    p = ctypes.cast(dummy, ctypes.c_void_p)
    bf16 = _lib.RF_BF16
    # router: x, weights and ids all null for T == 0 (with a shared gate, no shared_scale)
    assert lib.rf_moe_router_topk(None, bf16, p, bf16, None, 0, 64, 8, 2, 1, -1, 0, p, None,
                                  None, None, None, None, None, 0, None) == 0
    # grouped GEMMs over zero rows: no activation / output buffers
    assert lib.rf_moe_grouped_gemm_gated(None, p, None, p, p, None, None, 0, 8, 8, 0, 64, 32, bf16, 0, None) == 0
    assert lib.rf_moe_grouped_gemm_down_add(None, p, None, None, p, p, None, None, 0, 8, 8, 0, 64, 32,
                                            bf16, None) == 0
    # combine of zero tokens
    assert lib.rf_moe_combine(None, None, None, 0, 2, 64, bf16, None, None, None, 0, 0, None, None) == 0
    # combine + RMSNorm of zero tokens: both (empty) outputs may be null
    assert lib.rf_moe_combine_rmsnorm(None, None, None, 0, 2, 64, bf16, None, None, None, 0, p, None, 1e-6,
                                      None, None, None) == 0
