"""rf_moe_permute_noalloc — the permute for callers that cannot allocate device
memory (hosts that plan all device buffers up front, or plugins that are only
handed their inputs and outputs).  Its scratch is a fixed device array inside
the library instead of a caller workspace.

Called through the C ABI and checked against rf_moe_permute on the same
inputs, twice in a row (the shared array keeps the previous call's contents).
This file is collected last so that, in a run that stops at the first failure,
every other test has already run; it also passes on its own in a fresh process
(the first call performs the per-device set-up)."""

import pytest
import torch

from reframework_b200 import _lib
from reframework_b200._lib import dtype_code, lib, ptr, stream_of

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _outputs(T, K, E, align, H, dtype):
    cap = int(lib().rf_moe_rows_capacity(T * K, E, align))
    return {
        "offsets": torch.full((E + 1,), -7, dtype=torch.int32, device=DEV),
        "counts": torch.full((E,), -7, dtype=torch.int32, device=DEV),
        "row_of_slot": torch.full((max(T * K, 1),), -7, dtype=torch.int32, device=DEV),
        "src_slot": torch.full((max(cap, 1),), -7, dtype=torch.int32, device=DEV),
        "x_perm": torch.full((max(cap, 1), H), 3.0, dtype=dtype, device=DEV),
    }


def _run_workspace(ids, E, align, x):
    T, K = ids.shape
    o = _outputs(T, K, E, align, x.shape[1], x.dtype)
    wsb = int(lib().rf_moe_permute_workspace_size(T * K, E))
    ws = torch.empty(wsb, dtype=torch.uint8, device=DEV)
    rc = lib().rf_moe_permute(ptr(ids), T, K, E, align, ptr(x), dtype_code(x.dtype), x.shape[1],
                              ptr(o["offsets"]), ptr(o["counts"]), ptr(o["row_of_slot"]), ptr(o["src_slot"]),
                              ptr(o["x_perm"]), ptr(ws), wsb, stream_of(DEV))
    _lib.check(rc, "rf_moe_permute")
    return o


def _run_noalloc(ids, E, align, x):
    T, K = ids.shape
    o = _outputs(T, K, E, align, x.shape[1], x.dtype)
    rc = lib().rf_moe_permute_noalloc(ptr(ids), T, K, E, align, ptr(x), dtype_code(x.dtype), x.shape[1],
                                      ptr(o["offsets"]), ptr(o["counts"]), ptr(o["row_of_slot"]),
                                      ptr(o["src_slot"]), ptr(o["x_perm"]), stream_of(DEV))
    _lib.check(rc, "rf_moe_permute_noalloc")
    return o


def _compare(a, b):
    used = int(a["offsets"][-1])
    assert torch.equal(a["offsets"], b["offsets"])
    assert torch.equal(a["counts"], b["counts"])
    assert torch.equal(a["row_of_slot"], b["row_of_slot"])
    assert torch.equal(a["src_slot"][:used], b["src_slot"][:used])
    assert torch.equal(a["x_perm"][:used], b["x_perm"][:used])  # the tolerance for a copy: exact


@pytest.mark.parametrize("T,K,E,align,H,dtype", [
    (4096, 2, 8, 128, 512, torch.bfloat16),     # two calls with different routings in a row
    (3000, 6, 64, 128, 256, torch.float16),
    (37, 3, 5, 1, 64, torch.float32),
])
def test_noalloc_permute_matches_workspace_permute(T, K, E, align, H, dtype):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    g = torch.Generator().manual_seed(T + E)
    x = torch.randn(T, H, generator=g).to(dtype).to(DEV)
    for call in range(2):
        ids = torch.randint(0, E, (T, K), generator=g, dtype=torch.int32)
        if call == 1:
            ids[: T // 2] = E - 1  # a different, skewed routing on the second call
        ids = ids.to(DEV)
        ref = _run_workspace(ids, E, align, x)
        got = _run_noalloc(ids, E, align, x)
        torch.cuda.synchronize()
        _compare(got, ref)
    assert _lib.device_status() == 0


def test_noalloc_permute_rejects_sizes_beyond_its_scratch():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    E = 1024
    T, K = 70 * 1024, 1  # ceil(T*K/1024) * E = 70 * 1024 > 65536 words
    ids = torch.zeros(T, K, dtype=torch.int32, device=DEV)
    x = torch.zeros(T, 64, dtype=torch.bfloat16, device=DEV)
    o = _outputs(T, K, E, 1, 64, torch.bfloat16)
    rc = lib().rf_moe_permute_noalloc(ptr(ids), T, K, E, 1, ptr(x), dtype_code(x.dtype), 64,
                                      ptr(o["offsets"]), ptr(o["counts"]), ptr(o["row_of_slot"]),
                                      ptr(o["src_slot"]), ptr(o["x_perm"]), stream_of(DEV))
    assert rc == 1
    assert "exceeds the fixed scratch" in lib().rf_moe_last_error().decode()
