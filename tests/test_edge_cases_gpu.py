"""Edge cases of the drop-in layer on the GPU: an empty batch, a single [H]
token, every expert selected (top_k = E), a single expert, and the offloaded
layer with an empty batch — each against the CPU oracle's resident forward
(reframework/moe/moe_layer.py:451-519), with the tolerance of the layer dtype."""

import types

import pytest
import torch

from conftest import max_rel
from oracle import moe_oracle as O
from reframework_b200 import _lib
from reframework_b200.moe import FusedMoE

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


@pytest.fixture(autouse=True)
def _device_clean(cuda_ok):
    yield
    assert _lib.device_status() == 0


def _layer(E, K, H, I, dtype, *, renormalize=True, shared=0, shared_gate=False, seed=0):
    g = torch.Generator().manual_seed(seed)
    moe = FusedMoE(E, K, H, I, renormalize=renormalize, dtype=dtype, router_dtype=torch.float32,
                   num_shared_experts=shared, shared_intermediate_size=I if shared else 0,
                   shared_expert_gate=shared_gate)
    w = {"gate": (torch.randn(E, H, generator=g) * 0.02).to(dtype),
         "w1": (torch.randn(E, 2 * I, H, generator=g) * 0.02).to(dtype),
         "w2": (torch.randn(E, H, I, generator=g) * 0.02).to(dtype)}
    with torch.no_grad():
        moe.gate.copy_(w["gate"])
        for e in range(E):
            moe.experts_w1[e].copy_(w["w1"][e])
            moe.experts_w2[e].copy_(w["w2"][e])
        if shared:
            w["shared_w1"] = (torch.randn(shared, 2 * I, H, generator=g) * 0.02).to(dtype)
            w["shared_w2"] = (torch.randn(shared, H, I, generator=g) * 0.02).to(dtype)
            moe.shared_w1.copy_(w["shared_w1"])
            moe.shared_w2.copy_(w["shared_w2"])
            if shared_gate:
                w["shared_gate"] = (torch.randn(H, generator=g) * 0.02).to(dtype)
                moe.shared_gate.copy_(w["shared_gate"])
    return moe.to(DEV), w


def _oracle(x, w, K, renormalize=True):
    return O.moe_forward(x, w["gate"], w["w1"], w["w2"], top_k=K, renormalize=renormalize, router_fp32=True,
                         shared_w1=w.get("shared_w1"), shared_w2=w.get("shared_w2"),
                         shared_gate=w.get("shared_gate"))


@pytest.mark.parametrize("shared,shared_gate", [(0, False), (1, True), (2, False)])
def test_empty_batch(shared, shared_gate):
    moe, _ = _layer(8, 2, 256, 384, torch.bfloat16, shared=shared, shared_gate=shared_gate)
    x = torch.zeros(0, 256, dtype=torch.bfloat16, device=DEV)
    with torch.no_grad():
        out = moe(x)
        w, ids = moe.route(x)
        norm = types.SimpleNamespace(weight=torch.ones(256, device=DEV), eps=1e-6)
        normed, res = moe.forward_add_residual(x, torch.zeros_like(x), norm)
    torch.cuda.synchronize()
    assert out.shape == (0, 256) and out.dtype == torch.bfloat16
    assert w.shape == (0, 2) and ids.shape == (0, 2)
    assert normed.shape == (0, 256) and res.shape == (0, 256)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_single_token_vector_input(dtype):
    moe, w = _layer(8, 2, 256, 384, dtype, seed=1)
    g = torch.Generator().manual_seed(11)
    x = torch.randn(256, generator=g).to(dtype)
    with torch.no_grad():
        out = moe(x.to(DEV))
    ref = _oracle(x.reshape(1, -1), w, 2)
    assert out.shape == (1, 256)  # the reference's shape for one [H] token
    assert torch.equal(moe.route(x.to(DEV))[1].cpu(), ref["ids"])
    assert max_rel(out.cpu(), ref["out"]) < (1e-4 if dtype == torch.float32 else 1e-2)


@pytest.mark.parametrize("renormalize", [True, False])
def test_every_expert_selected(renormalize):
    E = K = 4
    moe, w = _layer(E, K, 256, 384, torch.bfloat16, renormalize=renormalize, seed=2)
    g = torch.Generator().manual_seed(12)
    x = torch.randn(96, 256, generator=g).bfloat16()
    with torch.no_grad():
        wts, ids = moe.route(x.to(DEV))
        out = moe(x.to(DEV))
    ref = _oracle(x, w, K, renormalize)
    assert torch.equal(ids.cpu(), ref["ids"])
    torch.testing.assert_close(wts.cpu(), ref["weights"], rtol=1e-5, atol=1e-6)
    assert max_rel(out.cpu(), ref["out"]) < 1e-2


def test_single_expert():
    moe, w = _layer(1, 1, 256, 384, torch.bfloat16, shared=1, shared_gate=True, seed=3)
    g = torch.Generator().manual_seed(13)
    x = torch.randn(33, 256, generator=g).bfloat16()
    with torch.no_grad():
        wts, ids = moe.route(x.to(DEV))
        out = moe(x.to(DEV))
    ref = _oracle(x, w, 1)
    assert torch.equal(ids.cpu(), ref["ids"]) and bool((wts.cpu() == 1.0).all())
    assert max_rel(out.cpu(), ref["out"]) < 1e-2


def test_offloaded_layer_empty_then_nonempty_batch():
    moe, w = _layer(8, 2, 256, 384, torch.bfloat16, seed=4)
    moe.build_offload_cache(DEV, 2)
    with torch.no_grad():
        empty = moe(torch.zeros(0, 256, dtype=torch.bfloat16, device=DEV))
        g = torch.Generator().manual_seed(14)
        x = torch.randn(40, 256, generator=g).bfloat16()
        out = moe(x.to(DEV))
    assert empty.shape == (0, 256)
    ref = _oracle(x, w, 2)
    assert max_rel(out.cpu(), ref["out"]) < 1e-2
