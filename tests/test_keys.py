"""Checkpoint key handling (CPU): HF names, PhiMoE / Mixtral names
(reference reframework/checkpoint/loader.py:83-103) and the state-dict round
trip of the bank-backed parameters."""

import torch

from reframework_b200.moe import FusedMoE, translate_phimoe_keys


def _layer(seed=0):
    torch.manual_seed(seed)
    m = FusedMoE(4, 2, 32, 48, dtype=torch.bfloat16)
    with torch.no_grad():
        m.gate.normal_()
        for e in range(4):
            m.experts_w1[e].normal_()
            m.experts_w2[e].normal_()
    return m


def test_translate_phimoe_keys_mapping():
    t = torch.zeros(1)
    sd = {
        "model.layers.3.block_sparse_moe.gate.weight": t,
        "model.layers.3.block_sparse_moe.experts.7.w1.weight": t,
        "model.layers.3.block_sparse_moe.experts.7.w3.weight": t,
        "model.layers.3.block_sparse_moe.experts.7.w2.weight": t,
        "model.layers.3.input_layernorm.bias": t,
        "model.layers.3.self_attn.w1.weight": t,  # not under experts: unchanged
    }
    out = translate_phimoe_keys(sd)
    assert set(out) == {
        "model.layers.3.mlp.gate.weight",
        "model.layers.3.mlp.experts.7.gate_proj.weight",
        "model.layers.3.mlp.experts.7.up_proj.weight",
        "model.layers.3.mlp.experts.7.down_proj.weight",
        "model.layers.3.input_layernorm.bias",
        "model.layers.3.self_attn.w1.weight",
    }


def test_load_state_dict_accepts_phimoe_names():
    src = _layer(1)
    hf = {k: v.detach().clone() for k, v in src.state_dict(prefix="model.layers.0.mlp").items()}
    phi = {}
    for k, v in hf.items():
        k = k.replace(".mlp.", ".block_sparse_moe.")
        k = k.replace(".gate_proj.", ".w1.").replace(".up_proj.", ".w3.").replace(".down_proj.", ".w2.")
        phi[k] = v
    a, b, c = _layer(2), _layer(3), _layer(4)
    a.load_state_dict(hf, prefix="model.layers.0.mlp")
    b.load_state_dict(phi, prefix="model.layers.0.block_sparse_moe")
    c.load_state_dict(translate_phimoe_keys(phi), prefix="model.layers.0.mlp")
    for m in (a, b, c):
        for k, v in m.state_dict().items():
            assert torch.equal(v, src.state_dict()[k]), k


def test_state_dict_views_share_the_bank():
    m = _layer(5)
    sd = m.state_dict()
    I = m.intermediate_size
    assert sd["experts.2.gate_proj.weight"].shape == (I, m.hidden_size)
    with torch.no_grad():
        sd["experts.2.up_proj.weight"].fill_(3.0)
    assert torch.all(m.experts_w1[2][I:] == 3.0)
