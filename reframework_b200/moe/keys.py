"""Checkpoint key names for the MoE layer.

The layer's own names are the HF ones of reframework/moe/moe_layer.py:631-660:
``gate.weight`` and ``experts.{e}.{gate_proj,up_proj,down_proj}.weight``.
PhiMoE / Mixtral checkpoints name the same tensors
``block_sparse_moe.experts.{e}.{w1,w3,w2}.weight`` (w1 = gate, w3 = up,
w2 = down); ``translate_phimoe_keys`` is the mapping of
reframework/checkpoint/loader.py:83-103, and ``expert_tensor`` lets
``load_state_dict`` accept either spelling directly.
"""

from __future__ import annotations

from typing import Dict, Optional

import torch

__all__ = ["translate_phimoe_keys", "expert_tensor", "PHIMOE_TAGS"]

# HF projection name -> PhiMoE / Mixtral name
PHIMOE_TAGS = {"gate_proj": "w1", "up_proj": "w3", "down_proj": "w2"}


def translate_phimoe_keys(state_dict: Dict[str, torch.Tensor]) -> Dict[str, torch.Tensor]:
    """``block_sparse_moe`` -> ``mlp`` and, under ``experts.``, ``w1/w3/w2`` ->
    ``gate_proj/up_proj/down_proj``; every other key passes through unchanged
    (reframework/checkpoint/loader.py:83-103)."""
    out = {}
    for k, v in state_dict.items():
        k2 = k.replace(".block_sparse_moe.", ".mlp.")
        if ".experts." in k2:
            for hf, phi in PHIMOE_TAGS.items():
                tail = f".{phi}.weight"
                if k2.endswith(tail):
                    k2 = k2[: -len(tail)] + f".{hf}.weight"
                    break
        out[k2] = v
    return out


def expert_tensor(state_dict: Dict[str, torch.Tensor], expert_prefix: str, proj: str) -> Optional[torch.Tensor]:
    """The ``proj`` weight (HF name) of the expert at ``expert_prefix``
    (e.g. ``model.layers.0.mlp.experts.3``), under its HF or its PhiMoE name;
    None when the state dict holds neither."""
    t = state_dict.get(f"{expert_prefix}.{proj}.weight")
    if t is None:
        t = state_dict.get(f"{expert_prefix}.{PHIMOE_TAGS[proj]}.weight")
    return t
