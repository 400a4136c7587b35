"""Seeded synthetic MoE-layer workloads (the five benchmark configurations).

There are no checkpoints or datasets on the target machines, so every weight,
activation and router bias is drawn from a seeded generator with the shapes and
value distributions of the benchmark configurations:

  C1  tiny, fp32        H=1024  E=8  K=2 I=2816  T=64    no bias
  C2  Mixtral-8x7B bf16 H=4096  E=8  K=2 I=14336 T=4096  bias ~ N(0,1)
  C3  Qwen1.5-MoE bf16  H=2048  E=60 K=4 I=1408  T=64    Zipf(1.1) bias,
                        shared SwiGLU FFN 5632 gated by sigmoid(x.w_s)
  C4  DeepSeek-V2-Lite  H=2048  E=64 K=6 I=1408  T=8192  2 shared FFNs of 1408
  C5  Mixtral-8x22B     H=6144  E=8  K=2 I=16384 T=2048 x 16 steps,
                        per-step bias log(Dirichlet(0.3) + 1e-9)

Weights ~ N(0, 0.02), activations ~ N(0, 1); everything is drawn on the CPU in
fp32 (``torch.Generator().manual_seed(seed)``) and then cast, so the same seed
gives the same tensors on every host.  ``generate(..., device="cuda")`` draws
directly on the device instead (used by the benchmark for the multi-GB
configurations, where CPU generation would dominate start-up; such tensors are
*not* comparable with the CPU draw and are never used for parity).

The draw order is fixed: router gate [E,H], w1 [E,2I,H], w2 [E,H,I], shared
expert weights, x [T,H], then the bias.  Changing it changes every fixture.
"""

from __future__ import annotations

from dataclasses import dataclass, replace
from typing import Dict, Optional

import numpy as np
import torch

__all__ = ["MoEConfig", "CONFIGS", "generate", "router_bias", "mini"]


@dataclass(frozen=True)
class MoEConfig:
    name: str
    hidden: int
    experts: int
    top_k: int
    inter: int
    tokens: int
    dtype: torch.dtype
    # routing: "none" (x.W_r), "normal" (N(0,1) bias), "zipf", "dirichlet"
    bias: str = "none"
    router_fp32: bool = True
    renormalize: bool = True
    shared_inter: int = 0          # FFN width of each shared expert (0 = none)
    shared_count: int = 0          # number of shared experts
    shared_gate: bool = False      # sigmoid(x.w_s) gate on the shared output
    steps: int = 1                 # routing draws (C5: one Dirichlet per step)
    seed: int = 0
    activation: str = "silu"

    @property
    def flops(self) -> float:
        """Algorithmic GEMM FLOPs of one forward (routed + shared experts)."""
        routed = 2.0 * self.tokens * self.top_k * 3 * self.hidden * self.inter
        shared = 2.0 * self.tokens * 3 * self.hidden * self.shared_inter * self.shared_count
        return routed + shared

    def expert_bytes(self) -> int:
        return 3 * self.hidden * self.inter * torch.tensor([], dtype=self.dtype).element_size()


CONFIGS: Dict[str, MoEConfig] = {
    "c1_tiny_fp32": MoEConfig("c1_tiny_fp32", 1024, 8, 2, 2816, 64, torch.float32,
                              bias="none", router_fp32=True),
    "c2_mixtral_bf16": MoEConfig("c2_mixtral_bf16", 4096, 8, 2, 14336, 4096, torch.bfloat16,
                                 bias="normal"),
    "c3_qwen_decode": MoEConfig("c3_qwen_decode", 2048, 60, 4, 1408, 64, torch.bfloat16,
                                bias="zipf", shared_inter=5632, shared_count=1,
                                shared_gate=True),
    "c4_dsv2lite_ep": MoEConfig("c4_dsv2lite_ep", 2048, 64, 6, 1408, 8192, torch.bfloat16,
                                bias="none", shared_inter=1408, shared_count=2),
    "c5_mixtral22b_offload": MoEConfig("c5_mixtral22b_offload", 6144, 8, 2, 16384, 2048,
                                       torch.bfloat16, bias="dirichlet", steps=16),
}


def mini(cfg: MoEConfig, *, hidden: int, inter: int, tokens: int,
         shared_inter: Optional[int] = None, name: Optional[str] = None, **kw) -> MoEConfig:
    """A shrunken copy of ``cfg`` (same E, K, routing, dtype) for fast parity cases."""
    return replace(
        cfg, name=name or f"{cfg.name}_mini", hidden=hidden, inter=inter, tokens=tokens,
        shared_inter=(shared_inter if shared_inter is not None else
                      (inter if cfg.shared_count else 0)), **kw)


def router_bias(cfg: MoEConfig, step: int = 0, *, gen: Optional[torch.Generator] = None) -> Optional[torch.Tensor]:
    """Per-expert logit bias [E] fp32 for ``cfg`` (None when the config has none).

    * normal:    b ~ N(0, 1), drawn from ``gen`` after the activations.
    * zipf:      b_e = log(r_e^-1.1 / sum_j r_j^-1.1), r = a seeded random rank permutation.
    * dirichlet: b = log(p + 1e-9), p ~ Dirichlet(0.3 * 1_E), one draw per step.
    """
    E = cfg.experts
    if cfg.bias == "none":
        return None
    if cfg.bias == "normal":
        assert gen is not None
        return torch.randn(E, generator=gen, dtype=torch.float32)
    if cfg.bias == "zipf":
        rng = np.random.default_rng(cfg.seed + 1009)
        ranks = rng.permutation(E) + 1
        p = ranks.astype(np.float64) ** -1.1
        p = p / p.sum()
        return torch.from_numpy(np.log(p)).float()
    if cfg.bias == "dirichlet":
        rng = np.random.default_rng(cfg.seed + 7919)
        draws = rng.dirichlet(np.full(E, 0.3), size=max(1, cfg.steps))
        return torch.from_numpy(np.log(draws[step] + 1e-9)).float()
    raise ValueError(f"unknown bias kind {cfg.bias!r}")


def generate(cfg: MoEConfig, *, device: str = "cpu", with_x: bool = True) -> Dict[str, object]:
    """Draw the layer's weights, activations and router bias.

    Returns a dict with ``gate`` [E,H], ``w1`` [E,2I,H] (rows 0..I-1 = gate_proj,
    I..2I-1 = up_proj), ``w2`` [E,H,I], optional ``shared_w1`` [S,2Is,H],
    ``shared_w2`` [S,H,Is], ``shared_gate`` [H], ``x`` [T,H] and ``bias`` (a
    list with one [E] tensor per routing step, or None).  Weights are in
    ``cfg.dtype``; ``gate`` is in ``cfg.dtype`` too (the router upcasts).
    """
    E, H, I, T = cfg.experts, cfg.hidden, cfg.inter, cfg.tokens
    dt = cfg.dtype
    if device == "cpu":
        g = torch.Generator().manual_seed(cfg.seed)

        def rn(*shape, scale=1.0):
            t = torch.randn(*shape, generator=g, dtype=torch.float32)
            if scale != 1.0:
                t.mul_(scale)
            return t.to(dt)
    else:
        g = torch.Generator(device=device).manual_seed(cfg.seed)

        def rn(*shape, scale=1.0):
            # drawn straight in the storage dtype to keep peak memory at 1x
            t = torch.randn(*shape, generator=g, dtype=dt, device=device)
            if scale != 1.0:
                t.mul_(scale)
            return t

    out: Dict[str, object] = {}
    out["gate"] = rn(E, H, scale=0.02)
    out["w1"] = rn(E, 2 * I, H, scale=0.02)
    out["w2"] = rn(E, H, I, scale=0.02)
    if cfg.shared_count:
        S, Is = cfg.shared_count, cfg.shared_inter
        out["shared_w1"] = rn(S, 2 * Is, H, scale=0.02)
        out["shared_w2"] = rn(S, H, Is, scale=0.02)
        out["shared_gate"] = rn(H, scale=0.02) if cfg.shared_gate else None
    if with_x:
        out["x"] = rn(T, H)
    if cfg.bias == "normal":
        gb = g if device == "cpu" else torch.Generator().manual_seed(cfg.seed + 1)
        out["bias"] = [torch.randn(E, generator=gb, dtype=torch.float32).to(device)]
    elif cfg.bias == "none":
        out["bias"] = None
    else:
        out["bias"] = [router_bias(cfg, s).to(device) for s in range(max(1, cfg.steps))]
    return out
