"""Generate the golden fixtures by running the Reframework reference itself.

Run in a container where the reference project is checked out (read-only):

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py --ref <reference root>

For every case it draws the seeded inputs with ``reframework_b200.workloads``,
runs the reference's torch MoE code on the CPU and saves, per case, a ``.pt``
file holding the config, the routing (``ids`` int64 [T,K], ``weights`` fp32
[T,K]), the per-expert token order the reference used (recorded by spying on
``Tensor.index_add_`` inside ``fused_experts``: ``perm_experts`` /
``perm_tokens``) and the output.  The inputs are not stored: tests redraw them
from the seed.

Reference code paths used (paths relative to the reference root):
  * ``FusedMoE.forward`` resident mode   reframework/moe/moe_layer.py:451-519
  * ``torch_fused_topk``                 reframework/moe/fused.py:32-46
  * ``fused_experts``                    reframework/moe/fused.py:49-87
  * ``FusedMoE._forward_streaming``      reframework/moe/moe_layer.py:354-420
  * ``MLP`` (shared experts)             reframework/layers/mlp.py:19-65
  * ``EPFusedMoE`` over 2 gloo ranks     reframework/parallel/ep.py:58-150,
                                         reframework/parallel/dist.py:135-176
  * ``FusedMoE._forward_split``          reframework/moe/moe_layer.py:523-627 with the
    int8 host bank (offload_cache.py:386-434, fused.py:89-197), at top-1 routing
    (where the reference's slot-to-token mapping is right) and RE_MAX_PACK=8 (so
    every miss is packed)
Where the benchmark configuration asks for an fp32 router with a bias (which
the reference's ``route`` cannot express), the case routes with
``softmax(x.float() @ gate.float().T + bias)`` through the reference's own
``torch_fused_topk`` and then calls the reference's ``fused_experts``.
"""

from __future__ import annotations

import argparse
import os
import sys
import tempfile

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from reframework_b200.workloads import CONFIGS, MoEConfig, generate, mini  # noqa: E402


def golden_cases():
    c = CONFIGS
    return [
        # (case name, config, mode)
        ("c1_tiny_fp32", c["c1_tiny_fp32"], "layer"),
        ("c2_mini_bf16", mini(c["c2_mixtral_bf16"], hidden=256, inter=512, tokens=256), "harness"),
        ("c3_mini_bf16", mini(c["c3_qwen_decode"], hidden=256, inter=128, tokens=64, shared_inter=512), "harness"),
        ("c4_mini_bf16", mini(c["c4_dsv2lite_ep"], hidden=256, inter=128, tokens=256), "harness"),
        ("c4_mini_norenorm", mini(c["c4_dsv2lite_ep"], hidden=256, inter=128, tokens=128,
                                  renormalize=False, name="c4_mini_norenorm"), "harness"),
        ("c5_mini_stream", mini(c["c5_mixtral22b_offload"], hidden=256, inter=256, tokens=128,
                                steps=3), "stream"),
        ("fp16_default", MoEConfig("fp16_default", 128, 8, 2, 256, 64, torch.float16,
                                   router_fp32=False, seed=3), "layer"),
        ("bf16_gelu_default", MoEConfig("bf16_gelu_default", 128, 8, 2, 128, 96, torch.bfloat16,
                                        router_fp32=False, seed=4, activation="gelu"), "layer"),
        ("fp32_gelu_tanh", MoEConfig("fp32_gelu_tanh", 128, 16, 3, 128, 40, torch.float32,
                                     seed=5, activation="gelu_tanh"), "layer"),
        ("bf16_entropy_k", MoEConfig("bf16_entropy_k", 128, 16, 4, 128, 64, torch.bfloat16,
                                     router_fp32=False, seed=6), "entropy"),
        ("ep2_mini_bf16", MoEConfig("ep2_mini_bf16", 256, 8, 2, 256, 64, torch.bfloat16,
                                    router_fp32=False, seed=7), "ep2"),
        ("int8_split_k1", mini(c["c5_mixtral22b_offload"], hidden=256, inter=256, tokens=96, steps=4,
                               top_k=1, seed=9, name="int8_split_k1"), "split"),
    ]


class _IndexAddSpy:
    """Record the ``index`` argument of every ``Tensor.index_add_`` call."""

    def __init__(self):
        self.calls = []

    def __enter__(self):
        self._orig = torch.Tensor.index_add_
        spy = self

        def index_add_(t, dim, index, source, *a, **k):
            spy.calls.append(index.detach().clone().long())
            return spy._orig(t, dim, index, source, *a, **k)

        torch.Tensor.index_add_ = index_add_
        return self

    def __exit__(self, *exc):
        torch.Tensor.index_add_ = self._orig


def _build_layer(FusedMoE, cfg: MoEConfig, d):
    moe = FusedMoE(cfg.experts, cfg.top_k, cfg.hidden, cfg.inter, activation=cfg.activation,
                   renormalize=cfg.renormalize, dtype=cfg.dtype)
    with torch.no_grad():
        moe.gate.copy_(d["gate"])
        for e in range(cfg.experts):
            moe.experts_w1[e].copy_(d["w1"][e])
            moe.experts_w2[e].copy_(d["w2"][e])
    return moe


def _ep_worker(rank, ctx, path, cfg_name, seed):
    # the parent's OpenMP pool does not survive fork(); stay single-threaded
    torch.set_num_threads(1)
    from reframework.moe import FusedMoE
    from reframework.parallel.ep import EPFusedMoE
    cfg = dict((n, c) for n, c, _ in golden_cases())[cfg_name]
    d = generate(cfg)
    base = _build_layer(FusedMoE, cfg, d)
    ep = EPFusedMoE.from_full(base, ctx.ep_size, ctx.ep_rank)
    with torch.no_grad():
        out = ep(d["x"])
    if rank == 0:
        torch.save(out, path)


def run_case(name: str, cfg: MoEConfig, mode: str):
    from reframework.moe import FusedMoE, fused_experts, torch_fused_topk
    from reframework.layers import MLP

    d = generate(cfg)
    x = d["x"]
    rec = {"name": name, "mode": mode, "config": {k: (str(v) if isinstance(v, torch.dtype) else v)
                                                   for k, v in cfg.__dict__.items()}}
    torch.manual_seed(1234)
    if mode in ("layer", "entropy"):
        moe = _build_layer(FusedMoE, cfg, d)
        if mode == "entropy":
            moe.entropy_adaptive_k = True
            moe.entropy_k_min = 2
        with torch.no_grad():
            w, ids = moe.route(x)
            with _IndexAddSpy() as spy:
                out = moe(x)
        rec.update(ids=ids, weights=w, out=out)
        if mode == "entropy":
            rec["entropy_k_min"] = 2
    elif mode == "harness":
        w1 = d["w1"]
        w2 = d["w2"]
        logits = x.float() @ d["gate"].float().t()
        if d["bias"] is not None:
            logits = logits + d["bias"][0]
        w, ids = torch_fused_topk(logits, cfg.top_k, cfg.renormalize)
        with torch.no_grad(), _IndexAddSpy() as spy:
            routed = fused_experts(x, w1, w2, w, ids, cfg.activation)
        out = routed
        if cfg.shared_count:
            sh = None
            for s in range(cfg.shared_count):
                mlp = MLP(cfg.hidden, cfg.shared_inter, cfg.activation).to(cfg.dtype)
                with torch.no_grad():
                    mlp.gate_up.weight.copy_(d["shared_w1"][s])
                    mlp.down.weight.copy_(d["shared_w2"][s])
                    y = mlp(x)
                sh = y if sh is None else sh + y
            if cfg.shared_gate:
                sg = torch.sigmoid(x.float() @ d["shared_gate"].float())
                sh = (sh.float() * sg.unsqueeze(-1)).to(x.dtype)
            out = routed + sh
            rec["routed_out"] = routed
        rec.update(ids=ids, weights=w, out=out, logits=logits)
    elif mode == "stream":
        moe = _build_layer(FusedMoE, cfg, d)
        moe.build_offload_cache(torch.device("cpu"), lru_capacity=4)
        os.environ["RE_CHUNK_SIZE"] = "4"
        outs, idss, wss = [], [], []
        try:
            for s in range(cfg.steps):
                logits = x.float() @ d["gate"].float().t() + d["bias"][s]
                w, ids = torch_fused_topk(logits, cfg.top_k, cfg.renormalize)
                with torch.no_grad():
                    o = moe._forward_streaming(x, x, w, ids, x.device)
                outs.append(o)
                idss.append(ids)
                wss.append(w)
        finally:
            del os.environ["RE_CHUNK_SIZE"]
        rec.update(ids=torch.stack(idss), weights=torch.stack(wss), out=torch.stack(outs),
                   cache_stats=moe._cache.stats.as_dict())
        spy = None
    elif mode == "split":
        moe = _build_layer(FusedMoE, cfg, d)
        moe.build_offload_cache(torch.device("cpu"), lru_capacity=4)
        moe.enable_cpu_split()
        os.environ["RE_MAX_PACK"] = "8"
        outs, idss, wss, res = [], [], [], []
        try:
            for s in range(cfg.steps):
                logits = x.float() @ d["gate"].float().t() + d["bias"][s]
                w, ids = torch_fused_topk(logits, cfg.top_k, cfg.renormalize)
                res.append(torch.tensor(sorted(moe._cache._lru.keys()), dtype=torch.long))
                with torch.no_grad():
                    o = moe._forward_split(x, x, w, ids)
                outs.append(o)
                idss.append(ids)
                wss.append(w)
        finally:
            del os.environ["RE_MAX_PACK"]
        rec.update(ids=torch.stack(idss), weights=torch.stack(wss), out=torch.stack(outs), resident_before=res,
                   resident_after=torch.tensor(sorted(moe._cache._lru.keys()), dtype=torch.long),
                   cache_stats=moe._cache.stats.as_dict())
        spy = None
    elif mode == "ep2":
        from reframework.parallel import run
        torch.set_num_threads(1)
        with tempfile.TemporaryDirectory() as td:
            p = os.path.join(td, "ep.pt")
            run(_ep_worker, world_size=2, backend="gloo",
                init_method="tcp://127.0.0.1:29731", ep_size=2, args=(p, name, cfg.seed))
            out_ep = torch.load(p)
        moe = _build_layer(FusedMoE, cfg, d)
        with torch.no_grad():
            w, ids = moe.route(x)
            out_full = moe(x)
        rec.update(ids=ids, weights=w, out=out_ep, out_single=out_full)
        spy = None
    else:
        raise ValueError(mode)

    if spy is not None:
        # fused_experts visits active experts in ascending order and calls
        # index_add_ once per expert with that expert's token ids, in order.
        exps = sorted(set(int(i) for i in rec["ids"].reshape(-1).tolist()))
        calls = spy.calls[-len(exps):]
        rec["perm_experts"] = torch.tensor(exps, dtype=torch.long)
        rec["perm_tokens"] = [c for c in calls]
    return rec


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="reference project root (read-only)")
    ap.add_argument("--only", default=None)
    args = ap.parse_args()
    sys.dont_write_bytecode = True
    sys.path.insert(0, args.ref)
    torch.set_num_threads(8)
    for name, cfg, mode in golden_cases():
        if args.only and name != args.only:
            continue
        rec = run_case(name, cfg, mode)
        path = os.path.join(HERE, f"{name}.pt")
        torch.save(rec, path)
        print(f"{name}: {os.path.getsize(path) / 1024:.1f} KB")


if __name__ == "__main__":
    main()
