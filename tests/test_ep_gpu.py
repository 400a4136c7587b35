"""Expert parallelism on GPUs: a 1-rank NCCL group on one GPU (the whole
dispatch / regroup / GEMM / return path with a trivial exchange), and 2-rank
runs (token-sharded and replicated contracts) when two GPUs are visible.
Multi-rank cases run as child processes with a short process-group timeout."""

import os
import socket
import subprocess
import sys

import pytest
import torch

from conftest import ROOT, golden_config, load_golden, max_rel

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _build(cfg, d, dev):
    from reframework_b200.moe import FusedMoE
    moe = FusedMoE(cfg.experts, cfg.top_k, cfg.hidden, cfg.inter, dtype=cfg.dtype,
                   router_dtype=torch.float32, num_shared_experts=cfg.shared_count,
                   shared_intermediate_size=cfg.shared_inter, shared_expert_gate=cfg.shared_gate)
    with torch.no_grad():
        moe.gate.copy_(d["gate"])
        for e in range(cfg.experts):
            moe.experts_w1[e].copy_(d["w1"][e])
            moe.experts_w2[e].copy_(d["w2"][e])
        if cfg.shared_count:
            moe.shared_w1.copy_(d["shared_w1"])
            moe.shared_w2.copy_(d["shared_w2"])
    moe = moe.to(dev)
    if d["bias"] is not None:
        moe.set_router_bias(d["bias"][0])
    return moe


def test_ep_single_rank_matches_fused(cuda_ok):
    import torch.distributed as dist
    from reframework_b200 import _lib
    from reframework_b200.parallel import dist as D
    from reframework_b200.parallel.ep import EPFusedMoE
    from reframework_b200.workloads import generate
    rec = load_golden("c4_mini_bf16")
    cfg = golden_config(rec)
    d = generate(cfg)
    dev = torch.device("cuda", 0)
    D.init(backend="nccl", init_method=f"tcp://127.0.0.1:{_free_port()}", rank=0, world_size=1,
           ep_size=1, timeout_s=60, device_id=dev)
    try:
        full = _build(cfg, d, dev)
        ep = EPFusedMoE.from_full(full, 1, 0, token_sharded=True)
        x = d["x"].to(dev)
        with torch.no_grad():
            a = full(x)
            b = ep(x)
        assert torch.equal(a, b)
        assert max_rel(b, rec["out"]) < 1e-2
        assert ep.last_plan.recv_total == cfg.tokens * cfg.top_k
        assert _lib.device_status() == 0
        ep.close()
    finally:
        D.destroy()


WORKER = r"""
import os, sys, torch
sys.path.insert(0, {root!r})
sys.path.insert(0, os.path.join({root!r}, "tests"))
from conftest import golden_config, load_golden, max_rel
from reframework_b200.parallel import dist as D
from reframework_b200.parallel.ep import EPFusedMoE
from reframework_b200.workloads import generate
from test_ep_gpu import _build
rank = int(os.environ["RANK"]); world = int(os.environ["WORLD_SIZE"])
dev = torch.device("cuda", rank)
torch.cuda.set_device(dev)
D.init(backend="nccl", init_method="tcp://127.0.0.1:{port}", rank=rank, world_size=world, ep_size=world,
       timeout_s=60, device_id=dev)
rec = load_golden("c4_mini_bf16")
cfg = golden_config(rec)
d = generate(cfg)
full = _build(cfg, d, dev)
x = d["x"].to(dev)
with torch.no_grad():
    ref = full(x)
    ep_rep = EPFusedMoE.from_full(full, world, rank, token_sharded=False)
    rep = ep_rep(x)   # reference contract
    T = x.shape[0]
    lo, hi = T * rank // world, T * (rank + 1) // world
    ep_sh = EPFusedMoE.from_full(full, world, rank, token_sharded=True)
    shard = ep_sh(x[lo:hi])          # rows cross NVLink as peer stores
    ep_nc = EPFusedMoE.from_full(full, world, rank, token_sharded=True)
    ep_nc.p2p = False
    nccl = ep_nc(x[lo:hi])           # rows through NCCL all-to-alls
    again = ep_sh(x[lo:hi])          # second step on the same peer buffers
assert torch.equal(shard, ref[lo:hi]), "token-sharded rows differ from the single-process layer"
assert torch.equal(nccl, shard) and torch.equal(again, shard), "peer-memory and NCCL exchanges differ"
assert torch.equal(rep, ref), "replicated-contract output differs"
assert max_rel(rep, rec["out"]) < 1e-2
# redundant experts: replica weights fetched from their owners, rows of an
# expert split across its holders; the result must not change by a bit
ep = EPFusedMoE.from_full(full, world, rank, token_sharded=True)
with torch.no_grad():
    ep(x[lo:hi])
    pl = ep.rebalance(redundant=2)
    assert sum(len(s) for s in pl.slots) > cfg.experts  # at least one replica somewhere
    bal = ep(x[lo:hi])
assert torch.equal(bal, ref[lo:hi]), "rebalanced EP output differs"
from reframework_b200 import _lib
assert _lib.device_status() == 0, "a kernel set the device error word"
for m in (ep_rep, ep_sh, ep_nc, ep):
    m.close()
D.barrier()
D.destroy()
print("rank", rank, "ok")
"""


def test_ep_two_ranks_match_single_process(cuda_ok):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    port = _free_port()
    code = WORKER.format(root=ROOT, port=port)
    env = dict(os.environ, WORLD_SIZE="2", NCCL_NVLS_ENABLE="0")
    procs = [subprocess.Popen([sys.executable, "-c", code], env=dict(env, RANK=str(r)),
                              stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True) for r in range(2)]
    outs = []
    for p in procs:
        try:
            out, _ = p.communicate(timeout=240)
        except subprocess.TimeoutExpired:
            p.kill()
            out, _ = p.communicate()
        outs.append(out)
    for r, (p, out) in enumerate(zip(procs, outs)):
        assert p.returncode == 0, f"rank {r} failed:\n{out[-3000:]}"
