"""MoE-layer benchmark (Mixtral-8x7B shape, 4096 prefill tokens per GPU).

    python bench.py [--gpus N --steps K --warmup W] [--impl reference] [--config NAME]

One step = one full MoE-layer forward (router -> permute -> grouped gated GEMM
-> grouped down GEMM -> combine) over one batch of synthetic tokens.  Inputs
are resident in HBM for ``value``; ``e2e`` goes through the public API
(``FusedMoE.forward``) with the tokens copied in from pinned host memory and
the output copied back inside the timed region.  With N > 1 GPUs (torchrun)
the layer is expert-parallel (``EPFusedMoE``: experts sharded, tokens
all-to-all over NCCL), each rank bringing its own 4096 tokens (weak scaling);
time = max over ranks.

``--impl reference`` times the CPU restatement of the reference's torch path
(oracle/moe_oracle.py, the reference's per-call expert restack included) on
the host cores, one full 4096-token forward per step (the same workload as
the GPU arm).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

METRIC = "MoE-layer tokens/s at Mixtral-8x7B shape (H4096 E8 top2 I14336, 4096 prefill tokens per GPU)"
UNIT = "tokens/s"
DATA = "synthetic: seeded N(0,0.02) weights, N(0,1) activations, N(0,1) per-expert router bias (fp32 router)"
L2_NOTE = "L2 flushed (256 MB write) before every timed step; weights 2.8 GB > 126 MB L2"


def peaks():
    """(bf16 burst TFLOP/s, HBM GB/s, source) from MEASURED_PEAKS.json."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d.get("bf16_tflops", 1590.0), d.get("hbm_gbs", 6650.0), "measured"
    return 1590.0, 6650.0, "fallback"


def sustained_bf16_peak():
    """The bf16 GEMM rate under the power cap (seconds-long cuBLAS loop): the
    denominator for a tensor kernel timed inside back-to-back layer steps."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        if "bf16_tflops_sustained" in d:
            return d["bf16_tflops_sustained"], "measured"
    return 1400.0, "fallback"


TRAFFIC_FILE = os.path.join("profiles", "traffic.json")


def committed_traffic():
    p = os.path.join(ROOT, TRAFFIC_FILE)
    if os.path.exists(p):
        try:
            return json.load(open(p))
        except Exception:
            return {}
    return {}


_SAMPLER = r"""
import sys, time, signal, pynvml
out, gpus = sys.argv[1], [int(g) for g in sys.argv[2].split(",")]
pynvml.nvmlInit()
hs = [pynvml.nvmlDeviceGetHandleByIndex(i) for i in gpus]
mx = max(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM) for h in hs)
stop = []
signal.signal(signal.SIGTERM, lambda *a: stop.append(1))
with open(out, "w") as f:
    f.write("max,%d\n" % mx); f.flush()
    while not stop:
        for i, h in zip(gpus, hs):
            try:
                f.write("%.4f,%d,%d,%d\n" % (time.time(), i, pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM),
                                             pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)))
            except pynvml.NVMLError:
                pass
        time.sleep(0.002)
"""


class Clocks:
    """SM clock and clock-event reasons read through NVML (read-only, nothing
    is set) every 2 ms by a separate sampler process while the timed region
    runs, so the sampling never competes with the benchmark's own host work."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
               "sw_power_cap": 0x4, "hw_power_brake_slowdown": 0x80}

    def __init__(self, gpus, path=None):
        self.gpus = list(gpus)
        self.path = path or f"/tmp/rf_clocks_{os.getpid()}.csv"
        self.proc = None

    def start(self):
        import subprocess
        try:
            self.proc = subprocess.Popen([sys.executable, "-c", _SAMPLER, self.path,
                                          ",".join(str(g) for g in self.gpus)],
                                         stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
            return
        t_end = time.time() + 20
        while time.time() < t_end:  # wait until the sampler is producing samples
            try:
                if sum(1 for _ in open(self.path)) > 2:
                    break
            except OSError:
                pass
            time.sleep(0.02)

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=10)
        except Exception:
            self.proc.kill()
        mx, samples = None, []
        try:
            for line in open(self.path):
                p = line.strip().split(",")
                if p[0] == "max":
                    mx = float(p[1])
                elif len(p) == 4:
                    samples.append((float(p[0]), int(p[1]), float(p[2]), int(p[3])))
        except OSError:
            return None
        if not samples or mx is None:
            return None
        sm = [s[2] for s in samples]
        loaded = [v for v in sm if v > 0.5 * mx] or sm
        reasons = sorted(n for n, bit in self.REASONS.items() if any(s[3] & bit for s in samples))
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": mx, "reasons": reasons,
                "samples": len(samples), "source": "NVML in a sampler process, 2 ms"}


# ------------------------------------------------------------------- GPU arm
def build_layer(cfg, d, device):
    from reframework_b200.moe import FusedMoE
    moe = FusedMoE(cfg.experts, cfg.top_k, cfg.hidden, cfg.inter, dtype=cfg.dtype,
                   router_dtype=torch.float32, device=device)
    with torch.no_grad():
        moe.gate.copy_(d["gate"])
        w1b, w2b = moe._resident_banks()
        w1b.copy_(d["w1"])
        w2b.copy_(d["w2"])
    if d["bias"] is not None:
        moe.set_router_bias(d["bias"][0])
    return moe


def staged_forward(moe, x, ev):
    """FusedMoE.forward (resident, no shared experts) with an event between stages."""
    from reframework_b200 import kernels as K
    ev[0].record()
    w, ids32, _, _, _ = moe._router(x, ids32=True, ids64=False)
    ev[1].record()
    p = K.permute(ids32, moe.num_experts, x=x)
    ev[2].record()
    w1b, w2b = moe._resident_banks()
    h = torch.empty(p.rows_cap, moe.intermediate_size, dtype=x.dtype, device=x.device)
    K.grouped_gemm_gated(p.x_perm, w1b, p.offsets, p.counts, h, activation=moe.activation)
    ev[3].record()
    y = torch.empty(p.rows_cap, moe.hidden_size, dtype=x.dtype, device=x.device)
    K.grouped_gemm_down(h, w2b, p.offsets, p.counts, y)
    ev[4].record()
    out = torch.empty_like(x)
    K.combine(y, p.row_of_slot, w, out)
    ev[5].record()
    return out


def e2e_run(fwd, xh, steps, dev):
    """Serving-style loop through the public API: every step copies its tokens
    host -> device (H2D stream), runs the forward on the compute stream and
    copies the output device -> host (D2H stream).  Double-buffered device
    inputs let step i+1's copy-in and step i's copy-out overlap step i's
    compute.  Returns the device time of all ``steps`` in ms."""
    comp = torch.cuda.current_stream(dev)
    h2d = torch.cuda.Stream(dev)
    d2h = torch.cuda.Stream(dev)
    xd = [torch.empty(xh.shape, dtype=xh.dtype, device=dev) for _ in range(2)]
    oh = [torch.empty_like(xh).pin_memory() for _ in range(2)]
    freed = [torch.cuda.Event() for _ in range(2)]
    t0 = torch.cuda.Event(enable_timing=True)
    t0.record(comp)
    h2d.wait_event(t0)
    d2h.wait_event(t0)
    for i in range(steps):
        b = i % 2
        with torch.cuda.stream(h2d):
            if i >= 2:
                h2d.wait_event(freed[b])
            xd[b].copy_(xh, non_blocking=True)
            ready = torch.cuda.Event()
            ready.record(h2d)
        comp.wait_event(ready)
        o = fwd(xd[b])
        freed[b].record(comp)
        done = torch.cuda.Event()
        done.record(comp)
        with torch.cuda.stream(d2h):
            d2h.wait_event(done)
            oh[b].copy_(o, non_blocking=True)
        o.record_stream(d2h)
    t1 = torch.cuda.Event(enable_timing=True)
    t1.record(d2h)
    comp.wait_stream(d2h)
    comp.wait_stream(h2d)
    t1.synchronize()
    return t0.elapsed_time(t1)


# router x2 (tensor-core logits, top-k), permute x3 (histogram, scatter, gather), gated GEMM, down GEMM, combine
LAUNCHES_PER_FORWARD = 8
# EP, exchange planned on the device and carried over peer memory: router x2, permute x2 (histogram,
# scatter), counts push + collect, planner, dispatch push + wait, regroup gather, gated GEMM, down GEMM
# storing its rows into the token ranks' return buffers + return wait, combine
EP_LAUNCHES_PER_FORWARD = 14


def ep_roofline(layer, cfg, traces, maxrank):
    """Roofline of the dominant kernel of an expert-parallel step: this rank's
    gated GEMM (its local rows x 2I x H), timed live by the CUDA events the
    layer records at its phase boundaries in every timed step.  Every rank
    computes its own; the line reports the slowest rank's launch."""
    durs = []
    for tr in traces:
        marks = {b[0]: a[1].elapsed_time(b[1]) for a, b in zip(tr, tr[1:])}
        if "gated GEMM" in marks:
            durs.append(marks["gated GEMM"])
    st = getattr(layer, "_dp", None) or {}
    rows = int(st["seg_cnt"].sum().item()) if "seg_cnt" in st else 0
    ms = statistics.mean(durs) if durs else 0.0
    flop = 2.0 * rows * cfg.hidden * 2 * cfg.inter
    ach = flop / (ms / 1e3) / 1e12 if ms > 0 else 0.0
    # the slowest rank: the lowest achieved rate (max over ranks of its negation)
    worst = -maxrank(-ach)
    bf16_peak, _, src = peaks()
    return {"kernel": "grouped gated GEMM (K3) over this rank's expert rows", "bound": "tensor",
            "achieved": worst, "peak": bf16_peak, "unit": "TFLOP/s", "frac": worst / bf16_peak,
            "peak_source": f"{src} bf16 burst (cuBLAS 8192^3, best of 10)",
            "achieved_rank0": ach, "rows_rank0": rows, "launch_ms_rank0": ms,
            "traffic": None, "traffic_source": "no ncu capture of the expert-parallel launch"}


def ep_launches(layer) -> int:
    """Launches of one EP forward (host-planned exchange: no planner kernel, and
    one more gather when replicas reorder the sent rows)."""
    if layer.p2p and layer.device_plan:
        return EP_LAUNCHES_PER_FORWARD
    plan = layer.last_plan  # + return push, - planner
    return EP_LAUNCHES_PER_FORWARD + (1 if plan is not None and plan.send_index is not None else 0)


def run_gpu(args):
    from reframework_b200.workloads import CONFIGS, generate
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    from reframework_b200.parallel.dist import bind_to_device_cpus
    # host threads and (first-touch) pinned buffers on the GPU's own NUMA node
    host_cpus = bind_to_device_cpus(dev)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    cfg = CONFIGS[args.config]
    T = cfg.tokens
    d = generate(cfg, device=str(dev), with_x=False)
    gx = torch.Generator(device=dev).manual_seed(cfg.seed + 101 + rank)
    x = torch.randn(T, cfg.hidden, generator=gx, device=dev, dtype=cfg.dtype)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    if world > 1:
        from reframework_b200.parallel.ep import EPFusedMoE
        full = build_layer(cfg, d, dev)
        layer = EPFusedMoE.from_full(full, world, rank, token_sharded=True)
        del full
        torch.cuda.empty_cache()
        if args.redundant > 0:
            # load-balancing calibration: one forward gives the global per-expert
            # counts, then every rank takes `redundant` replicas of busy experts
            with torch.no_grad():
                layer(x)
            layer.rebalance(redundant=args.redundant)

        def fwd(inp):
            return layer(inp)
        stage_fn = None
    else:
        layer = build_layer(cfg, d, dev)
        fwd = layer
        stage_fn = staged_forward
    del d

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    nev = 6
    with torch.no_grad():
        for _ in range(args.warmup):
            if stage_fn:
                stage_fn(layer, x, [torch.cuda.Event(enable_timing=True) for _ in range(nev)])
            else:
                fwd(x)
        clocks = Clocks(range(world), args.clocks_out)
        if rank == 0:
            clocks.start()  # before the barrier: no rank may start timing while rank 0 sets up sampling
        barrier()
        step_ms, stage_ms, phase_traces = [], [], []
        for _ in range(args.steps):
            flush.zero_()
            if stage_fn:
                ev = [torch.cuda.Event(enable_timing=True) for _ in range(nev)]
                stage_fn(layer, x, ev)
                stage_ms.append(ev)
            else:
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                layer.trace = []  # phase-boundary events (the gated GEMM's live duration)
                e0.record()
                fwd(x)
                e1.record()
                stage_ms.append([e0, e1])
                phase_traces.append(layer.trace)
        barrier()
        if world > 1:
            layer.trace = None
        for ev in stage_ms:
            step_ms.append(ev[0].elapsed_time(ev[-1]))
        # ---- e2e through the public API with host buffers (serving-style pipeline)
        xh = x.to("cpu").pin_memory()
        e2e_run(fwd, xh, max(1, args.warmup), dev)
        barrier()
        e2e_total_ms = e2e_run(fwd, xh, args.steps, dev)
        barrier()
        clk = clocks.stop() if rank == 0 else None
    from reframework_b200 import _lib
    status = _lib.device_status()
    if status != 0:
        raise RuntimeError(f"device error word set during the benchmark: {_lib.DEV_ERRORS.get(status, status)}")

    def maxrank(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    ms = maxrank(sum(step_ms) / len(step_ms))
    ms_e2e = maxrank(e2e_total_ms / args.steps)
    tokens = T * world
    res = {
        "metric": METRIC, "value": tokens / (ms / 1e3), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "step_ms_rank0": {"min": min(step_ms), "median": statistics.median(step_ms), "max": max(step_ms)},
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": DATA,
        "config": {"workload": cfg.name, "hidden": cfg.hidden, "experts": cfg.experts, "top_k": cfg.top_k,
                   "inter": cfg.inter, "tokens_per_gpu": T, "global_tokens": tokens,
                   "router": "fp32 logits + N(0,1) bias", "parallelism": f"ep{world}" if world > 1 else "single",
                   "l2": L2_NOTE},
        "eplb": ({"redundant_slots_per_rank": args.redundant, "placement": [list(s) for s in layer.placement.slots],
                  "calibration": "global per-expert counts of the first warm-up forward"}
                 if world > 1 else None),
        "e2e": {"value": tokens / (ms_e2e / 1e3), "unit": UNIT,
                "h2d_bytes_per_step": x.numel() * x.element_size(),
                "d2h_bytes_per_step": x.numel() * x.element_size(),
                "ms_per_step": ms_e2e, "api": "FusedMoE.forward" if world == 1 else "EPFusedMoE.forward",
                "pipeline": "H2D of step i+1 and D2H of step i on two copy streams overlap step i's forward",
                "host_cpus": (f"{len(host_cpus)} CPUs local to the GPU" if host_cpus else "unbound")},
        "gpu_launches": args.steps * (LAUNCHES_PER_FORWARD if world == 1 else ep_launches(layer)),
        "clocks": clk,
    }
    if stage_fn:
        names = ["router", "permute", "gemm_gated", "gemm_down", "combine"]
        per = {n: statistics.mean(ev[i].elapsed_time(ev[i + 1]) for ev in stage_ms) for i, n in enumerate(names)}
        res["stages_ms"] = per
        bf16_peak, hbm_peak, src = peaks()
        rows = T * cfg.top_k
        flop_g = 2.0 * rows * cfg.hidden * 2 * cfg.inter
        flop_d = 2.0 * rows * cfg.inter * cfg.hidden
        ach = flop_g / (per["gemm_gated"] / 1e3) / 1e12
        trd = committed_traffic()
        sus, sus_src = sustained_bf16_peak()
        sm_mhz = clk["sm_mhz"] if clk else None
        res["roofline"] = {"kernel": trd.get("gemm_gated_kernel", "grouped gated GEMM (K3)"), "bound": "tensor",
                           "achieved": ach, "peak": bf16_peak, "unit": "TFLOP/s", "frac": ach / bf16_peak,
                           "peak_source": f"{src} bf16 burst (cuBLAS 8192^3, best of 10): K3 is a 1-2 ms "
                                          "launch inside a sub-second timed region",
                           "peak_sustained": sus, "frac_sustained": ach / sus,
                           "traffic": trd.get("gemm_gated_bytes_per_launch"),
                           "traffic_source": (f"{TRAFFIC_FILE}: dram__bytes_read.sum + dram__bytes_write.sum of "
                                              "one K3 launch of this workload from a committed ncu capture, "
                                              "not measured in this run") if trd else None,
                           "algorithmic_flop_per_launch": flop_g,
                           "k3_ms_x_sm_mhz": (per["gemm_gated"] * sm_mhz) if sm_mhz else None,
                           "clock_note": "sm_mhz is NVML's reported clock sampled every 2 ms; ncu's "
                                         "sm__cycles_elapsed.avg.per_second for K3 is in the profile summary"}
        tot_ms = per["gemm_gated"] + per["gemm_down"]
        res["gemms_tflops"] = (flop_g + flop_d) / (tot_ms / 1e3) / 1e12
        res["layer_tflops"] = cfg.flops / (ms / 1e3) / 1e12
        byt_perm = rows * cfg.hidden * 2 * 2
        res["hbm"] = {"permute_gbs": byt_perm / (per["permute"] / 1e3) / 1e9,
                      "combine_gbs": (rows + T) * cfg.hidden * 2 / (per["combine"] / 1e3) / 1e9,
                      "peak_gbs": hbm_peak}
    if world > 1:
        res["roofline"] = ep_roofline(layer, cfg, phase_traces, maxrank)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        res["cpu_baseline"] = cpu_baseline(cfg, layer, budget_s=args.cpu_budget)
    if world > 1:
        layer.close()  # peer buffers (collective)
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(res))


# ------------------------------------------------------------ CPU reference arm
def _cpu_info():
    info = {"cores": os.cpu_count()}
    try:
        flags = open("/proc/cpuinfo").read()
        info["amx"] = "amx_bf16" in flags
        for line in flags.splitlines():
            if line.startswith("model name"):
                info["cpu"] = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    return info


def _cpu_layer_forward(x, gate, w1_list, w2_list, bias, top_k):
    """The reference's resident FusedMoE.forward on the CPU: restack every expert
    (moe_layer.py:444-445), fp32 router + bias, torch_fused_topk, fused_experts."""
    from oracle import moe_oracle as O
    w1 = torch.stack(w1_list, 0)
    w2 = torch.stack(w2_list, 0)
    w, ids = O.route(x, gate, top_k, True, bias=bias)
    return O.fused_experts(x, w1, w2, w, ids)


def cpu_baseline(cfg, layer, budget_s=25.0, sample_tokens=None):
    """Time the oracle port of the reference layer on the host cores (rank 0, N=1):
    full forwards of all the workload's tokens, as many as fit in the budget."""
    sample_tokens = sample_tokens or cfg.tokens
    torch.set_num_threads(os.cpu_count())
    w1b, w2b = layer._resident_banks()
    w1 = [w.cpu() for w in w1b]
    w2 = [w.cpu() for w in w2b]
    gate = layer.gate.detach().cpu()
    bias = layer.router_bias.cpu() if layer.router_bias is not None else None
    g = torch.Generator().manual_seed(5)
    x = torch.randn(sample_tokens, cfg.hidden, generator=g).to(cfg.dtype)
    _cpu_layer_forward(x, gate, w1, w2, bias, cfg.top_k)  # warm-up (thread pool, allocator)
    times = []
    t_end = time.perf_counter() + budget_s
    while not times or (time.perf_counter() < t_end and len(times) < 5):
        t0 = time.perf_counter()
        _cpu_layer_forward(x, gate, w1, w2, bias, cfg.top_k)
        times.append(time.perf_counter() - t0)
    s = statistics.median(times)
    info = _cpu_info()
    return {"value": sample_tokens / s, "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{sample_tokens} of the {cfg.tokens} tokens per call, {len(times)} timed calls "
                      f"(median {s:.2f} s) after one warm-up call; restack + fp32 router + torch bf16 "
                      "experts on the CPU",
            "cpu": info.get("cpu"), "amx": info.get("amx")}


def run_reference(args):
    """--impl reference: the reference path's CPU restatement on the host cores."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from reframework_b200.workloads import CONFIGS, generate
    cfg = CONFIGS[args.config]
    torch.set_num_threads(os.cpu_count())
    d = generate(cfg, with_x=False)
    w1 = list(d["w1"])
    w2 = list(d["w2"])
    bias = d["bias"][0] if d["bias"] is not None else None
    sample = args.ref_tokens or cfg.tokens
    g = torch.Generator().manual_seed(6)
    x = torch.randn(sample, cfg.hidden, generator=g).to(cfg.dtype)
    for _ in range(args.warmup):
        _cpu_layer_forward(x, d["gate"], w1, w2, bias, cfg.top_k)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        _cpu_layer_forward(x, d["gate"], w1, w2, bias, cfg.top_k)
        times.append(time.perf_counter() - t0)
    ms = 1e3 * sum(times) / len(times)
    v = sample / (ms / 1e3)
    info = _cpu_info()
    res = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": DATA,
        "config": {"workload": cfg.name, "hidden": cfg.hidden, "experts": cfg.experts, "top_k": cfg.top_k,
                   "inter": cfg.inter, "tokens_per_gpu": cfg.tokens, "sample_tokens_per_step": sample,
                   "same_config": sample == cfg.tokens, "parallelism": "cpu"},
        "cpu_baseline": {"value": v, "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
                         "sample": f"{sample} tokens per step (of {cfg.tokens}), {args.steps} timed steps after "
                                   f"{args.warmup} warm-up; reference restack + fp32 router + per-expert "
                                   "torch bf16 GEMMs",
                         "cpu": info.get("cpu"), "amx": info.get("amx")},
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(res))


def run_generic(args):
    """Other resident single-GPU workloads (C1 tiny fp32, C3 decode with a gated
    shared expert, C4 with two shared experts): eager forward and CUDA-graph
    replay, both timed with CUDA events, L2 flushed between steps."""
    from reframework_b200.moe import FusedMoE
    from reframework_b200.moe.graph import capture_forward
    from reframework_b200.workloads import CONFIGS, generate
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = CONFIGS[args.config]
    d = generate(cfg, device=str(dev), with_x=False)
    moe = FusedMoE(cfg.experts, cfg.top_k, cfg.hidden, cfg.inter, dtype=cfg.dtype, renormalize=cfg.renormalize,
                   router_dtype=torch.float32, num_shared_experts=cfg.shared_count,
                   shared_intermediate_size=cfg.shared_inter, shared_expert_gate=cfg.shared_gate, device=dev)
    with torch.no_grad():
        moe.gate.copy_(d["gate"])
        w1b, w2b = moe._resident_banks()
        w1b.copy_(d["w1"])
        w2b.copy_(d["w2"])
        if cfg.shared_count:
            moe.shared_w1.copy_(d["shared_w1"])
            moe.shared_w2.copy_(d["shared_w2"])
            if cfg.shared_gate:
                moe.shared_gate.copy_(d["shared_gate"])
    if d["bias"] is not None:
        moe.set_router_bias(d["bias"][0])
    del d
    gx = torch.Generator(device=dev).manual_seed(cfg.seed + 101)
    x = torch.randn(cfg.tokens, cfg.hidden, generator=gx, device=dev, dtype=cfg.dtype)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def timed(fn):
        for _ in range(args.warmup):
            fn(x)
        torch.cuda.synchronize()
        evs = []
        for _ in range(args.steps):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn(x)
            b.record()
            evs.append((a, b))
        torch.cuda.synchronize()
        return statistics.mean(a.elapsed_time(b) for a, b in evs)

    with torch.no_grad():
        ms_eager = timed(moe)
        graphed = capture_forward(moe, x)
        clocks = Clocks([0])
        clocks.start()
        ms_graph = timed(graphed)
        clk = clocks.stop()
        _, ids = moe.route(x)
    from reframework_b200 import _lib
    if _lib.device_status() != 0:
        raise RuntimeError("device error word set during the benchmark")
    active = int((torch.bincount(ids.reshape(-1), minlength=cfg.experts) > 0).sum())
    esz = torch.tensor([], dtype=cfg.dtype).element_size()
    weight_bytes = active * 3 * cfg.hidden * cfg.inter * esz + \
        cfg.shared_count * 3 * cfg.hidden * cfg.shared_inter * esz
    act_bytes = cfg.tokens * cfg.hidden * esz * (2 + 2 * cfg.top_k)
    bf16_peak, hbm_peak, src = peaks()
    ms = ms_graph
    hbm_ach = (weight_bytes + act_bytes) / (ms / 1e3) / 1e9
    tf_ach = cfg.flops / (ms / 1e3) / 1e12
    hbm_bound = (weight_bytes + act_bytes) / (hbm_peak * 1e9) > cfg.flops / (bf16_peak * 1e12)
    res = {
        "metric": f"MoE-layer tokens/s ({cfg.name})", "value": cfg.tokens / (ms / 1e3), "unit": UNIT,
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": str(cfg.dtype).replace("torch.", ""),
        "data": "synthetic: seeded N(0,0.02) weights, N(0,1) activations, config router bias",
        "config": {"workload": cfg.name, "hidden": cfg.hidden, "experts": cfg.experts, "top_k": cfg.top_k,
                   "inter": cfg.inter, "tokens": cfg.tokens, "shared": [cfg.shared_count, cfg.shared_inter,
                                                                          cfg.shared_gate],
                   "active_experts": active, "l2": L2_NOTE.split(";")[0]},
        "eager_ms_per_step": ms_eager, "graph_ms_per_step": ms_graph,
        "roofline": ({"bound": "hbm", "achieved": hbm_ach, "peak": hbm_peak, "unit": "GB/s",
                      "frac": hbm_ach / hbm_peak, "peak_source": src,
                      "algorithmic_bytes": weight_bytes + act_bytes} if hbm_bound else
                     {"bound": "tensor", "achieved": tf_ach, "peak": bf16_peak, "unit": "TFLOP/s",
                      "frac": tf_ach / bf16_peak, "peak_source": f"{src} bf16 burst (cuBLAS 8192^3, best of 10)",
                      "peak_sustained": sustained_bf16_peak()[0],
                      "frac_sustained": tf_ach / sustained_bf16_peak()[0]}),
        "clocks": clk,
    }
    print(json.dumps(res))


def run_offload(args):
    """Offload workload (C5): experts in pinned host memory, a few device slots.

    Each step routes 2048 tokens with its own Dirichlet(0.3) expert bias and
    runs the exact streaming forward (FusedMoE._forward_offload): resident
    experts first, every missing expert copied host->device on the copy
    stream into an evicted slot while earlier experts compute.  Reported:
    tokens/s over the steps, the host->device bytes and achieved GB/s, and the
    cache statistics."""
    from reframework_b200.moe import FusedMoE
    from reframework_b200.workloads import CONFIGS, generate
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = CONFIGS[args.config]
    d = generate(cfg, device=str(dev), with_x=False)
    moe = FusedMoE(cfg.experts, cfg.top_k, cfg.hidden, cfg.inter, dtype=cfg.dtype,
                   router_dtype=torch.float32, device=dev)
    with torch.no_grad():
        moe.gate.copy_(d["gate"])
        w1b, w2b = moe._resident_banks()
        w1b.copy_(d["w1"])
        w2b.copy_(d["w2"])
    biases = d["bias"]
    del d, w1b, w2b
    cache = moe.build_offload_cache(dev, lru_capacity=args.slots)
    if args.split:
        moe.enable_cpu_split()  # misses on int8 copies (the reference's CPU/GPU split, on the GPU)
    torch.cuda.empty_cache()
    bw = cache.measure_bandwidth()
    gx = torch.Generator(device=dev).manual_seed(cfg.seed + 101)
    x = torch.randn(cfg.tokens, cfg.hidden, generator=gx, device=dev, dtype=cfg.dtype)
    steps = max(args.steps, 1)
    with torch.no_grad():
        for s in range(args.warmup):
            moe.set_router_bias(biases[s % len(biases)])
            moe(x)
        torch.cuda.synchronize()
        cache.stats.reset()
        clocks = Clocks([0])
        clocks.start()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for s in range(steps):
            moe.set_router_bias(biases[s % len(biases)])
            moe(x)
        e1.record()
        torch.cuda.synchronize()
        clk = clocks.stop()
    ms = e0.elapsed_time(e1) / steps
    st = cache.stats.as_dict()
    h2d_bytes = (cache.stats.transfers_bytes + cache.int8_transfer_bytes) / steps
    res = {
        "metric": ("MoE-layer tokens/s with the expert offload cache (Mixtral-8x22B shape, 2048 tokens/step)"
                   + (", expert split: misses on int8 copies" if args.split else "")),
        "value": cfg.tokens / (ms / 1e3), "unit": UNIT, "n_gpus": 1, "steps": steps, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: seeded N(0,0.02) weights, N(0,1) activations, per-step log(Dirichlet(0.3)) bias",
        "config": {"workload": cfg.name, "hidden": cfg.hidden, "experts": cfg.experts, "top_k": cfg.top_k,
                   "inter": cfg.inter, "tokens_per_step": cfg.tokens, "device_slots": args.slots,
                   "policy": "lru (RE_CACHE_POLICY)", "expert_mb": cache.expert_bytes(0) / 2 ** 20,
                   "mode": "expert split (int8 misses)" if args.split else "exact streaming"},
        "offload": {"h2d_bytes_per_step": h2d_bytes, "h2d_gbs_achieved": h2d_bytes / (ms / 1e3) / 1e9,
                    "h2d_gbs_measured_peak": bw, "stats": st,
                    "copy_bound_ms_per_step": h2d_bytes / (bw * 1e9) * 1e3 if bw else None},
        "clocks": clk,
    }
    print(json.dumps(res))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="native", choices=["native", "reference"])
    ap.add_argument("--config", default="c2_mixtral_bf16")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-budget", type=float, default=25.0)
    ap.add_argument("--ref-tokens", type=int, default=0,
                    help="reference arm: tokens per step (0 = the workload's full token count)")
    ap.add_argument("--clocks-out", default=None,
                    help="CSV of the NVML clock samples (default: a temporary file)")
    ap.add_argument("--redundant", type=int, default=2,
                    help="EP: replica expert slots per rank for load balancing (0 = contiguous shards only)")
    ap.add_argument("--slots", type=int, default=4, help="offload workload: device expert slots")
    ap.add_argument("--split", action="store_true",
                    help="offload workload: the expert split (misses on int8 copies) instead of exact streaming")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.config.startswith("c5"):
        run_offload(args)
    elif args.config != "c2_mixtral_bf16" and int(os.environ.get("WORLD_SIZE", "1")) == 1:
        run_generic(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
