#!/usr/bin/env python
"""MoE-layer benchmark: tokens/s of one DeepSeek-V3-dimension MoE layer on B200.

Workload (the one the metric is quoted on): hidden 7168,
256 routed + 1 shared experts, moe_intermediate 2048, 8 groups / top-4 groups,
top-8, sigmoid + bias routing, routed_scaling 2.5, MXFP4 experts drawn from
N(0, 0.02), bf16 tokens ~ N(0, 1), uniform-random router, T = 128 tokens
(decode).  A step is one full layer (router -> layout -> expert gate/up ->
down -> combine, shared expert included) replayed from a CUDA graph.  The
expert weights the step touches (~5.9 GB) are far larger than L2 (126 MB),
so no L2 flush is needed between steps.

Prints ONE JSON line (rank 0).  With N > 1 (torchrun) the layer runs expert
parallel: each rank holds 256/N routed experts plus the shared expert and its
own T = 128 tokens (weak scaling), dispatch and combine are NCCL all-to-alls,
and the time is the max over ranks.  ``--impl reference`` times the reference
CPU expert path instead.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from datetime import timedelta
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

EXPERT_BYTES = 23_396_352          # MXFP4 codes + E8M0 scales of one V3 expert (gate/up + down)
GU_BYTES = 2 * 2048 * 3584 + 2 * 2048 * 224
DN_BYTES = 7168 * 1024 + 7168 * 64
ROUTER_BYTES = 256 * 7168 * 4
# DRAM traffic / algorithmic bytes of the gate/up launch: dram__bytes_read.sum +
# dram__bytes_write.sum of one ncu capture of `bench.py --experts 64 --profile-small`
# (65 experts streamed).  Traffic grows with the number of experts streamed, so the
# full launch's traffic is this ratio times its algorithmic bytes.
GU_TRAFFIC_RATIO = (1.0408e9 + 7.37e6) / 1_013_841_920
METRIC = "MoE-layer tokens/s at 1/2/4/8 B200; % of HBM / FP4 tensor roofline"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=400)
    p.add_argument("--warmup", type=int, default=20)
    p.add_argument("--impl", choices=["mosaic", "reference"], default="mosaic")
    p.add_argument("--tokens", type=int, default=128)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-extras", action="store_true", help="skip the T sweep and the prefill line")
    p.add_argument("--experts", type=int, default=256, help="routed experts in the bank (V3: 256)")
    p.add_argument("--act", choices=["bf16", "fp8"], default="bf16",
                   help="activation mode of the main layer (bf16: decode configs; fp8: prefill configs)")
    p.add_argument("--profile-small", action="store_true",
                   help="small case for ncu captures: no extras, no CPU baseline, 2 profiled stage runs")
    p.add_argument("--hc-only", action="store_true",
                   help="only the hyper-connection pre-mix + RMSNorm timing (prints its JSON; for ncu captures)")
    p.add_argument("--router-only", action="store_true",
                   help="only the router (V3: H 7168, E 256, groups 8/4, top 8) at T = 1, 128, 2048, 8192, "
                        "or at --tokens when given (prints its JSON; for ncu captures)")
    return p.parse_args()


def peaks():
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        d = json.loads(f.read_text())
        return d.get("hbm_gbs", 6650.0), d.get("bf16_tflops", 1590.0), "measured"
    return 6650.0, 1590.0, "fallback"


class Clocks:
    """nvidia-smi sampler running during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", str(self.gpu)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.15)
        return self

    def __exit__(self, *a):
        self.out = ""
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out = ""

    def summary(self):
        rows = [r.split(",") for r in (self.out or "").strip().splitlines() if r.count(",") >= 8]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if "Active" in v and "Not" not in v})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def gpu_index(local_rank: int) -> int:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        try:
            return int(vis.split(",")[local_rank])
        except (ValueError, IndexError):
            return local_rank
    return local_rank


def timed_graph(graph, steps, warmup, dist_on):
    for _ in range(warmup):
        graph.replay()
    torch.cuda.synchronize()
    if dist_on:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        graph.replay()
    b.record()
    torch.cuda.synchronize()
    if dist_on:
        torch.distributed.barrier()
    ms = a.elapsed_time(b) / steps
    if dist_on:
        t = torch.tensor([ms], device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    return ms


def check_device_error(layer, t, where):
    """Fail loudly if a kernel of the timed region recorded an error (e.g. a bounded wait that ran out)."""
    from mosaic_b200 import ops

    code = ops.read_error(layer.workspace(t, torch.device("cuda")))
    if code:
        raise RuntimeError(f"device error {code} recorded during {where}")


def capture(layer, x):
    static_x = x.clone()
    for _ in range(3):
        layer(static_x)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        static_y = layer(static_x)
    return g, static_x, static_y


def stage_times(layer, x, reps=20):
    """Per-stage device times (ms) of the eager layer from events recorded by the C ABI."""
    import ctypes

    from mosaic_b200 import _capi as C
    from mosaic_b200 import ops

    t = x.shape[0]
    dims = layer.cfg.dims(t, layer.bank.has_shared)
    ws = layer.workspace(t, x.device)
    y = torch.empty_like(x)
    w = torch.empty(t, layer.cfg.num_experts_per_tok, device=x.device)
    idx = torch.empty(t, layer.cfg.num_experts_per_tok, dtype=torch.int64, device=x.device)
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(7)]
    for e in evs:
        e.record()
    handles = (ctypes.c_void_p * 7)(*[e.cuda_event for e in evs])
    bank = layer.bank.c_struct()
    acc = [0.0] * 6
    for i in range(reps + 2):
        st = C.lib().mosaic_moe_forward_profiled(ctypes.byref(dims), ops._ptr(x), ops._ptr(layer.router.weight.data),
                                                 ops._ptr(layer.router.e_score_correction_bias.data),
                                                 ctypes.byref(bank), ops._ptr(y), ops._ptr(w), ops._ptr(idx),
                                                 ops._ptr(ws), ws.numel(), ops._stream(), handles)
        C.check(st, "mosaic_moe_forward_profiled")
        torch.cuda.synchronize()
        if i >= 2:
            for j in range(6):
                acc[j] += evs[j].elapsed_time(evs[j + 1])
    names = ["router", "layout", "quant", "gemm_gate_up", "gemm_down", "combine"]
    return {n: a / reps for n, a in zip(names, acc)}, idx


def e2e(layer, x, steps, dist_on):
    """Public-API time with host buffers: pinned H2D of x, layer(x), D2H of y, every step."""
    xh = x.cpu().pin_memory()
    yh = torch.empty_like(xh).pin_memory()
    xd = torch.empty_like(x)
    for _ in range(3):
        xd.copy_(xh, non_blocking=True)
        yh.copy_(layer(xd), non_blocking=True)
    torch.cuda.synchronize()
    if dist_on:
        torch.distributed.barrier()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        xd.copy_(xh, non_blocking=True)
        yh.copy_(layer(xd), non_blocking=True)
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / steps
    if dist_on:
        t = torch.tensor([ms], device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    return ms, xh.numel() * xh.element_size(), yh.numel() * yh.element_size()


def cpu_baseline(layer, x, idx, w, n_sample=16, seed=0):
    import numpy as np

    from mosaic_b200 import synthetic
    from oracle.cpu_path import time_layer_sample

    rng = np.random.default_rng(seed)
    touched = np.unique(idx.cpu().numpy())
    sample = np.sort(rng.choice(touched, size=min(n_sample, len(touched)), replace=False))
    bank = synthetic.bank_to_oracle(layer.bank, sample)
    bank["experts"] = sample
    c = layer.cfg
    r = time_layer_sample(x.cpu(), layer.router.weight.data.cpu(), layer.router.e_score_correction_bias.data.cpu(),
                          bank, idx.cpu().numpy(), w.cpu().numpy(), top_k=c.num_experts_per_tok, n_group=c.n_group,
                          topk_group=c.topk_group, route_scale=c.routed_scaling_factor, n_sample=len(sample))
    r["sample"] = (f"T={x.shape[0]} tokens, router on all tokens, {len(sample)} of {r['distinct_experts']} touched "
                   f"experts timed on their own tokens (+ shared expert on all tokens), best of {r['reps']} reps, "
                   f"scaled to the full layer; FP8-activation semantics (VNNI consumes E4M3)")
    return r


def run_reference(args):
    """--impl reference: the reference CPU expert path on the host cores (rank 0 only)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import numpy as np

    from oracle import formats as fm
    from oracle.cpu_path import time_layer_sample
    from oracle.router import route

    torch.set_num_threads(os.cpu_count() or 1)
    t, h, inter, e = args.tokens, 7168, 2048, 256
    g = torch.Generator().manual_seed(1234)
    bound = 1.0 / h ** 0.5
    rw = (torch.rand(e, h, generator=g) * 2 - 1) * bound
    bias = torch.randn(e, generator=g) * 0.01
    x = torch.randn(t, h, generator=g).to(torch.bfloat16)
    w, idx = route(x, rw, bias, top_k=8, n_group=8, topk_group=4, route_scale=2.5)
    touched = np.unique(idx.numpy())
    rng = np.random.default_rng(0)
    n_sample = 8
    sample = np.sort(rng.choice(touched, size=min(n_sample, len(touched)), replace=False))
    gu, dn = [], []
    for _ in list(sample) + ["shared"]:
        gu.append(fm.pack_mxfp4_nk(torch.randn(2 * inter, h, generator=g) * 0.02))
        dn.append(fm.pack_mxfp4_nk(torch.randn(h, inter, generator=g) * 0.02))
    bank = {"gu_packed": np.stack([p for p, _ in gu[:-1]]), "gu_scale": np.stack([s for _, s in gu[:-1]]),
            "dn_packed": np.stack([p for p, _ in dn[:-1]]), "dn_scale": np.stack([s for _, s in dn[:-1]]),
            "sh_gu_packed": gu[-1][0], "sh_gu_scale": gu[-1][1], "sh_dn_packed": dn[-1][0],
            "sh_dn_scale": dn[-1][1], "experts": sample}
    time_layer_sample(x, rw, bias, bank, idx.numpy(), w.numpy(), top_k=8, n_group=8, topk_group=4,
                      route_scale=2.5, reps=1)  # warm-up
    secs = []
    r = None
    steps = max(1, min(args.steps, 5))
    for _ in range(steps):
        r = time_layer_sample(x, rw, bias, bank, idx.numpy(), w.numpy(), top_k=8, n_group=8, topk_group=4,
                              route_scale=2.5, reps=1)
        secs.append(r["layer_seconds"])
    ms = 1e3 * sum(secs) / len(secs)
    value = t / (ms / 1e3)
    sample_desc = (f"T={t} decode tokens (V3 dims), router on all tokens, {len(sample)} of {r['distinct_experts']} "
                   f"touched experts timed on their own tokens + shared expert, scaled to the full layer, "
                   f"{steps} steps; FP8-activation semantics")
    out = {"metric": METRIC, "value": value, "unit": "tokens/s", "impl": "reference", "n_gpus": args.gpus,
           "steps": steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
           "vs_baseline": None, "dtype": "mxfp4*fp8 (cpu)", "data": "synthetic (seeded, CPU-generated)",
           "config": {"workload": "V3 MoE layer decode, T=128, 256+1 experts, top-8, groups 8/4",
                      "tokens": t, "hidden": h, "inter": inter, "experts": e, "parallelism": "cpu"},
           "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": r["cores"], "kind": r["kind"],
                            "sample": sample_desc, "cpu": r["cpu"]},
           "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    emit(out)


def timed_eager(fn, steps, warmup):
    """Device time (ms) per call of fn over `steps` calls, max over ranks."""
    dist = torch.distributed
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        fn()
    b.record()
    torch.cuda.synchronize()
    dist.barrier()
    ms = torch.tensor([a.elapsed_time(b) / steps], device="cuda")
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    return float(ms.item())


def run_ep(args, rank, world, local, hbm, peak_src):
    """N > 1: expert parallelism (BASELINE configs 4/5 layout).  Every rank holds
    E/N routed experts + the shared expert and its own decode tokens.  The
    headline step uses the device-driven peer-memory exchange and runs as one
    CUDA graph; the NCCL all-to-all path (host-synchronised split sizes) is
    timed beside it.  Times are the max over ranks."""
    from mosaic_b200 import synthetic
    from mosaic_b200.ep import ExpertParallelMoELayer

    dist = torch.distributed
    n_exp, t, h = args.experts, args.tokens, 7168
    # the same bank on every rank (same seed), each rank keeps its own shard
    layer, _ = synthetic.make_layer(tokens=1, seed=1234, act_mode="bf16", n_experts=n_exp)
    ep = ExpertParallelMoELayer.from_layer(layer, exchange="p2p", max_tokens=t)
    ep_nccl = ExpertParallelMoELayer(layer.cfg, ep.bank)
    ep_nccl.router = ep.router
    layer.bank = None  # drop the full bank: only the local shard stays resident
    torch.cuda.empty_cache()
    x = synthetic.make_tokens(t, h, 1234 + rank)
    steps, warmup = args.steps, max(args.warmup, 3)

    # one CUDA graph per layer step (peer exchange: no host synchronisation)
    xs = x.clone()
    for _ in range(3):
        ep(xs)
    torch.cuda.synchronize()
    dist.barrier()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        ys = ep(xs)
    with Clocks(gpu_index(local)) as clk:
        ms = timed_graph(g, steps, warmup, True)
    clocks = clk.summary()
    if ep.peer_exchange().error():
        raise RuntimeError("device error recorded in the peer exchange")
    idx = ep.last_idx.clone()
    lo, hi = ep.e_lo, ep.e_hi
    # distinct local experts this rank streamed in a step, from every rank's routing
    all_idx = [torch.empty_like(idx) for _ in range(world)]
    dist.all_gather(all_idx, idx)
    ids = torch.unique(torch.cat(all_idx))
    u_local = int(((ids >= lo) & (ids < hi)).sum().item())
    rank_bytes = (u_local + 1) * EXPERT_BYTES + ROUTER_BYTES
    frac = torch.tensor([rank_bytes / (ms * 1e-3) / 1e9 / hbm], device="cuda")
    dist.all_reduce(frac, op=dist.ReduceOp.MIN)

    # e2e through the public API with host buffers: pinned H2D, the graph-replayed
    # step, D2H of the result, every step
    xh = x.cpu().pin_memory()
    yh = torch.empty_like(xh).pin_memory()

    def step_e2e():
        xs.copy_(xh, non_blocking=True)
        g.replay()
        yh.copy_(ys, non_blocking=True)

    e2e_ms = timed_eager(step_e2e, max(steps // 4, 10), 3)
    # the NCCL all-to-all path, eager (split sizes read on the host every step)
    nccl_ms = timed_eager(lambda: ep_nccl(x), max(steps // 4, 10), 3)
    sc, rc = ep_nccl.last_counts
    if ep.peer_exchange().error():
        raise RuntimeError("device error recorded in the peer exchange")
    out = {
        "metric": METRIC, "value": t * world / (ms / 1e3), "unit": "tokens/s", "n_gpus": world, "steps": steps,
        "warmup": warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "mxfp4*bf16 (bf16 as hi+lo e4m3, fp32 accumulate)",
        "data": "synthetic (seeded N(0,0.02) experts, N(0,1) tokens)",
        "config": {"workload": f"V3 MoE layer decode, expert parallel over {world} GPUs, T={t} per rank",
                   "tokens_per_gpu": t, "hidden": h, "inter": 2048, "experts": n_exp,
                   "experts_per_gpu": n_exp // world, "shared": "replicated", "top_k": 8, "groups": "8/4",
                   "parallelism": f"ep{world}",
                   "exchange": "NVLink peer-memory stores with device-side counts and flags (CUDA IPC)",
                   "l2": "no flush: every rank streams its touched experts (>> 126 MB L2) each step",
                   "graph": "one CUDA graph per layer step"},
        "clocks": clocks,
        # router 2, dispatch 3, exchange 3, shared expert 5, received rows 5, return 2, combine 1
        "gpu_launches": 21 * steps,
        "roofline": {"kernel": "whole EP layer step per rank (HBM: local experts streamed)", "bound": "hbm",
                     "achieved": rank_bytes / (ms * 1e-3) / 1e9, "peak": hbm, "unit": "GB/s",
                     "frac": float(frac.item()), "traffic": None, "peak_source": peak_src,
                     "distinct_local_experts": u_local},
        "exchange_bytes_per_rank": {"dispatch": sum(sc) * (2 * h + 16), "return": sum(sc) * h * 4},
        "nccl_path": {"ms_per_step": nccl_ms, "tokens_per_s": t * world / (nccl_ms / 1e3),
                      "exchange": "NCCL all_to_all_single, eager"},
        "e2e": {"value": t * world / (e2e_ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": xh.numel() * 2,
                "d2h_bytes_per_step": yh.numel() * 2, "ms_per_step": e2e_ms},
    }
    del g
    if not args.no_extras:
        # 4096 FP8 tokens per rank, uniform routing (NCCL exchange)
        from mosaic_b200 import MoEConfig

        cfgp = MoEConfig(act_mode="fp8", **{k: v for k, v in synthetic.V3.items()})
        epp = ExpertParallelMoELayer(cfgp, ep.bank)
        epp.router.weight.data = ep.router.weight.data
        epp.router.e_score_correction_bias.data = ep.router.e_score_correction_bias.data
        tp = 4096
        xp = synthetic.make_tokens(tp, h, 4321 + rank)
        msp = timed_eager(lambda: epp(xp), 10, 3)
        flops = tp * world * 9 * 88_080_384
        out["ep_prefill"] = {"tokens_per_gpu": tp, "ms": msp, "tokens_per_s": tp * world / (msp / 1e3),
                             "expert_tflops_per_gpu": flops / world / (msp * 1e-3) / 1e12,
                             "act": "fp8 (e4m3, per-128 pow2 scales)", "routing": "uniform",
                             "exchange": "NCCL all_to_all_single"}
        del epp, xp
    if not args.no_extras and world >= 4:
        # the 58-layer decode stack, expert parallel, one CUDA graph
        del ep_nccl
        ep.close()
        del ep
        torch.cuda.empty_cache()
        out["stack"] = run_stack(58, t, world, rank)
        if rank == 0:
            emit(out)
        dist.barrier()
        dist.destroy_process_group()
        return
    if rank == 0:
        emit(out)
    ep.close()
    del ep, ep_nccl
    dist.barrier()
    dist.destroy_process_group()


def run_stack(n_layers, t, world, rank):
    """Decode step through n_layers independent V3 MoE layers (fresh uniform
    router each, every layer reading the step's hidden states), expert parallel
    over the group, the whole step captured in one CUDA graph.  One peer
    exchange serves every layer (they run one after the other)."""
    from mosaic_b200 import MoEConfig, synthetic
    from mosaic_b200.ep import CudaEPKernels, ExpertParallelMoELayer, PeerExchange, expert_range

    dist = torch.distributed
    h, n_exp = 7168, 256
    kern = CudaEPKernels()  # workspaces shared: the layers run one after the other
    cfg = MoEConfig(act_mode="bf16", **synthetic.V3)
    lo, hi = expert_range(n_exp, world, rank)
    px = PeerExchange(max_tokens=t, top_k=8, n_experts=n_exp, hidden=h, partial_f32=True)
    layers = []
    for layer_id in range(n_layers):
        bank = synthetic.make_local_bank(h, 2048, n_exp, seed=5000 + layer_id, lo=lo, hi=hi)
        ep = ExpertParallelMoELayer(cfg, bank, exchange="p2p", peer_exchange=px, kernels=kern)
        w, b = synthetic.make_router_weights(h, n_exp, seed=7000 + layer_id)
        ep.router.weight.data = w
        ep.router.e_score_correction_bias.data = b
        layers.append(ep)
    x = synthetic.make_tokens(t, h, 99 + rank)
    outs = [None] * n_layers

    def step(xin):
        for i, ep in enumerate(layers):
            outs[i] = ep(xin)
        return outs[-1]

    for _ in range(2):
        step(x)
    torch.cuda.synchronize()
    dist.barrier()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        step(x)
    ms = timed_graph(g, 20, 3, True)
    if px.error():
        raise RuntimeError("device error recorded in the peer exchange (stack)")
    res = {"layers": n_layers, "tokens_per_gpu": t, "ms_per_step": ms, "ms_per_layer": ms / n_layers,
           "tokens_per_s": t * world / (ms / 1e3), "experts_per_gpu": hi - lo,
           "expert_weights_per_gpu_gb": n_layers * (hi - lo + 1) * EXPERT_BYTES / 1e9,
           "graph": f"one CUDA graph, {n_layers} layers x 21 kernels",
           "note": "layers are independent (each reads the step's hidden states); no norm / attention between them"}
    del g
    for ep in layers:
        ep.close()
    px.close()
    del layers, outs
    torch.cuda.empty_cache()
    return res


_RESULT_FD = None


def offload_bench(layer, n_layers=4, steps=10, warmup=3):
    """Experts streamed from pinned host memory through an LRU expert cache that
    holds about one layer's selection: every layer of a step misses, so the step
    time is the host-to-device copy of the selected experts plus the expert path."""
    from mosaic_b200 import synthetic
    from mosaic_b200.offload import ExpertCache, HostBank, OffloadedMoELayer

    host = HostBank.from_bank(layer.bank)
    res = {}
    for t in (1, 8):
        probe = synthetic.make_tokens(t, 7168, 700 + t)
        _, idx = layer.router(probe)
        cap = int(torch.unique(idx).numel()) + 8
        cache = ExpertCache(7168, 2048, capacity=cap)
        offs = []
        for key in range(n_layers):
            o = OffloadedMoELayer(layer.cfg, host, cache, layer_key=key)
            o.router.weight.data = layer.router.weight.data
            o.router.e_score_correction_bias.data = layer.router.e_score_correction_bias.data
            offs.append(o)
        xs = [synthetic.make_tokens(t, 7168, 800 + i) for i in range(steps + warmup)]
        for i in range(warmup):
            for o in offs:
                o(xs[i])
        torch.cuda.synchronize()
        b0, m0 = cache.bytes_copied, cache.misses
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(warmup, warmup + steps):
            for o in offs:
                o(xs[i])
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / steps
        copied = (cache.bytes_copied - b0) / steps
        res[str(t)] = {"ms_per_layer": ms / n_layers, "cache_experts": cap, "layers": n_layers,
                       "h2d_bytes_per_layer": copied / n_layers, "h2d_GBs": copied / (ms * 1e-3) / 1e9,
                       "misses_per_layer": (cache.misses - m0) / steps / n_layers}
        del offs, cache
    return res


def hc_bench(hbm, steps=20, warmup=3):
    """The fused hyper-connection pre-mix + RMSNorm (+ E4M3 act_quant) in front of
    the MoE at the V3 hidden size, hc = 4: the residual copies are read twice
    (the tensor-core mix, then the per-token pre-mix); "GBs" counts one read."""
    from mosaic_b200.hc import HyperConnections, RMSNorm, ffn_pre_norm

    d, hcm = 7168, 4
    hc = HyperConnections(d, hc_mult=hcm).cuda()
    norm = RMSNorm(d).cuda()
    res = {}
    for t in (128, 8192):
        g = torch.Generator(device="cuda").manual_seed(t)
        x = torch.randn(t, hcm, d, generator=g, device="cuda").to(torch.bfloat16)
        for quant in (False, True):
            for _ in range(warmup):
                ffn_pre_norm(x, hc, norm, quant=quant)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()  # replayed: device time without the host's launch gaps
            with torch.cuda.graph(graph):
                ffn_pre_norm(x, hc, norm, quant=quant)
            graph.replay()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(steps):
                graph.replay()
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / steps
            del graph
            nbytes = t * (hcm * d * 2 + d * 2 + (d + d // 32 if quant else 0))
            res[f"T{t}" + ("_quant" if quant else "")] = {
                "ms": ms, "GBs": nbytes / (ms * 1e-3) / 1e9, "hbm_frac": nbytes / (ms * 1e-3) / 1e9 / hbm,
                "mix_tflops": 2 * t * 24 * hcm * d / (ms * 1e-3) / 1e12}
    return res


def router_bench(tokens, steps=20, warmup=3):
    """mosaic_router alone at the V3 router dims: logits on the tensor cores
    (split-K; the W split in-kernel up to T = 128) and the group-limited top 8.
    Each timed call is a CUDA-graph replay of 10 router calls."""
    import ctypes
    from mosaic_b200 import _capi as C
    from mosaic_b200.ops import _ptr

    lib = C.lib()
    h, e = 7168, 256
    res = {}
    for t in tokens:
        g = torch.Generator(device="cuda").manual_seed(t)
        x = torch.randn(t, h, generator=g, device="cuda").to(torch.bfloat16)
        w = (torch.rand(e, h, generator=g, device="cuda") * 2 - 1) / h ** 0.5
        b = torch.randn(e, generator=g, device="cuda") * 0.01
        ws = torch.empty(lib.mosaic_router_workspace_bytes(t, h, e), dtype=torch.uint8, device="cuda")
        wo = torch.empty(t, 8, device="cuda")
        io = torch.empty(t, 8, dtype=torch.int64, device="cuda")

        def call():
            st = lib.mosaic_router(_ptr(x), _ptr(w), _ptr(b), t, h, e, 8, 8, 4, 2.5, 1, _ptr(wo), _ptr(io), _ptr(ws),
                                   ws.numel(), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
            C.check(st, "mosaic_router")

        for _ in range(warmup):
            call()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(10):
                call()
        graph.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
        del graph
        us = e0.elapsed_time(e1) / (10 * steps) * 1e3
        res[f"T{t}"] = {"us": us, "logit_tflops": 2 * t * e * h / (us * 1e-6) / 1e12}
    return res


def emit(out: dict) -> None:
    """Write the result line to the real stdout (see main)."""
    os.write(_RESULT_FD if _RESULT_FD is not None else 1, (json.dumps(out) + "\n").encode())


def main():
    global _RESULT_FD
    # Libraries write to stdout from C (NCCL's version banner, for one); the
    # result must be the only line there, so stdout points at stderr while
    # the bench runs and emit() writes to a saved copy of the real stdout.
    sys.stdout.flush()
    _RESULT_FD = os.dup(1)
    os.dup2(2, 1)
    args = parse()
    if args.impl == "reference":
        run_reference(args)
        return
    from mosaic_b200 import MoELayer, synthetic

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist_on = world > 1
    if dist_on:
        torch.distributed.init_process_group("nccl", timeout=timedelta(seconds=300))
    hbm, bf16_tf, peak_src = peaks()
    if args.hc_only:
        emit({"hc_pre_norm": hc_bench(hbm)})
        return
    if args.router_only:
        tokens = [args.tokens] if "--tokens" in sys.argv else [1, 128, 2048, 8192]
        emit({"router": router_bench(tokens, steps=max(args.steps // 20, 5), warmup=max(args.warmup, 3))})
        return
    if dist_on:
        run_ep(args, rank, world, local, hbm, peak_src)
        return
    n_exp = args.experts
    t = args.tokens
    layer, x = synthetic.make_layer(tokens=t, seed=1234 + rank, act_mode=args.act, n_experts=n_exp)

    g, sx, sy = capture(layer, x)
    steps, warmup = args.steps, max(args.warmup, 3)
    with Clocks(gpu_index(local)) as clk:
        ms = timed_graph(g, steps, warmup, dist_on)
    clocks = clk.summary()
    check_device_error(layer, t, "graph replays")
    stages, idx = stage_times(layer, x, reps=2 if args.profile_small else 20)
    u = int(torch.unique(idx).numel())
    w_last = layer.last_weights
    layer_bytes = (u + 1) * EXPERT_BYTES + ROUTER_BYTES + 2 * t * 7168 * 2
    gu_bytes = (u + 1) * GU_BYTES
    achieved = gu_bytes / (stages["gemm_gate_up"] * 1e-3) / 1e9
    e2e_ms, bi, bo = e2e(layer, x, max(steps // 4, 10), dist_on)
    check_device_error(layer, t, "e2e")
    value = t * world / (ms / 1e3)
    out = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": steps, "warmup": warmup,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": ("mxfp4*bf16 (bf16 as hi+lo e4m3, fp32 accumulate)" if args.act == "bf16"
                  else "mxfp4*fp8 (e4m3, per-128 pow2 scales, fp32 accumulate)"), "data": "synthetic (seeded N(0,0.02) experts, N(0,1) tokens)",
        "config": {"workload": (f"V3 MoE layer decode (BASELINE config 2), T={t}" if args.act == "bf16"
                                else f"V3 MoE layer, FP8 activations, T={t}, uniform routing"),
                   "tokens_per_gpu": t, "hidden": 7168,
                   "inter": 2048, "experts": n_exp, "shared": 1, "top_k": 8, "groups": "8/4",
                   "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                   "l2": "no flush: ~5.9 GB of touched expert weights per step >> 126 MB L2",
                   "graph": "one CUDA graph per layer step"},
        "clocks": clocks,
        "gpu_launches": 7 * steps,
        "roofline": {"kernel": "moe_gemm_kernel (gate/up, tcgen05 mxf8f6f4)", "bound": "hbm",
                     "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm, "traffic": GU_TRAFFIC_RATIO * gu_bytes,
                     "traffic_source": "ncu dram bytes of a 65-expert launch scaled by experts streamed",
                     "algorithmic_bytes": gu_bytes, "peak_source": peak_src,
                     "note": "algorithmic bytes = (distinct experts + shared) x gate/up MXFP4 codes + scales"},
        "layer_roofline": {"bytes": layer_bytes, "achieved_gbs": layer_bytes / (ms * 1e-3) / 1e9,
                           "frac": layer_bytes / (ms * 1e-3) / 1e9 / hbm, "distinct_experts": u},
        "stages_ms": stages,
        "e2e": {"value": t * world / (e2e_ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": bi,
                "d2h_bytes_per_step": bo, "ms_per_step": e2e_ms},
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline and not args.profile_small:
        try:
            r = cpu_baseline(layer, x, idx, w_last)
            out["cpu_baseline"] = {"value": r["tokens_per_s"], "unit": "tokens/s", "cores": r["cores"],
                                   "kind": r["kind"], "sample": r["sample"], "cpu": r["cpu"],
                                   "layer_ms": r["layer_seconds"] * 1e3}
        except Exception as exc:  # report, do not hide
            out["cpu_baseline"] = {"value": None, "error": f"{type(exc).__name__}: {exc}"}
    if not args.no_extras and not args.profile_small:
        # each extra is reported on its own: one that fails records its error
        # in the line and the headline numbers above are still printed
        def extra(key, fn):
            try:
                out[key] = fn()
            except Exception as exc:  # report, do not hide
                out[key] = {"error": f"{type(exc).__name__}: {exc}"}

        def decode_sweep():
            sweep = {}
            for tt in (1, 8, 32):
                lt = MoELayer(layer.cfg, layer.bank)
                lt.router.weight.data = layer.router.weight.data
                lt.router.e_score_correction_bias.data = layer.router.e_score_correction_bias.data
                xt = synthetic.make_tokens(tt, 7168, 99 + tt)
                gt, _, _ = capture(lt, xt)
                mst = timed_graph(gt, 200, 10, dist_on)
                st_t, idx_t = stage_times(lt, xt, reps=5)
                ut = int(torch.unique(idx_t).numel())
                bt = (ut + 1) * EXPERT_BYTES + ROUTER_BYTES + 2 * tt * 7168 * 2
                sweep[str(tt)] = {"ms": mst, "tokens_per_s": tt * world / (mst / 1e3), "distinct_experts": ut,
                                  "layer_hbm_frac": bt / (mst * 1e-3) / 1e9 / hbm,
                                  "gate_up_hbm_frac": (ut + 1) * GU_BYTES / (st_t["gemm_gate_up"] * 1e-3) / 1e9
                                  / hbm}
                del gt
            return sweep

        def prefill():
            # 8192 tokens, FP8 activations, Zipf(1.2) load
            from mosaic_b200 import MoEConfig

            cfgp = MoEConfig(act_mode="fp8", **{k: v for k, v in synthetic.V3.items()})
            lp = MoELayer(cfgp, layer.bank)
            lp.router.weight.data = layer.router.weight.data.clone()
            lp.router.e_score_correction_bias.data = layer.router.e_score_correction_bias.data.clone()
            zipf = synthetic.calibrate_zipf_bias(lp, alpha=1.2, tokens=8192, seed=5)
            xp = synthetic.make_tokens(8192, 7168, 555)
            gp, _, _ = capture(lp, xp)
            msp = timed_graph(gp, 20, 3, dist_on)
            st_p, _ = stage_times(lp, xp, reps=5)
            del gp
            flops = 8192 * 9 * 88_080_384
            gemm_ms = st_p["gemm_gate_up"] + st_p["gemm_down"]
            return {"tokens": 8192, "ms": msp, "tokens_per_s": 8192 * world / (msp / 1e3),
                    "expert_tflops": flops / (gemm_ms * 1e-3) / 1e12,
                    "frac_fp8_nominal_4500": flops / (gemm_ms * 1e-3) / 1e12 / 4500.0,
                    "frac_fp4_nominal_9000": flops / (gemm_ms * 1e-3) / 1e12 / 9000.0,
                    "stages_ms": st_p, "zipf": zipf}

        extra("decode_sweep", decode_sweep)
        extra("prefill", prefill)
        extra("offload", lambda: offload_bench(layer))
        extra("hc_pre_norm", lambda: hc_bench(hbm))
    del g
    if rank == 0:
        emit(out)
    if dist_on:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
