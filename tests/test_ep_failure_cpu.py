"""Failure detection of the expert-parallel layer on gloo CPU ranks (no GPU).

A rank leaves only between steps, with nothing of its own in flight:

- one that says so (``PeerHealth.leave``) is seen by the others before they
  launch their next step (``PeerFailure`` from the store check, no collective);
- one that stalls (never joins the next step) or exits without a word ends the
  others' next collective through the process group's short timeout or the
  broken connection, raised as ``PeerFailure`` instead of a hang.
"""
from __future__ import annotations

import os
import socket
import time
import traceback
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

PG_TIMEOUT_S = 4


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, scenario, out_q):
    try:
        import sys

        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        sys.path.insert(0, root)
        torch.set_num_threads(1)
        store = dist.TCPStore("127.0.0.1", port, world, rank == 0, timeout=timedelta(seconds=60))
        dist.init_process_group("gloo", store=store, rank=rank, world_size=world,
                                timeout=timedelta(seconds=PG_TIMEOUT_S))
        from mosaic_b200 import MoEConfig, PeerFailure, PeerHealth
        from mosaic_b200.ep import ExpertParallelMoELayer, expert_range
        from tests.ep_cpu_kernels import CpuEPKernels
        from tests.golden.recipes import MOE_CASES, make_moe_case
        from tests.helpers import pack_case

        case = make_moe_case(**MOE_CASES["S"])
        c = case["cfg"]
        obank, _ = pack_case(case)
        cfg = MoEConfig(hidden_size=c["H"], moe_intermediate_size=c["I"], n_routed_experts=c["E"],
                        num_experts_per_tok=c["k"], n_group=c["n_group"], topk_group=c["topk_group"],
                        routed_scaling_factor=c["scale"], swiglu_limit=c["swiglu_limit"], act_mode="bf16")
        lo, hi = expert_range(c["E"], world, rank)
        local = {k: np.concatenate([obank[k][lo:hi], obank["sh_" + k][None]]) for k in
                 ("gu_packed", "gu_scale", "dn_packed", "dn_scale")}
        health = PeerHealth(store, world, rank)
        layer = ExpertParallelMoELayer(cfg, None, kernels=CpuEPKernels(case["router_w"], case["bias"], cfg, local),
                                       health=health)
        x = case["x"][rank * 16:(rank + 1) * 16]
        layer(x)  # step 1: every rank
        if rank == 1:  # the rank that goes, between steps
            if scenario == "leave":
                health.leave()
                store.set("test/left", "1")
                out_q.put((rank, "left", 0.0))
            elif scenario == "stall":
                out_q.put((rank, "stalling", 0.0))
                time.sleep(60)  # never joins step 2; the parent ends it
            else:  # "exit": gone without a word
                out_q.put((rank, "exiting", 0.0))
            os._exit(0)
        if scenario == "leave":
            store.wait(["test/left"])
        t0 = time.monotonic()
        try:
            layer(x)  # step 2
            out_q.put((rank, "no error", time.monotonic() - t0))
        except PeerFailure as e:
            out_q.put((rank, "PeerFailure: " + str(e).splitlines()[0][:200], time.monotonic() - t0))
        os._exit(0)
    except Exception:
        out_q.put((rank, "crash:\n" + traceback.format_exc(), -1.0))
        os._exit(1)


def _run(scenario):
    ctx = mp.get_context("spawn")
    out_q = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, scenario, out_q)) for r in range(2)]
    for p in procs:
        p.start()
    procs[0].join(timeout=120)
    for p in procs:  # the stalled rank (or anything left) is ended here
        if p.is_alive():
            p.kill()
        p.join(timeout=30)
    res = {}
    while not out_q.empty():
        r, what, dt = out_q.get()
        res[r] = (what, dt)
    return res


def test_rank_that_leaves_is_seen_before_the_next_launch():
    res = _run("leave")
    what, dt = res[0]
    assert what.startswith("PeerFailure: rank(s) [1] left"), res
    assert dt < 1.0, res  # the store check, no collective timeout


@pytest.mark.parametrize("scenario", ["stall", "exit"])
def test_rank_that_stops_ends_the_next_collective_with_an_error(scenario):
    res = _run(scenario)
    what, dt = res[0]
    assert what.startswith("PeerFailure: expert-parallel exchange failed on rank 0"), res
    assert dt < PG_TIMEOUT_S + 10, res  # bounded by the process group's timeout


def test_peer_health_store_semantics():
    """One store, three ranks' views: a departure is seen by the others (not by the
    rank itself), every departed rank is named, and prefixes keep groups apart."""
    from mosaic_b200 import PeerFailure, PeerHealth

    store = dist.HashStore()
    views = [PeerHealth(store, 3, r) for r in range(3)]
    other_group = PeerHealth(store, 3, 0, prefix="another_layer_group")
    for v in views:
        v.check()  # nobody left
    views[2].leave()
    views[2].check()  # its own departure is not a peer failure
    with pytest.raises(PeerFailure, match=r"\[2\]"):
        views[0].check()
    views[1].leave()
    with pytest.raises(PeerFailure, match=r"\[1, 2\]"):
        views[0].check()
    assert views[1].left() == [2] and views[2].left() == [1]
    other_group.check()  # a different prefix sees nothing
