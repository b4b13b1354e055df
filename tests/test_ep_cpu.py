"""Expert-parallel layer orchestration on gloo CPU ranks (no GPU).

Each rank holds its tokens and its contiguous slice of the experts; the layer
routes, dispatches by all-to-all, runs its experts on what it received, returns
the partials and combines.  With the oracle-backed test kernels the result must
equal the single-process oracle layer on the same tokens.
"""
from __future__ import annotations

import os
import socket
import traceback

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _local_bank(obank: dict, lo: int, hi: int) -> dict:
    return {k: np.concatenate([obank[k][lo:hi], obank["sh_" + k][None]]) for k in
            ("gu_packed", "gu_scale", "dn_packed", "dn_scale")}


def _worker(rank, world, port, case_name, mode, tokens_split, err_q, hash_k=None):
    try:
        import sys

        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        sys.path.insert(0, root)
        torch.set_num_threads(1)
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
        from mosaic_b200 import MoEConfig
        from mosaic_b200.ep import ExpertParallelMoELayer, expert_range
        from oracle.moe import moe_layer
        from oracle.router import hash_route, route
        from tests.ep_cpu_kernels import CpuEPKernels
        from tests.golden.recipes import MOE_CASES, make_hash_case, make_moe_case
        from tests.helpers import pack_case

        case = make_moe_case(**MOE_CASES[case_name])
        c = case["cfg"]
        obank, _ = pack_case(case)
        cfg = MoEConfig(hidden_size=c["H"], moe_intermediate_size=c["I"], n_routed_experts=c["E"],
                        num_experts_per_tok=c["k"], n_group=c["n_group"], topk_group=c["topk_group"],
                        routed_scaling_factor=c["scale"], swiglu_limit=c["swiglu_limit"], act_mode=mode,
                        scoring_func="sigmoid" if hash_k is None else "sqrtsoftplus")
        bounds = np.cumsum([0] + tokens_split)
        x_local = case["x"][bounds[rank]:bounds[rank + 1]]
        lo, hi = expert_range(c["E"], world, rank)
        kern = CpuEPKernels(case["router_w"], case["bias"], cfg, _local_bank(obank, lo, hi))
        if hash_k is None:
            layer = ExpertParallelMoELayer(cfg, None, kernels=kern)
            y = layer(x_local).float().numpy()
            w, idx = route(case["x"], case["router_w"], case["bias"], top_k=c["k"], n_group=c["n_group"],
                           topk_group=c["topk_group"], route_scale=c["scale"])
        else:  # hash-routed layer: ids by token id from a [V, hash_k] table
            _, _, table, tok = make_hash_case(int(bounds[-1]), c["H"], c["E"], hash_k, 211, seed=17)
            layer = ExpertParallelMoELayer(cfg, None, kernels=kern, layer_idx=4)
            layer.hash_router.tid2eid = table
            y = layer(x_local, tok[bounds[rank]:bounds[rank + 1]]).float().numpy()
            w, idx = hash_route(case["x"], case["router_w"], table, tok.numpy(), n_experts=c["E"],
                                score_func="sqrtsoftplus", route_scale=c["scale"])
        ref = moe_layer(case["x"], w, idx, obank, mode=mode, swiglu_limit=c["swiglu_limit"])
        ref = ref[bounds[rank]:bounds[rank + 1]]
        assert y.shape == ref.shape
        if y.size:
            rel = np.linalg.norm(y - ref) / max(np.linalg.norm(ref), 1e-30)
            assert rel <= 2e-3, f"rank {rank}: rel L2 {rel}"
            assert np.mean(y == ref) > 0.98, f"rank {rank}: only {np.mean(y == ref):.3f} of outputs bit-equal"
        # every rank received exactly the assignments of its experts
        sc, rc = layer.last_counts
        ids = idx.numpy()
        mine = ((ids >= lo) & (ids < hi)).sum()
        assert sum(rc) == mine, (rank, sum(rc), mine)
        dist.barrier()
        dist.destroy_process_group()
    except Exception:  # report to the parent, which fails the test
        err_q.put(f"rank {rank}:\n{traceback.format_exc()}")
        raise


def _run(world, case_name, mode, tokens_split, hash_k=None):
    ctx = mp.get_context("spawn")
    err_q = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, case_name, mode, tokens_split, err_q, hash_k))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    errors = []
    while not err_q.empty():
        errors.append(err_q.get())
    assert not alive, "a rank did not finish"
    assert not errors, "\n".join(errors)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]


@pytest.mark.parametrize("mode", ["bf16", "fp8"])
def test_ep_world2_matches_single_process(mode):
    _run(2, "S", mode, [40, 24])  # ragged token split


def test_ep_world4_uneven_and_empty_rank():
    _run(4, "S", "bf16", [30, 0, 20, 14])  # one rank has no tokens of its own


def test_ep_world2_hash_routed():
    """HashMoELayer semantics across ranks: a [V, 3] table (3 experts per token, not
    the config's 4) routes by token id; each rank passes its own tokens' ids."""
    _run(2, "S", "bf16", [40, 24], hash_k=3)
