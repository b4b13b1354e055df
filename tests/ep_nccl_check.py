"""Run under torchrun (one process per GPU): the expert-parallel layer over NCCL
must give, on every rank, exactly the single-GPU layer's output for that rank's
tokens.  Prints EP_OK per passing rank.  Used by tests/test_gpu_ep.py."""
from __future__ import annotations

import os
import sys
from datetime import timedelta

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def check_p2p(rank) -> bool:
    """Device-driven peer-memory exchange: eager and CUDA-graph steps equal the
    single-GPU layer on every rank, with no device error."""
    from mosaic_b200 import synthetic
    from mosaic_b200.ep import ExpertParallelMoELayer

    ok = True
    for act_mode, t, units in (("bf16", 128, False), ("fp8", 256, False), ("fp8", 256, True)):
        layer, _ = synthetic.make_layer(tokens=1, seed=78, act_mode=act_mode, n_experts=64)
        x = synthetic.make_tokens(t, 7168, 2000 + rank)
        ep = ExpertParallelMoELayer.from_layer(layer, exchange="p2p", max_tokens=t, unit_rows=units)
        ref = layer(x)
        for _ in range(3):
            y = ep(x)
        torch.cuda.synchronize()
        if not torch.equal(y, ref):
            ok = False
            print(f"rank {rank} p2p {act_mode} units={units}: eager mismatch", flush=True)
        xs = x.clone()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            ys = ep(xs)
        x2 = synthetic.make_tokens(t, 7168, 3000 + rank)
        xs.copy_(x2)
        for _ in range(5):
            g.replay()
        torch.cuda.synchronize()
        if not torch.equal(ys, layer(x2)):
            ok = False
            print(f"rank {rank} p2p {act_mode} units={units}: graph mismatch", flush=True)
        err = ep.peer_exchange().error()
        if err:
            ok = False
            print(f"rank {rank} p2p {act_mode} units={units}: device error {err}", flush=True)
        del g
        ep.close()
        del layer, ep
        torch.cuda.empty_cache()
    return ok


def main():
    rank = int(os.environ["RANK"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120))
    from mosaic_b200 import synthetic
    from mosaic_b200.ep import ExpertParallelMoELayer

    ok = True
    ok &= check_p2p(rank)
    for act_mode, t, e in (("bf16", 128, 64), ("fp8", 512, 64), ("bf16", 1, 64)):
        layer, _ = synthetic.make_layer(tokens=1, seed=77, act_mode=act_mode, n_experts=e)  # same bank everywhere
        x = synthetic.make_tokens(t, 7168, 1000 + rank)  # each rank its own tokens
        ep = ExpertParallelMoELayer.from_layer(layer)
        for _ in range(2):
            y = ep(x)
        ref = layer(x)
        torch.cuda.synchronize()
        if not torch.equal(y, ref):
            ok = False
            print(f"rank {rank} {act_mode} T={t}: mismatch, max abs {(y.float() - ref.float()).abs().max()}",
                  flush=True)
        del layer, ep
        torch.cuda.empty_cache()
    dist.barrier()
    dist.destroy_process_group()
    if ok:
        print(f"EP_OK rank {rank}", flush=True)
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()
