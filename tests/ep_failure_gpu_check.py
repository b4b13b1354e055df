"""Run under torchrun on 2 GPUs (one process per GPU, NCCL_NVLS_ENABLE=0): a rank
leaves the expert-parallel group between steps, with nothing of its own in
flight, and the survivor's next step raises PeerFailure before it launches
anything.  Used by tests/test_gpu_ep.py (2-GPU boxes).

The layer uses the NCCL exchange, so no rank maps another rank's memory; the
departing rank announces itself in the process group's store
(``PeerHealth.leave``) and exits; the survivor checks the store before its
next step.  Prints STEP1_OK, LEFT and PEER_FAILURE_SEEN.
"""
from __future__ import annotations

import os
import sys
import time
from datetime import timedelta

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main():
    rank = int(os.environ["RANK"])
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    dist.init_process_group("nccl", timeout=timedelta(seconds=30))
    from mosaic_b200 import MoEConfig, MoELayer, PeerFailure, PeerHealth, synthetic
    from mosaic_b200.ep import ExpertParallelMoELayer

    store = dist.distributed_c10d._get_default_store()
    health = PeerHealth(store, 2, rank, prefix="ep_failure_gpu")
    cfg = MoEConfig(hidden_size=512, moe_intermediate_size=256, n_routed_experts=32, num_experts_per_tok=4,
                    n_group=4, topk_group=2, routed_scaling_factor=2.5, act_mode="bf16")
    layer = MoELayer(cfg, synthetic.make_bank(512, 256, 32, 5))
    synthetic.make_router(layer, 5)
    ep = ExpertParallelMoELayer.from_layer(layer)
    ep.health = health
    x = synthetic.make_tokens(48, 512, 600 + rank)
    y = ep(x)  # step 1 on both ranks
    torch.cuda.synchronize()
    if not torch.equal(y, layer(x)):
        print(f"rank {rank}: step 1 differs from the single-GPU layer", flush=True)
        os._exit(1)
    print(f"rank {rank} STEP1_OK", flush=True)
    dist.barrier()
    torch.cuda.synchronize()
    if rank == 1:  # leaves between steps: nothing in flight
        health.leave()
        store.set("ep_failure_gpu/test_left", "1")
        print("rank 1 LEFT", flush=True)
        os._exit(0)
    store.wait(["ep_failure_gpu/test_left"])
    t0 = time.monotonic()
    try:
        ep(x)
        print("rank 0: step 2 ran without an error", flush=True)
        os._exit(1)
    except PeerFailure as e:
        print(f"rank 0 PEER_FAILURE_SEEN after {time.monotonic() - t0:.3f} s: {e}", flush=True)
    # no collective with the departed rank: leave without tearing the group down
    os._exit(0)


if __name__ == "__main__":
    main()
