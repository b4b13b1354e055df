"""mosaic_router_noalloc against mosaic_router on the GPU.

Collected last (file name) so it also runs after every other test has used the
device; it must pass alone as well.  The no-alloc entry point keeps its split-K
partials in the library's fixed device scratch, so two calls in a row must each
match the workspace entry point bit for bit (the second call finds the first
call's partials in the scratch and must overwrite them all).
"""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

# (T, H, E, top_k, n_group, topk_group): decode and prefill V3 routing, and a
# small ungrouped case whose split count differs.
CASES = [(128, 7168, 256, 8, 8, 4), (2048, 7168, 256, 8, 8, 4), (8192, 7168, 256, 8, 8, 4), (5, 512, 32, 4, 1, 1)]


def _inputs(t, h, e, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(t, h, generator=g, device="cuda").to(torch.bfloat16)
    w = torch.randn(e, h, generator=g, device="cuda") / h ** 0.5
    b = torch.randn(e, generator=g, device="cuda") * 0.01
    return x, w, b


@pytest.mark.parametrize("t,h,e,k,ng,tg", CASES)
def test_noalloc_matches_workspace_router_two_calls(t, h, e, k, ng, tg):
    from mosaic_b200 import ops

    kw = dict(top_k=k, n_group=ng, topk_group=tg, route_scale=2.5, norm_topk_prob=True)
    outs = []
    for call in range(2):
        x, w, b = _inputs(t, h, e, seed=10 * t + call)  # different inputs per call
        ref_w, ref_i = ops.router(x, w, b, **kw)
        got_w = torch.full((t, k), float("nan"), device="cuda")
        got_i = torch.full((t, k), -1, dtype=torch.int64, device="cuda")
        ops.router_noalloc(x, w, b, got_w, got_i, **kw)
        torch.cuda.synchronize()
        assert torch.equal(got_i, ref_i), f"call {call}: expert ids differ"
        assert torch.equal(got_w, ref_w), f"call {call}: weights differ"
        outs.append(got_i)
    assert not torch.equal(outs[0], outs[1])  # the two calls really routed different tokens


def test_noalloc_allocates_no_device_memory():
    from mosaic_b200 import ops

    t, h, e = 128, 7168, 256
    x, w, b = _inputs(t, h, e, seed=3)
    wo = torch.empty(t, 8, device="cuda")
    io = torch.empty(t, 8, dtype=torch.int64, device="cuda")
    ops.router_noalloc(x, w, b, wo, io, top_k=8, n_group=8, topk_group=4, route_scale=2.5)  # set-up call
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    stats0 = torch.cuda.memory_stats().get("allocation.all.allocated", 0)
    for _ in range(5):
        ops.router_noalloc(x, w, b, wo, io, top_k=8, n_group=8, topk_group=4, route_scale=2.5)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert torch.cuda.memory_stats().get("allocation.all.allocated", 0) == stats0
    assert free1 == free0


def test_noalloc_rejects_oversize_without_launch():
    from mosaic_b200 import ops

    t, h, e = 32768, 7168, 256
    x = torch.zeros(t, h, dtype=torch.bfloat16, device="cuda")
    w = torch.zeros(e, h, device="cuda")
    wo = torch.empty(t, 8, device="cuda")
    io = torch.empty(t, 8, dtype=torch.int64, device="cuda")
    with pytest.raises(ValueError, match="workspace"):
        ops.router_noalloc(x, w, None, wo, io, top_k=8, n_group=8, topk_group=4)


def test_noalloc_capturable_after_setup():
    """After the set-up call, the entry point records into a CUDA graph and the
    replay matches the workspace router."""
    from mosaic_b200 import ops

    t, h, e = 128, 7168, 256
    x, w, b = _inputs(t, h, e, seed=5)
    kw = dict(top_k=8, n_group=8, topk_group=4, route_scale=2.5)
    wo = torch.empty(t, 8, device="cuda")
    io = torch.empty(t, 8, dtype=torch.int64, device="cuda")
    ops.router_noalloc(x, w, b, wo, io, **kw)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        ops.router_noalloc(x, w, b, wo, io, **kw)
    x2, _, _ = _inputs(t, h, e, seed=6)
    x.copy_(x2)
    wo.zero_()
    g.replay()
    torch.cuda.synchronize()
    ref_w, ref_i = ops.router(x, w, b, **kw)
    assert torch.equal(io, ref_i) and torch.equal(wo, ref_w)
    del g
