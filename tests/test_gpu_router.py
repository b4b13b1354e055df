"""GPU router against the oracle router.

Bar: expert indices (and their descending order) bit-exact for every token
whose selection is decidable in fp32 (oracle.router.route_ties); tokens with
only an ORDER tie are compared as sets; weights within rtol 1e-5.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle.router import route, route_ties
from tests.golden.recipes import GATE_CASES, make_gate_case

pytestmark = pytest.mark.gpu
GOLD = Path(__file__).parent / "golden"


@pytest.fixture(scope="module")
def ops():
    from mosaic_b200 import ops as o

    return o


def _check(ops, x, wt, bias, k, ng, tg, scale, max_ties=None):
    w_ref, i_ref = route(x, wt, bias, top_k=k, n_group=ng, topk_group=tg, route_scale=scale)
    w, idx = ops.router(x.cuda(), wt.cuda(), bias.cuda(), top_k=k, n_group=ng, topk_group=tg, route_scale=scale)
    idx = idx.cpu().numpy()
    w = w.cpu().numpy()
    sel_tie, order_tie = route_ties(x, wt, bias, top_k=k, n_group=ng, topk_group=tg)
    ir = i_ref.numpy()
    for t in range(x.shape[0]):
        if sel_tie[t]:
            continue
        if order_tie[t]:
            assert sorted(idx[t]) == sorted(ir[t]), t
        else:
            assert np.array_equal(idx[t], ir[t]), (t, idx[t], ir[t])
            np.testing.assert_allclose(w[t], w_ref.numpy()[t], rtol=1e-5, atol=1e-7)
    if max_ties is not None:
        assert sel_tie.sum() <= max_ties
    return sel_tie.sum()


@pytest.mark.parametrize("name", list(GATE_CASES))
def test_router_matches_reference_gate_golden(ops, name):
    gold = np.load(GOLD / "router.npz")
    t, h, e, k, scale = GATE_CASES[name]
    x, wt, bias = make_gate_case(t, h, e, seed=77 + e)
    w, idx = ops.router(x.cuda(), wt.cuda(), bias.cuda(), top_k=k, route_scale=scale)
    sel_tie, order_tie = route_ties(x, wt, bias, top_k=k)
    gi = gold[name + "_idx"]
    got = idx.cpu().numpy()
    for ti in range(t):
        if sel_tie[ti]:
            continue
        if order_tie[ti]:
            assert sorted(got[ti]) == sorted(gi[ti])
        else:
            assert np.array_equal(got[ti], gi[ti])
            np.testing.assert_allclose(w.cpu().numpy()[ti], gold[name + "_weights"][ti], rtol=1e-5)


@pytest.mark.parametrize("t", [1, 8, 32, 128])
def test_router_v3_decode_group_limited(ops, t):
    x, wt, bias = make_gate_case(t, 7168, 256, seed=1000 + t)
    _check(ops, x, wt, bias, 8, 8, 4, 2.5, max_ties=max(1, t // 32))


def test_router_small_config(ops):
    x, wt, bias = make_gate_case(64, 512, 32, seed=4)
    _check(ops, x, wt, bias, 4, 4, 2, 2.5, max_ties=2)


def test_router_prefill_size(ops):
    x, wt, bias = make_gate_case(2048, 7168, 256, seed=9)
    n = _check(ops, x, wt, bias, 8, 8, 4, 2.5)
    assert n <= 20


def test_router_deterministic(ops):
    x, wt, bias = make_gate_case(128, 7168, 256, seed=5)
    a = ops.router(x.cuda(), wt.cuda(), bias.cuda(), top_k=8, n_group=8, topk_group=4, route_scale=2.5)
    b = ops.router(x.cuda(), wt.cuda(), bias.cuda(), top_k=8, n_group=8, topk_group=4, route_scale=2.5)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])


def test_router_rejects_bad_shapes(ops):
    x = torch.zeros(4, 256, dtype=torch.bfloat16, device="cuda")
    wt = torch.zeros(32, 256, device="cuda")
    with pytest.raises(ValueError):
        ops.router(x, wt, None, top_k=4, n_group=3, topk_group=1)  # 32 % 3 != 0
    with pytest.raises(ValueError):
        ops.router(x, wt, None, top_k=9)


@pytest.mark.parametrize("e", [250, 100, 36, 33, 256])
def test_router_ragged_expert_counts(ops, e):
    """Expert counts that are not a multiple of 4 or of the per-lane width take
    the scalar partial-sum path; all must match the oracle."""
    x, wt, bias = make_gate_case(24, 1024, e, seed=300 + e)
    _check(ops, x, wt, bias, 4, 1, 1, 1.0, max_ties=1)


@pytest.mark.parametrize("t", [4736, 8192])
def test_router_tensor_core_logits(ops, t):
    """Large batches use the tensor-core logits with W split into three bf16 parts
    by a separate pass (x . (hi + mid + lo), fp32 accumulation; 2 and 1 K splits
    here): the same bar as the FMA kernels, ids exact outside fp32 ties."""
    x, wt, bias = make_gate_case(t, 7168, 256, seed=7000 + t)
    _check(ops, x, wt, bias, 8, 8, 4, 2.5, max_ties=max(1, t // 32))


@pytest.mark.parametrize("t", [1, 7, 129, 300, 1000, 2048])
def test_router_tensor_core_split_k(ops, t):
    """Smaller batches split K over up to 64 CTAs per 128 x 128 tile.  T <= 128
    (at most two K slices per CTA) also split W inside the kernel (the swizzled
    part tiles written by the converter warps); the top-k pass adds the splits
    (8 warps per token from 16 splits up)."""
    x, wt, bias = make_gate_case(t, 7168, 256, seed=7100 + t)
    _check(ops, x, wt, bias, 8, 8, 4, 2.5, max_ties=max(1, t // 32))


@pytest.mark.parametrize("e", [16, 48, 144, 208])
def test_router_tensor_core_expert_tiles(ops, e):
    """Expert counts that leave a partial 128-expert tile (N = E mod 128) or a
    single small one; rows past E read as zeros."""
    x, wt, bias = make_gate_case(200, 1024, e, seed=7200 + e)
    _check(ops, x, wt, bias, 4, 1, 1, 1.0, max_ties=1)


def test_router_fma_path_hidden_not_multiple_of_64(ops):
    """H = 992 (a multiple of 32, not of 64) keeps the split-K FMA kernels."""
    x, wt, bias = make_gate_case(128, 992, 256, seed=7300)
    _check(ops, x, wt, bias, 8, 8, 4, 2.5, max_ties=4)
