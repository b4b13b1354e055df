"""Router variants on the GPU against the reference's recorded outputs and the oracle.

Bars: expert ids bit-exact (descending order included) for every token whose
selection is decidable in fp32 (oracle.router.route_ties with the score
function's derivative), order ties compared as sets; weights within rtol 1e-5
(the GPU's split-K logits differ from torch's CPU GEMM by rounding only);
table-less hash ids and weights bit-exact; hash-routed and sqrtsoftplus MoE
layers within the layer tolerance of the sigmoid layer (bf16 5e-3, fp8 2e-3).
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle.moe import moe_layer
from oracle.router import hash_route, route, route_ties
from tests.golden.recipes import (MOE_CASES, ROUTING_CASES, SALTED_CASES, make_gate_case, make_hash_case,
                                  make_moe_case, salted_token_ids)
from tests.helpers import gpu_bank, pack_case, rel_l2
from tests.test_oracle_routing import case_inputs

pytestmark = pytest.mark.gpu
GOLD = Path(__file__).parent / "golden"
TOL = {"bf16": 5e-3, "fp8": 2e-3}


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLD / "routing.npz")


def _compare(idx, w, ref_idx, ref_w, sel_tie, order_tie):
    for t in range(idx.shape[0]):
        if sel_tie[t]:
            continue
        if order_tie[t]:
            assert sorted(idx[t]) == sorted(ref_idx[t]), t
        else:
            assert np.array_equal(idx[t], ref_idx[t]), (t, idx[t], ref_idx[t])
            np.testing.assert_allclose(w[t], ref_w[t], rtol=1e-5, atol=1e-7)


@pytest.mark.parametrize("name", list(ROUTING_CASES))
def test_routing_matches_reference_golden(gold, name):
    from mosaic_b200 import ops

    c = ROUTING_CASES[name]
    x, wt, bias, table, tok = case_inputs(name)
    if table is None:
        norm = True if c["src"] == "router" else c["score"] != "softmax"
        w, idx = ops.router(x.cuda(), wt.cuda(), bias.cuda(), top_k=c["k"], route_scale=c["scale"],
                            norm_topk_prob=norm, score_func=c["score"])
        sel_tie, order_tie = route_ties(x, wt, bias, top_k=c["k"], score_func=c["score"])
    else:
        w, idx = ops.hash_router(x.cuda(), wt.cuda(), table.cuda(), tok.cuda(), n_experts=c["E"], layer_idx=3,
                                 score_func=c["score"], route_scale=c["scale"])
        sel_tie = order_tie = np.zeros(c["T"], dtype=bool)
    torch.cuda.synchronize()
    _compare(idx.cpu().numpy(), w.cpu().numpy(), gold[name + "_idx"], gold[name + "_weights"], sel_tie, order_tie)


@pytest.mark.parametrize("e,layer_idx", SALTED_CASES)
def test_salted_hash_bit_exact(gold, e, layer_idx):
    from mosaic_b200 import ops

    tok = salted_token_ids()
    x = torch.zeros(tok.numel(), 256, dtype=torch.bfloat16, device="cuda")
    w, idx = ops.hash_router(x, None, None, tok.cuda(), n_experts=e, layer_idx=layer_idx, route_scale=1.5)
    assert np.array_equal(idx.cpu().numpy(), gold[f"salted_{e}_{layer_idx}_idx"])
    assert np.array_equal(w.cpu().numpy(), gold[f"salted_{e}_{layer_idx}_weights"])
    # no token ids: 0..T-1
    w, idx = ops.hash_router(x[:64], None, None, None, n_experts=e, layer_idx=layer_idx, route_scale=1.5)
    assert np.array_equal(idx.cpu().numpy(), gold[f"salted_{e}_{layer_idx}_idx"][-64:])


@pytest.mark.parametrize("score", ["sqrtsoftplus", "softmax"])
@pytest.mark.parametrize("t", [1, 32, 128, 2048])
def test_group_limited_variants_v3(score, t):
    """The V3 shape (E 256, 8 groups, top-4 groups, top-8) with the other score functions."""
    from mosaic_b200 import ops

    x, wt, bias = make_gate_case(t, 7168, 256, seed=3000 + t)
    w_ref, i_ref = route(x, wt, bias, top_k=8, n_group=8, topk_group=4, route_scale=2.5, score_func=score)
    w, idx = ops.router(x.cuda(), wt.cuda(), bias.cuda(), top_k=8, n_group=8, topk_group=4, route_scale=2.5,
                        score_func=score)
    sel_tie, order_tie = route_ties(x, wt, bias, top_k=8, n_group=8, topk_group=4, score_func=score)
    assert sel_tie.sum() <= max(1, t // 32)
    _compare(idx.cpu().numpy(), w.cpu().numpy(), i_ref.numpy(), w_ref.numpy(), sel_tie, order_tie)


def test_hash_table_v4_prefill():
    """V4 hash layer at prefill size: vocabulary 129280, E 256, k 6, T 4096."""
    from mosaic_b200 import ops

    x, wt, table, tok = make_hash_case(4096, 4096, 256, 6, 129280, seed=41)
    w_ref, i_ref = hash_route(x, wt, table, tok, n_experts=256, score_func="sqrtsoftplus", route_scale=1.5)
    w, idx = ops.hash_router(x.cuda(), wt.cuda(), table.cuda(), tok.cuda(), n_experts=256,
                             score_func="sqrtsoftplus", route_scale=1.5)
    assert torch.equal(idx.cpu(), i_ref)
    np.testing.assert_allclose(w.cpu().numpy(), w_ref.numpy(), rtol=1e-5, atol=1e-7)


def test_hash_table_id_out_of_range_sets_error_word():
    """An id outside [0, E) in the table is a device-side error (MOSAIC_ERR_RANGE), read
    back through mosaic_read_error; the call itself returns normally."""
    from mosaic_b200 import _capi as C
    from mosaic_b200 import ops

    t, h, e = 8, 512, 32
    x, wt, table, tok = make_hash_case(t, h, e, 2, 20, seed=5, in_table=True)
    table[int(tok[3]), 1] = e  # one bad entry, on a row token 3 reads
    table = table.cuda()
    ext = ops.route_ext("sqrtsoftplus", tid2eid=table, token_ids=tok.cuda(), hash_routing=True)
    lib = C.lib()
    ws = torch.empty(lib.mosaic_router_workspace_bytes(t, h, e), dtype=torch.uint8, device="cuda")
    ws.zero_()
    w = torch.empty(t, 2, device="cuda")
    idx = torch.empty(t, 2, dtype=torch.int64, device="cuda")
    xg, wg = x.cuda(), wt.cuda()
    tokg = tok.cuda()
    ext.token_ids = tokg.data_ptr()
    st = lib.mosaic_router_ext(ctypes.byref(ext), ops._ptr(xg), ops._ptr(wg), None, t, h, e, 2, 1, 1, 1.5, 1,
                               ops._ptr(w), ops._ptr(idx), ops._ptr(ws), ws.numel(), ops._stream())
    C.check(st, "mosaic_router_ext")
    assert ops.read_error(ws) == C.MOSAIC_ERR_RANGE
    assert ops.read_error(ws) == 0  # reset


@pytest.fixture(scope="module")
def moe_s():
    case = make_moe_case(**MOE_CASES["S"])
    obank, full = pack_case(case)
    return case, obank, full


def _cfg(c, mode, score):
    from mosaic_b200 import MoEConfig

    return MoEConfig(hidden_size=c["H"], moe_intermediate_size=c["I"], n_routed_experts=c["E"],
                     num_experts_per_tok=c["k"], n_group=c["n_group"], topk_group=c["topk_group"],
                     routed_scaling_factor=c["scale"], swiglu_limit=c["swiglu_limit"], act_mode=mode,
                     scoring_func=score)


@pytest.mark.parametrize("mode", ["bf16", "fp8"])
@pytest.mark.parametrize("score", ["sqrtsoftplus", "softmax"])
def test_moe_layer_score_functions(moe_s, mode, score):
    from mosaic_b200 import MoELayer, ops

    case, obank, full = moe_s
    c = case["cfg"]
    layer = MoELayer(_cfg(c, mode, score), gpu_bank(full))
    layer.router.weight.data = case["router_w"].cuda()
    layer.router.e_score_correction_bias.data = case["bias"].cuda()
    x = case["x"].cuda()
    y = layer(x)
    torch.cuda.synchronize()
    assert ops.read_error(layer.workspace(x.shape[0], x.device)) == 0
    w_ref, i_ref = route(case["x"], case["router_w"], case["bias"], top_k=c["k"], n_group=c["n_group"],
                         topk_group=c["topk_group"], route_scale=c["scale"], score_func=score)
    sel_tie, _ = route_ties(case["x"], case["router_w"], case["bias"], top_k=c["k"], n_group=c["n_group"],
                            topk_group=c["topk_group"], score_func=score)
    assert not sel_tie.any()
    assert torch.equal(layer.last_idx.cpu(), i_ref)
    w = layer.last_weights.cpu()
    np.testing.assert_allclose(w.numpy(), w_ref.numpy(), rtol=1e-5, atol=1e-7)
    ref = moe_layer(case["x"], w, i_ref, obank, mode=mode, swiglu_limit=c["swiglu_limit"])
    assert rel_l2(y.float().cpu().numpy(), ref) <= TOL[mode]


@pytest.mark.parametrize("mode", ["bf16", "fp8"])
@pytest.mark.parametrize("kind", ["table", "table_1d", "salted"])
def test_hash_moe_layer(moe_s, mode, kind, monkeypatch):
    """HashMoELayer (layers.py:376-405): table or salted ids, shared expert included."""
    from mosaic_b200 import HashMoELayer, ops

    case, obank, full = moe_s
    c = case["cfg"]
    t = c["T"]
    cfg = _cfg(c, mode, "sqrtsoftplus")
    if kind == "salted":
        monkeypatch.setenv("MOSAICVM_EXACT_TARGET", "0")
    layer = HashMoELayer(cfg, 2, gpu_bank(full))
    layer.hash_router.weight.data = case["router_w"].cuda()
    _, _, table, tok = make_hash_case(t, c["H"], c["E"], None if kind == "table_1d" else c["k"], 300, seed=8)
    if kind != "salted":
        layer.hash_router.tid2eid = table
    x = case["x"].cuda().view(1, t, -1)
    y = layer(x, tok.cuda().view(1, t))
    torch.cuda.synchronize()
    assert y.shape == x.shape
    w_ref, i_ref = hash_route(case["x"], case["router_w"], None if kind == "salted" else table, tok,
                              n_experts=c["E"], layer_idx=2, score_func="sqrtsoftplus", route_scale=c["scale"])
    assert torch.equal(layer.last_idx.cpu(), i_ref)
    w = layer.last_weights.cpu()
    np.testing.assert_allclose(w.numpy(), w_ref.numpy(), rtol=1e-5, atol=1e-7)
    dims = cfg.dims(t, True)
    dims.top_k = i_ref.shape[1]
    assert ops.read_error(layer._ws.get(dims, x.device)) == 0
    ref = moe_layer(case["x"], w, i_ref, obank, mode=mode, swiglu_limit=c["swiglu_limit"])
    assert rel_l2(y.view(t, -1).float().cpu().numpy(), ref) <= TOL[mode]
