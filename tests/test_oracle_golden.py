"""The CPU oracle against golden vectors recorded from the reference itself.

Fixtures come from ``tests/golden/gen_golden.py`` (which imports the
reference's ``pack_mxfp4_nk``, ``act_quant_ref``,
``reference_fp4_linear_source_semantics``, ``dequant_fp4``, the vendored
sigmoid ``Gate``, ``grouped_expert_forward`` and ``SharedExpertMLP``), plus the
reference's own known-answer tests restated (``tests/test_moe_layout.py``,
``tests/test_emit_tiles.py``, ``tests/test_mxfp4.py``).
"""
from __future__ import annotations

import hashlib
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import formats as fm
from oracle.layout import emit_tiles, layout_assignments, moe_rows
from oracle.moe import moe_layer
from oracle.router import route, route_ties
from tests.golden.recipes import GATE_CASES, MOE_CASES, make_gate_case, make_moe_case

GOLD = Path(__file__).parent / "golden"


@pytest.fixture(scope="module")
def fmt():
    return np.load(GOLD / "formats.npz")


def test_e2m1_lut_locked():
    assert fm.E2M1_LUT == (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
                           -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0)


def test_pack_matches_reference(fmt):
    p, s = fm.pack_mxfp4_nk(fmt["pack_w"])
    assert np.array_equal(p, fmt["pack_packed"])
    assert np.array_equal(s, fmt["pack_scale"])


def test_pack_edges_match_reference(fmt):
    p, s = fm.pack_mxfp4_nk(fmt["edge_w"])
    assert np.array_equal(p, fmt["edge_packed"])
    assert np.array_equal(s, fmt["edge_scale"])
    deq = fm.dequant_fp4(p, s)
    assert np.array_equal(deq.view(np.uint32), fmt["edge_dequant"].view(np.uint32))


def test_pack_roundtrip_codes(fmt):
    p, s = fm.pack_mxfp4_nk(fmt["pack_w"])
    p2, s2 = fm.pack_mxfp4_nk(fm.dequant_fp4(p, s))
    assert np.array_equal(p, p2) and np.array_equal(s, s2)


def test_scale_127_is_identity():
    codes = np.arange(32, dtype=np.uint8) % 16
    packed = (codes[0::2] | (codes[1::2] << 4)).reshape(1, 16)
    deq = fm.dequant_fp4(packed, np.array([[127]], dtype=np.uint8))
    assert np.array_equal(deq[0], np.array(fm.E2M1_LUT * 2, dtype=np.float32))


@pytest.mark.parametrize("key", ["act", "actb"])
def test_act_quant_matches_reference(fmt, key):
    q, s = fm.act_quant_ref(fmt[key + "_x"])
    assert np.array_equal(s.view(np.uint32), fmt[key + "_s"].view(np.uint32))
    assert np.array_equal(q, fmt[key + "_q"])


@pytest.mark.parametrize("key", ["lin_a", "lin_b", "lin_c"])
def test_fp4_linear_matches_reference(fmt, key):
    q, s = fm.act_quant_ref(fmt[key + "_x"])
    y = fm.to_bf16(fm.fp4_linear_source(q, s, fmt[key + "_packed"], fmt[key + "_scale"]))
    assert np.array_equal(y.view(np.uint32), fmt[key + "_y"].view(np.uint32))


@pytest.mark.parametrize("name", list(GATE_CASES))
def test_router_degenerate_equals_reference_gate(name):
    gold = np.load(GOLD / "router.npz")
    t, h, e, k, scale = GATE_CASES[name]
    x, wt, bias = make_gate_case(t, h, e, seed=77 + e)
    sha = hashlib.sha256()
    for a in (x.float().numpy(), wt.numpy(), bias.numpy()):
        sha.update(np.ascontiguousarray(a).tobytes())
    assert sha.hexdigest().encode() == gold[name + "_sha"].tobytes()
    for n_group, topk_group in ((1, 1), (8 if e >= 256 else 4, 8 if e >= 256 else 4)):
        w, idx = route(x, wt, bias, top_k=k, n_group=n_group, topk_group=topk_group, route_scale=scale)
        assert np.array_equal(idx.numpy(), gold[name + "_idx"])
        np.testing.assert_allclose(w.numpy(), gold[name + "_weights"], rtol=2e-7, atol=0)


def test_router_group_limit_restricts_groups():
    x, wt, bias = make_gate_case(32, 512, 32, seed=5)
    w, idx = route(x, wt, bias, top_k=4, n_group=4, topk_group=2, route_scale=2.5)
    groups = idx.numpy() // 8
    assert all(len(set(r)) <= 2 for r in groups.tolist())
    np.testing.assert_allclose(w.sum(-1).numpy(), 2.5, rtol=1e-6)
    sel_tie, _ = route_ties(x, wt, bias, top_k=4, n_group=4, topk_group=2)
    assert sel_tie.sum() <= 2


def test_layout_known_answer():
    sorted_ids, perm, offsets, counts = layout_assignments([3, 0, 3, 1], 4)
    assert counts.tolist() == [1, 1, 0, 2]
    assert offsets.tolist() == [0, 1, 2, 2, 4]
    assert perm.tolist() == [1, 3, 0, 2]
    assert sorted_ids.tolist() == [0, 1, 3, 3]


@pytest.mark.parametrize("block_m", [1, 8, 16])
def test_emit_tiles_known_answer(block_m):
    counts = [0, 1, block_m - 1, block_m, block_m + 1, 3 * block_m + 2]
    exp = []
    for e, c in enumerate(counts):
        for t in range((c + block_m - 1) // block_m):
            exp.append((e, t * block_m, min(block_m, c - t * block_m)))
    assert emit_tiles(counts, block_m) == exp
    assert emit_tiles([0] * 5, block_m) == []


def test_moe_rows_bijection():
    rng = np.random.default_rng(0)
    idx = np.stack([rng.permutation(16)[:4] for _ in range(10)])
    counts, offsets, row_of, row_token, row_slot = moe_rows(idx, 16)
    r = row_of.reshape(-1)
    assert sorted(r.tolist()) == list(range(40))
    assert np.array_equal(row_token[r], np.repeat(np.arange(10), 4))
    assert np.array_equal(row_slot[r], np.tile(np.arange(4), 10))
    assert counts[-1] == 10 and offsets[-1] == 50


def _bank(case):
    e = case["cfg"]["E"]
    gu = [fm.pack_mxfp4_nk(case["w_gu"][i]) for i in range(e + 1)]
    dn = [fm.pack_mxfp4_nk(case["w_dn"][i]) for i in range(e + 1)]
    return {"gu_packed": np.stack([p for p, _ in gu[:e]]), "gu_scale": np.stack([s for _, s in gu[:e]]),
            "dn_packed": np.stack([p for p, _ in dn[:e]]), "dn_scale": np.stack([s for _, s in dn[:e]]),
            "sh_gu_packed": gu[e][0], "sh_gu_scale": gu[e][1],
            "sh_dn_packed": dn[e][0], "sh_dn_scale": dn[e][1]}, gu, dn


@pytest.mark.parametrize("name", list(MOE_CASES))
def test_moe_bf16_matches_reference_grouped_forward(name):
    gold = np.load(GOLD / "moe.npz")
    case = make_moe_case(**MOE_CASES[name])
    bank, gu, dn = _bank(case)
    sha = hashlib.sha256()
    for a in (np.stack([p for p, _ in gu]), np.stack([s for _, s in gu]),
              np.stack([p for p, _ in dn]), np.stack([s for _, s in dn])):
        sha.update(np.ascontiguousarray(a).tobytes())
    assert sha.hexdigest().encode() == gold[name + "_sha"].tobytes()
    w = gold[name + "_weights"]
    idx = gold[name + "_idx"]
    y, _, routed, shared = moe_layer(case["x"], w, idx, bank, mode="bf16",
                                     swiglu_limit=case["cfg"]["swiglu_limit"], return_parts=True)
    for got, key in ((routed, "routed"), (shared, "shared"), (y, "y")):
        ref = gold[name + "_" + key]
        rel = np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30)
        assert rel < 2e-3, (key, rel)
        # bf16 results: nearly every element identical, the rest one ulp apart
        diff = np.abs(got.view(np.int32) - ref.view(np.int32)) >> 16
        assert (diff <= 1).mean() > 0.995, key
