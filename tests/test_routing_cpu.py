"""Router variants without a GPU: host-side validation of mosaic_route_ext and
the module mirrors' contracts (HashRouter, HashMoELayer, scoring_func)."""
from __future__ import annotations

import ctypes

import pytest
import torch

from mosaic_b200 import _capi as C
from mosaic_b200 import ops

FAKE = 1 << 20  # a 256-aligned non-null address; nothing is launched in these tests


def _ext(**kw):
    e = C.RouteExtC()
    for k, v in kw.items():
        setattr(e, k, v)
    return e


def _router_ext(ext, top_k=4, T=4, E=32, x=FAKE):
    return C.lib().mosaic_router_ext(ctypes.byref(ext), x, FAKE, None, T, 512, E, top_k, 1, 1, 1.0, 1, FAKE, FAKE,
                                     FAKE, 1 << 30, None)


def test_score_enum_matches_header():
    text = (C.LIB_PATH.parents[1] / "include" / "mosaic_moe.h").read_text()
    for name, code in (("SIGMOID", 0), ("SQRTSOFTPLUS", 1), ("SOFTMAX", 2)):
        assert f"MOSAIC_SCORE_{name} = {code}" in text
        assert getattr(C, f"MOSAIC_SCORE_{name}") == code


def test_route_ext_struct_layout():
    # int32 x4, int64, two pointers: 40 bytes on LP64, table_rows at 16
    assert ctypes.sizeof(C.RouteExtC) == 40
    assert C.RouteExtC.table_rows.offset == 16 and C.RouteExtC.tid2eid.offset == 24


@pytest.mark.parametrize("ext,status", [
    (dict(score_func=3), C.MOSAIC_ERR_UNSUPPORTED),
    (dict(score_func=-1), C.MOSAIC_ERR_UNSUPPORTED),
    (dict(hash=2), C.MOSAIC_ERR_SHAPE),
    (dict(reserved=1), C.MOSAIC_ERR_SHAPE),
    (dict(hash=1, layer_idx=-1), C.MOSAIC_ERR_SHAPE),        # salted hash: negative layer
    (dict(hash=1), C.MOSAIC_ERR_SHAPE),                      # salted hash with top_k 4
    (dict(hash=1, tid2eid=FAKE, table_rows=0), C.MOSAIC_ERR_SHAPE),
    (dict(hash=1, tid2eid=FAKE + 2, table_rows=10), C.MOSAIC_ERR_ALIGN),
    (dict(hash=1, tid2eid=FAKE, table_rows=10, token_ids=FAKE + 4), C.MOSAIC_ERR_ALIGN),
])
def test_router_ext_validation_before_launch(ext, status):
    assert _router_ext(_ext(**ext)) == status


def test_router_ext_router_checks_still_apply():
    # a table-routed call still needs the router's shapes and alignment
    assert _router_ext(_ext(hash=1, tid2eid=FAKE, table_rows=10), top_k=9) == C.MOSAIC_ERR_SHAPE
    assert _router_ext(_ext(score_func=1), x=FAKE + 4) == C.MOSAIC_ERR_ALIGN
    # the salted hash reads no x / weight but still checks E and T
    assert _router_ext(_ext(hash=1), top_k=1, E=257) == C.MOSAIC_ERR_SHAPE
    assert _router_ext(_ext(hash=1), top_k=1, T=0) == C.MOSAIC_ERR_SHAPE


def test_forward_ext_validation_before_launch():
    d = C.MoEDims(tokens=8, hidden=512, inter=256, n_experts=32, top_k=4, n_group=1, topk_group=1, act_mode=0,
                  norm_topk_prob=1, has_shared=1, route_scale=1.5, swiglu_limit=0.0)
    bank = C.ExpertBankC(FAKE, FAKE, FAKE, FAKE)
    lib = C.lib()

    def call(ext, rw=FAKE):
        return lib.mosaic_moe_forward_ext(ctypes.byref(d), ctypes.byref(ext), FAKE, rw, None, ctypes.byref(bank),
                                          FAKE, FAKE, FAKE, FAKE, 1 << 30, None)

    assert call(_ext(score_func=7)) == C.MOSAIC_ERR_UNSUPPORTED
    assert call(_ext(hash=1)) == C.MOSAIC_ERR_SHAPE  # salted hash needs top_k 1
    assert call(_ext(score_func=1), rw=None) == C.MOSAIC_ERR_SHAPE  # score routing needs the router weight


def test_scoring_func_names():
    from mosaic_b200 import MoEConfig

    for sf in ("sigmoid", "sqrtsoftplus", "softmax"):
        MoEConfig(scoring_func=sf).validate()
        assert ops.score_func_code(sf) == C.SCORE_FUNCS[sf]
    with pytest.raises(ValueError, match="unknown scoring_func"):
        MoEConfig(scoring_func="tanh").validate()


def test_hash_table_conversion():
    t = ops.hash_table(torch.tensor([3, 1, 2]), "cpu")
    assert t.dtype == torch.int32 and t.shape == (3, 1)
    t = ops.hash_table(torch.arange(12, dtype=torch.int64).view(4, 3), "cpu")
    assert t.shape == (4, 3) and t.is_contiguous()
    with pytest.raises(ValueError):
        ops.hash_table(torch.tensor([2 ** 33]), "cpu")
    with pytest.raises(ValueError):
        ops.hash_table(torch.zeros(4, 2), "cpu")


def test_hash_router_contracts(monkeypatch):
    """No table under the exact target raises ExactContractError (layers.py:177-179);
    a table id outside [0, E) raises before anything is launched."""
    from mosaic_b200 import ExactContractError, HashRouter, MoEConfig

    cfg = MoEConfig(hidden_size=256, n_routed_experts=8, num_experts_per_tok=2, n_group=1, topk_group=1,
                    scoring_func="sqrtsoftplus", routed_scaling_factor=1.5)
    r = HashRouter(cfg, 2)
    monkeypatch.setenv("MOSAICVM_EXACT_TARGET", "1")
    with pytest.raises(ExactContractError):
        r(torch.zeros(3, 256))
    r.tid2eid = torch.tensor([[0, 8], [1, 2]], dtype=torch.int32)
    with pytest.raises(IndexError):
        r(torch.zeros(3, 256))


def test_hash_moe_layer_mirrors_reference_attributes():
    from mosaic_b200 import HashMoELayer, MoEConfig

    cfg = MoEConfig(hidden_size=256, moe_intermediate_size=128, n_routed_experts=8, num_experts_per_tok=2,
                    n_group=1, topk_group=1, scoring_func="sqrtsoftplus")
    layer = HashMoELayer(cfg, 1)
    assert layer.router is None and layer.hash_router.layer_idx == 1
    assert layer.hash_router.weight.shape == (8, 256) and layer.hash_router.tid2eid is None
    with pytest.raises(NotImplementedError):
        layer(torch.zeros(1, 2, 256))
