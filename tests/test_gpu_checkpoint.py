"""Checkpoint loader on the GPU: a small V4-contract checkpoint (two layers, the
first hash-routed) loads into resident MXFP4 banks byte for byte, and the loaded
layers match the oracle on the same tensors (routing bit-exact, layer output
within the bf16 / fp8 layer tolerances 5e-3 / 2e-3)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.moe import moe_layer
from oracle.router import hash_route, route, route_ties
from tests.ckpt_fixture import CKPT, expected_bank, make_checkpoint
from tests.helpers import rel_l2

pytestmark = pytest.mark.gpu
TOL = {"bf16": 5e-3, "fp8": 2e-3}


def _obank(arrs):
    gu_p, gu_s, dn_p, dn_s = arrs
    return {"gu_packed": gu_p[:-1], "gu_scale": gu_s[:-1], "dn_packed": dn_p[:-1], "dn_scale": dn_s[:-1],
            "sh_gu_packed": gu_p[-1], "sh_gu_scale": gu_s[-1], "sh_dn_packed": dn_p[-1], "sh_dn_scale": dn_s[-1]}


@pytest.fixture(scope="module")
def ckpt(tmp_path_factory):
    root = tmp_path_factory.mktemp("ckpt")
    return root, make_checkpoint(root, shards=2)


@pytest.mark.parametrize("mode", ["bf16", "fp8"])
def test_loaded_layers_match_oracle(ckpt, mode):
    from mosaic_b200 import HashMoELayer, MoELayer
    from mosaic_b200.checkpoint import ShardIndex, load_moe_layer, moe_config_from_checkpoint

    root, tensors = ckpt
    cfg, n_hash, _ = moe_config_from_checkpoint(root, act_mode=mode)
    idx = ShardIndex(root)
    t = 24
    g = torch.Generator().manual_seed(4)
    x = torch.randn(t, CKPT["H"], generator=g).to(torch.bfloat16)
    tok = torch.randint(-100, 400, (t,), generator=g)
    for li in range(CKPT["layers"]):
        layer = load_moe_layer(idx, li, cfg=cfg, num_hash_layers=n_hash, keep_packed=True)
        arrs = expected_bank(tensors, li)
        b = layer.bank
        for got, want in zip((b.gu_packed, b.gu_scale, b.dn_packed, b.dn_scale), arrs):
            assert np.array_equal(got.cpu().numpy(), want)
        pre = f"layers.{li}."
        wt = tensors[pre + "ffn.gate.weight"].float()
        if li < n_hash:
            assert isinstance(layer, HashMoELayer)
            y = layer(x.cuda().view(1, t, -1), tok.cuda()).view(t, -1)
            w_ref, i_ref = hash_route(x, wt, tensors[pre + "ffn.gate.tid2eid"], tok.numpy(), n_experts=CKPT["E"],
                                      score_func="sqrtsoftplus", route_scale=1.5)
        else:
            assert isinstance(layer, MoELayer) and layer.router is not None
            y = layer(x.cuda())
            bias = tensors[pre + "ffn.gate.bias"]
            assert torch.equal(layer.router.e_score_correction_bias.cpu(), bias.to(torch.bfloat16).float())
            w_ref, i_ref = route(x, wt, bias.to(torch.bfloat16).float(), top_k=CKPT["k"], route_scale=1.5,
                                 score_func="sqrtsoftplus")
            sel_tie, _ = route_ties(x, wt, bias, top_k=CKPT["k"], score_func="sqrtsoftplus")
            assert not sel_tie.any()
        torch.cuda.synchronize()
        assert torch.equal(layer.last_idx.cpu(), i_ref)
        w = layer.last_weights.cpu()
        np.testing.assert_allclose(w.numpy(), w_ref.numpy(), rtol=1e-5, atol=1e-7)
        ref = moe_layer(x, w, i_ref, _obank(arrs), mode=mode, swiglu_limit=10.0)
        assert rel_l2(y.float().cpu().numpy(), ref) <= TOL[mode]


def test_load_all_layers_shares_one_stager(ckpt):
    from mosaic_b200.checkpoint import load_moe_layers

    root, tensors = ckpt
    layers = load_moe_layers(root)
    assert len(layers) == CKPT["layers"]
    assert layers[0].hash_router.tid2eid.shape == (CKPT["vocab"], CKPT["k"])
    assert layers[0].bank.gu_packed is None  # reference-layout copies dropped by default


def test_non_mxfp4_shared_expert_is_refused(tmp_path):
    from mosaic_b200.checkpoint import load_moe_layer

    make_checkpoint(tmp_path, shared_format="bf16")
    with pytest.raises(NotImplementedError, match="shared expert stored as BF16"):
        load_moe_layer(tmp_path, 1)
