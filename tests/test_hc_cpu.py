"""Hyper-connection + RMSNorm oracle against vectors recorded from the reference
(``HyperConnections.pre/post``, ``RMSNorm``, ``act_quant_ref``; mosaicvm/model/
layers.py:19-29, 222-271), and the C ABI's host-side validation (no GPU)."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from mosaic_b200 import _capi as C
from oracle.formats import act_quant_ref
from oracle.hc import hc_post, hc_pre, rms_norm
from tests.golden.recipes import HC_ORACLE_CASES, make_hc_case

GOLD = Path(__file__).parent / "golden"


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLD / "hc.npz")


@pytest.mark.parametrize("name", list(HC_ORACLE_CASES))
def test_oracle_hc_matches_reference(gold, name):
    b, s, hc, d, iters, seed = HC_ORACLE_CASES[name]
    x, fn, base, scale, norm_w, y = make_hc_case(b, s, hc, d, seed)
    y_pre, post, comb = hc_pre(x, fn, base, scale, iters=iters, eps=1e-6, norm_eps=1e-6)
    assert np.array_equal(y_pre.float().numpy(), gold[name + "_y_pre"])
    assert np.array_equal(post.numpy(), gold[name + "_post"])
    assert np.array_equal(comb.numpy(), gold[name + "_comb"])
    y_norm = rms_norm(y_pre, norm_w, 1e-6)
    assert np.array_equal(y_norm.float().numpy(), gold[name + "_y_norm"])
    q, qs = act_quant_ref(y_norm.float().numpy().reshape(-1, d))
    assert np.array_equal(q, gold[name + "_q"]) and np.array_equal(qs, gold[name + "_qs"])
    out = hc_post(y, x, post, comb)
    assert np.array_equal(out.float().numpy(), gold[name + "_out_post"])


def test_hc_validation_before_launch():
    lib = C.lib()
    f = 1 << 20
    # D not a multiple of 128, hc out of range, iters 0, q without its scale, misaligned x
    def call(*a):
        return lib.mosaic_hc_pre_norm(*a, f, 1 << 30, None)

    assert call(f, f, f, f, f, 4, 200, 4, 20, 1e-6, 1e-6, f, f, f, None, None) == 1
    assert call(f, f, f, f, f, 4, 256, 5, 20, 1e-6, 1e-6, f, f, f, None, None) == 1
    assert call(f, f, f, f, f, 4, 256, 4, 0, 1e-6, 1e-6, f, f, f, None, None) == 1
    assert call(f, f, f, f, f, 4, 256, 4, 20, 1e-6, 1e-6, f, f, f, f, None) == 1
    assert call(f + 8, f, f, f, f, 4, 256, 4, 20, 1e-6, 1e-6, f, f, f, None, None) == 3
    assert lib.mosaic_hc_pre_norm(f, f, f, f, f, 4, 256, 4, 20, 1e-6, 1e-6, f, f, f, None, None, None, 0,
                                  None) == 1  # no workspace
    assert lib.mosaic_hc_pre_norm_workspace_bytes(4, 200, 4) == 0
    assert lib.mosaic_hc_post(f, f, f, f, 4, 12, 4, f, None) == 1
    assert lib.mosaic_hc_post(f, f + 2, f, f, 4, 256, 4, f, None) == 3


def test_hc_module_contracts():
    from mosaic_b200.hc import HyperConnections, RMSNorm, ffn_pre_norm

    hc = HyperConnections(256)
    assert hc.fn.shape == (24, 1024) and hc.base.shape == (24,) and hc.scale.shape == (3,)
    with pytest.raises(ValueError, match="bf16"):
        hc.pre(torch.zeros(1, 2, 4, 256))
    with pytest.raises(ValueError, match="CUDA"):
        hc.pre(torch.zeros(1, 2, 4, 256, dtype=torch.bfloat16))
    with pytest.raises(TypeError, match="bf16"):
        RMSNorm(256)(torch.zeros(2, 256))
    with pytest.raises(ValueError, match="CUDA"):
        RMSNorm(256)(torch.zeros(2, 256, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="width 256"):
        RMSNorm(256)(torch.zeros(2, 128, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="one epsilon"):
        ffn_pre_norm(torch.zeros(1, 2, 4, 256, dtype=torch.bfloat16), hc, RMSNorm(256, eps=1e-5))
