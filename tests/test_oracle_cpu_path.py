"""The CPU baseline's FP4 linear (reference VNNI kernel compiled from the
reference source, and the plain-C port) equals the oracle / golden vectors bit for bit."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from oracle import formats as fm
from oracle.cpu_path import PORT_LIB, VNNI_LIB, FP4LinearCPU, host_has_avx_vnni

GOLD = Path(__file__).parent / "golden"

KINDS = []
if PORT_LIB.exists():
    KINDS.append("port")
if VNNI_LIB.exists() and host_has_avx_vnni():
    KINDS.append("reference")


@pytest.mark.skipif(not KINDS, reason="oracle C checkers not built (python oracle/build.py)")
@pytest.mark.parametrize("kind", KINDS)
@pytest.mark.parametrize("key", ["lin_a", "lin_b", "lin_c"])
def test_cpu_linear_matches_reference_golden(kind, key):
    g = np.load(GOLD / "formats.npz")
    lin = FP4LinearCPU(kind)
    q, s = fm.act_quant_ref(g[key + "_x"])
    n = g[key + "_packed"].shape[0]
    if kind == "reference" and n % 8:
        pytest.skip("VNNI kernel needs N % 8 == 0")
    y = fm.to_bf16(lin(q, s, lin.prepare(g[key + "_packed"], g[key + "_scale"])))
    assert np.array_equal(y.view(np.uint32), g[key + "_y"].view(np.uint32))


@pytest.mark.skipif(not KINDS, reason="oracle C checkers not built")
@pytest.mark.parametrize("kind", KINDS)
def test_cpu_linear_matches_oracle_fp32(kind):
    rng = np.random.default_rng(0)
    w = rng.standard_normal((64, 512)).astype(np.float32) * 0.02
    x = rng.standard_normal((7, 512)).astype(np.float32)
    p, s = fm.pack_mxfp4_nk(w)
    q, sa = fm.act_quant_ref(fm.to_bf16(x))
    lin = FP4LinearCPU(kind)
    y = lin(q, sa, lin.prepare(p, s))
    ref = fm.fp4_linear_source(q, sa, p, s)
    assert np.array_equal(y.view(np.uint32), ref.view(np.uint32))


@pytest.mark.skipif(not PORT_LIB.exists(), reason="oracle C checkers not built")
def test_fast_oracle_layer_matches_numpy_oracle():
    """moe_layer(fast=True) (the C linears used at V3 sizes) against the numpy
    oracle pinned to the reference goldens: FP8 path bit-equal, bf16 path
    within fp32 summation-order noise."""
    import torch

    from oracle.moe import moe_layer
    from tests.golden.recipes import MOE_CASES, make_moe_case
    from tests.helpers import pack_case, rel_l2

    case = make_moe_case(**MOE_CASES["S"])
    obank, _ = pack_case(case)
    c = case["cfg"]
    for mode in ("fp8", "bf16"):
        a = moe_layer(case["x"], case["weights"], case["idx"], obank, mode=mode, swiglu_limit=c["swiglu_limit"])
        b = moe_layer(case["x"], case["weights"], case["idx"], obank, mode=mode, swiglu_limit=c["swiglu_limit"],
                      fast=True)
        if mode == "fp8":
            assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
        else:
            assert rel_l2(b, a) < 1e-3
    assert isinstance(case["x"], torch.Tensor)
