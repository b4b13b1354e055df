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


@pytest.mark.skipif(not KINDS, reason="oracle C checkers not built")
def test_cpu_layer_path_matches_the_fp8_oracle():
    """The whole-layer CPU baseline (router, every touched expert through the
    reference CPU kernel, shared expert, ordered combine) equals the FP8 oracle
    layer bit for bit and routes like the golden recipe."""
    import torch

    from oracle.cpu_path import LayerCPU
    from oracle.moe import moe_layer
    from tests.golden.recipes import MOE_CASES, make_moe_case
    from tests.helpers import pack_case

    case = make_moe_case(**MOE_CASES["S"])
    obank, _ = pack_case(case)
    c = case["cfg"]
    cpu = LayerCPU(obank)
    y, sec, (w, idx) = cpu.step(case["x"], case["router_w"], case["bias"], top_k=c["k"], n_group=c["n_group"],
                                topk_group=c["topk_group"], route_scale=c["scale"], limit=c["swiglu_limit"])
    assert torch.equal(idx, case["idx"]) and sec > 0
    ref = moe_layer(case["x"], w, idx, obank, mode="fp8", swiglu_limit=c["swiglu_limit"])
    assert np.array_equal(y.view(np.uint32), ref.view(np.uint32))


@pytest.mark.skipif(not KINDS, reason="oracle C checkers not built")
def test_vnni_operand_preparation_matches_the_layout():
    """The C preparation of the reference kernel's weight operands equals the
    numpy restatement of mosaicvm/bench/vnni_source.py:38-54."""
    from oracle.cpu_path import decode_e2m1

    rng = np.random.default_rng(3)
    p, s = fm.pack_mxfp4_nk(rng.standard_normal((64, 256)).astype(np.float32) * 0.02)
    lin = FP4LinearCPU(KINDS[-1])
    if lin.kind != "reference":
        pytest.skip("the reference kernel's layout is prepared for the reference kind only")
    prep = lin.prepare(p, s)
    qw = np.rint(decode_e2m1(p) * 2.0).astype(np.int8)
    assert np.array_equal(prep[1], qw.reshape(8, 8, 64, 4).transpose(0, 2, 1, 3))
    assert np.array_equal(prep[3], qw.reshape(64, 8, 32).sum(-1, dtype=np.int32))
