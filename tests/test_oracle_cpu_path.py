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
