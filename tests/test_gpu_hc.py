"""Hyper-connection pre-mix + RMSNorm (+ act_quant) and post-mix on the GPU.

Bars: post / comb within rtol 1e-4, atol 1e-6 (the mixing dot products run over
hc*D products in another order than torch's CPU GEMM); bf16 outputs bit-equal on
at least 98 % of the elements and everywhere within two bf16 ulps of the value
(the pre-mix is rounded to bf16 before the RMSNorm rounds again, so a one-ulp
flip in the first becomes up to two in the second) plus 2^-14 of the row's
RMS.  The absolute term covers cancellation: an output
sum_m pre_m * x_m of terms ~1 that nearly cancels carries the fp32 error of its
terms (pre differs from the reference in its last bits), which is large
relative to the tiny result but not to the row.  The fused E4M3 act_quant is
bit-equal to act_quant_ref applied to the kernel's own bf16 output.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle.formats import act_quant_ref
from oracle.hc import hc_post, hc_pre, rms_norm
from tests.golden.recipes import HC_CASES, HC_ORACLE_CASES, make_hc_case

pytestmark = pytest.mark.gpu
GOLD = Path(__file__).parent / "golden"


def _bf16_close(got, ref, what):
    got = np.asarray(got, dtype=np.float32)
    ref = np.asarray(ref, dtype=np.float32)
    rms = np.sqrt(np.mean(ref.astype(np.float64) ** 2, axis=-1, keepdims=True))
    tol = np.maximum(np.abs(ref), np.abs(got)) * 2.0 ** -6 + rms * 2.0 ** -14 + 1e-30
    assert np.all(np.abs(got - ref) <= tol), (what, float(np.max(np.abs(got - ref) / tol)))
    assert np.mean(got == ref) >= 0.98, (what, float(np.mean(got == ref)))


def _modules(hc_mult, d, iters, fn, base, scale, norm_w):
    from mosaic_b200.hc import HyperConnections, RMSNorm

    hc = HyperConnections(d, hc_mult=hc_mult, sinkhorn_iters=iters)
    hc.fn.data, hc.base.data, hc.scale.data = fn.cuda(), base.cuda(), scale.cuda()
    norm = RMSNorm(d)
    norm.weight.data = norm_w.cuda()
    return hc, norm


@pytest.mark.parametrize("name", list(HC_CASES))
def test_hc_matches_reference_golden(name):
    from mosaic_b200.hc import ffn_pre_norm

    gold = np.load(GOLD / "hc.npz")
    b, s, hcm, d, iters, seed = HC_CASES[name]
    x, fn, base, scale, norm_w, y = make_hc_case(b, s, hcm, d, seed)
    hc, norm = _modules(hcm, d, iters, fn, base, scale, norm_w)
    xg = x.cuda()
    y_pre, post, comb = hc.pre(xg)
    torch.cuda.synchronize()
    _bf16_close(y_pre.float().cpu(), gold[name + "_y_pre"], "y_pre")
    np.testing.assert_allclose(post.cpu().numpy(), gold[name + "_post"], rtol=1e-4, atol=1e-6)
    np.testing.assert_allclose(comb.cpu().numpy(), gold[name + "_comb"], rtol=1e-4, atol=1e-6)
    yn, post2, comb2, q, qs = ffn_pre_norm(xg, hc, norm, quant=True)
    torch.cuda.synchronize()
    from mosaic_b200 import ops

    assert ops.read_error(hc.last_workspace) == 0
    assert torch.equal(post2, post) and torch.equal(comb2, comb)
    _bf16_close(yn.float().cpu(), gold[name + "_y_norm"], "y_norm")
    q_ref, s_ref = act_quant_ref(yn.float().cpu().numpy().reshape(-1, d))
    assert np.array_equal(q.view(torch.uint8).cpu().numpy().reshape(-1, d), q_ref)
    assert np.array_equal(qs.cpu().numpy().reshape(-1, d // 128), s_ref)
    out = hc.post(y.cuda(), xg, torch.from_numpy(gold[name + "_post"]).cuda(),
                  torch.from_numpy(gold[name + "_comb"]).cuda())
    torch.cuda.synchronize()
    _bf16_close(out.float().cpu(), gold[name + "_out_post"], "post-mix")


@pytest.mark.parametrize("t", [1, 37, 300, 1001])
def test_hc_pre_norm_v3_dims(t):
    """D 7168 (the MoE hidden size of the BASELINE configs), 1..1001 tokens: every
    tokens-per-CTA variant (1, 2, 4) and a partial last group."""
    from mosaic_b200.hc import ffn_pre_norm

    d, hcm = 7168, 4
    x, fn, base, scale, norm_w, _ = make_hc_case(1, t, hcm, d, seed=60 + t)
    hc, norm = _modules(hcm, d, 20, fn, base, scale, norm_w)
    yn, post, comb = ffn_pre_norm(x.cuda(), hc, norm)
    torch.cuda.synchronize()
    from mosaic_b200 import ops

    assert ops.read_error(hc.last_workspace) == 0  # no pipeline wait of the mixing kernel ran out
    y_pre, post_r, comb_r = hc_pre(x, fn, base, scale, iters=20, eps=1e-6, norm_eps=1e-6)
    ref = rms_norm(y_pre, norm_w, 1e-6)
    np.testing.assert_allclose(post.cpu().numpy(), post_r.numpy(), rtol=1e-4, atol=1e-6)
    np.testing.assert_allclose(comb.cpu().numpy(), comb_r.numpy(), rtol=1e-4, atol=1e-6)
    _bf16_close(yn.float().cpu(), ref.float(), "y_norm")



@pytest.mark.parametrize("t,hcm,d", [(130, 4, 12288), (150, 2, 16384), (151, 3, 8192), (2000, 1, 1024)])
def test_hc_pre_norm_kernel_variants(t, hcm, d):
    """Both pre-mix kernels: D <= 8192 takes the bulk-copy ring (hc 3 x D 8192
    with four chunks per thread, and 2000 tokens of hc 1 x D 1024 that wrap
    every CTA's ring of barriers many times, both groups of each CTA busy);
    D 12288 and 16384 take the register kernel."""
    from mosaic_b200.hc import ffn_pre_norm

    x, fn, base, scale, norm_w, _ = make_hc_case(1, t, hcm, d, seed=70 + hcm)
    hc, norm = _modules(hcm, d, 20, fn, base, scale, norm_w)
    yn, post, comb, q, qs = ffn_pre_norm(x.cuda(), hc, norm, quant=True)
    torch.cuda.synchronize()
    from mosaic_b200 import ops

    assert ops.read_error(hc.last_workspace) == 0
    y_pre, post_r, comb_r = hc_pre(x, fn, base, scale, iters=20, eps=1e-6, norm_eps=1e-6)
    ref = rms_norm(y_pre, norm_w, 1e-6)
    np.testing.assert_allclose(post.cpu().numpy(), post_r.numpy(), rtol=1e-4, atol=1e-6)
    np.testing.assert_allclose(comb.cpu().numpy(), comb_r.numpy(), rtol=1e-4, atol=1e-6)
    _bf16_close(yn.float().cpu(), ref.float(), "y_norm")
    q_ref, s_ref = act_quant_ref(yn.float().cpu().numpy().reshape(-1, d))
    assert np.array_equal(q.view(torch.uint8).cpu().numpy().reshape(-1, d), q_ref)
    assert np.array_equal(qs.cpu().numpy().reshape(-1, d // 128), s_ref)

def test_hc_pre_norm_feeds_the_moe_layer():
    """The fused output drives a MoE layer exactly like the same bf16 tensor built on the host."""
    from mosaic_b200 import synthetic
    from mosaic_b200.hc import ffn_pre_norm

    layer, _ = synthetic.make_layer(tokens=8, seed=3, act_mode="bf16", n_experts=32)
    d = layer.cfg.hidden_size
    x, fn, base, scale, norm_w, _ = make_hc_case(1, 8, 4, d, seed=70)
    hc, norm = _modules(4, d, 20, fn, base, scale, norm_w)
    yn, _, _ = ffn_pre_norm(x.cuda(), hc, norm)
    y1 = layer(yn)
    y2 = layer(yn.clone())
    torch.cuda.synchronize()
    assert torch.equal(y1, y2) and torch.isfinite(y1.float()).all()


@pytest.mark.parametrize("name", list(HC_ORACLE_CASES))
def test_rms_norm_matches_reference_golden(name):
    """Standalone RMSNorm on the reference's own pre-mix output (y_pre, bf16)
    against the reference RMSNorm's output: the same bf16 input, so only the
    order of the sum of squares differs; act_quant of the result is bit-equal
    to act_quant_ref of the kernel's bf16 output."""
    from mosaic_b200.hc import RMSNorm

    gold = np.load(GOLD / "hc.npz")
    b, s, hcm, d, iters, seed = HC_ORACLE_CASES[name]
    _, _, _, _, norm_w, _ = make_hc_case(b, s, hcm, d, seed)
    x = torch.from_numpy(gold[name + "_y_pre"]).to(torch.bfloat16).cuda()
    norm = RMSNorm(d)
    norm.weight.data = norm_w.cuda()
    y = norm(x)
    torch.cuda.synchronize()
    assert y.dtype == torch.bfloat16 and y.shape == x.shape
    _bf16_close(y.float().cpu(), gold[name + "_y_norm"], "rms_norm")
    if d % 128 == 0:
        y2, q, qs = norm(x, quant=True)
        torch.cuda.synchronize()
        assert torch.equal(y2, y)
        q_ref, s_ref = act_quant_ref(y.float().cpu().numpy().reshape(-1, d))
        assert np.array_equal(q.view(torch.uint8).cpu().numpy().reshape(-1, d), q_ref)
        assert np.array_equal(qs.cpu().numpy().reshape(-1, d // 128), s_ref)


@pytest.mark.parametrize("t,d", [(1, 8), (3, 136), (257, 7168), (64, 16384), (2, 65536)])
def test_rms_norm_against_oracle(t, d):
    """Widths from one vector to MOSAIC_RMS_NORM_MAX_D (partial last pass of the
    block, more passes than one, the widest shared-memory row)."""
    from mosaic_b200.hc import RMSNorm

    g = torch.Generator().manual_seed(t * 7 + d)
    x = (torch.randn(t, d, generator=g) * 3).to(torch.bfloat16)
    w = 1 + 0.1 * torch.randn(d, generator=g)
    norm = RMSNorm(d, eps=1e-6)
    norm.weight.data = w.cuda()
    y = norm(x.cuda())
    torch.cuda.synchronize()
    _bf16_close(y.float().cpu(), rms_norm(x, w, 1e-6).float(), "rms_norm")


def test_rms_norm_rejects_other_dtypes():
    from mosaic_b200.hc import RMSNorm

    with pytest.raises(TypeError):
        RMSNorm(256).cuda()(torch.zeros(2, 256, device="cuda"))
