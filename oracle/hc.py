"""Hyper-connection pre/post mixes and RMSNorm around the MoE (test oracle).

Test infrastructure only: the tests and ``__graft_entry__.smoke()`` use it as
the checker; the product never calls it.  fp32 torch on the CPU, in the
reference's operation order:

* ``rms_norm``   <- ``mosaicvm/model/layers.py:19-29`` (``RMSNorm.forward``)
* ``sinkhorn``   <- ``mosaicvm/model/layers.py:222-234`` (``hc_split_sinkhorn``)
* ``hc_pre``     <- ``mosaicvm/model/layers.py:258-267`` (``HyperConnections.pre``)
* ``hc_post``    <- ``mosaicvm/model/layers.py:269-271`` (``HyperConnections.post``)

Pinned against the reference modules' own outputs in tests/golden/hc.npz.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    dtype = x.dtype
    x = x.float()
    x = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps)
    return (x * weight.float()).to(dtype)


def sinkhorn(mixes, hc_scale, hc_base, hc_mult: int, iters: int, eps: float):
    pre_raw = mixes[..., :hc_mult]
    post_raw = mixes[..., hc_mult:2 * hc_mult]
    comb_raw = mixes[..., 2 * hc_mult:].reshape(*mixes.shape[:-1], hc_mult, hc_mult)
    pre = torch.sigmoid(pre_raw * hc_scale[0] + hc_base[:hc_mult]) + eps
    post = 2 * torch.sigmoid(post_raw * hc_scale[1] + hc_base[hc_mult:2 * hc_mult])
    comb = comb_raw * hc_scale[2] + hc_base[2 * hc_mult:].reshape(hc_mult, hc_mult)
    comb = F.softmax(comb, dim=-1) + eps
    for _ in range(max(iters - 1, 0)):
        comb = comb / (comb.sum(dim=-1, keepdim=True) + eps)
        comb = comb / (comb.sum(dim=-2, keepdim=True) + eps)
    return pre, post, comb


def hc_pre(x, fn, base, scale, *, iters: int, eps: float, norm_eps: float):
    """x [..., hc, D] -> (y [..., D] in x's dtype, post [..., hc], comb [..., hc, hc])."""
    hc_mult = x.shape[-2]
    x_flat = x.flatten(-2).float()
    rsqrt = torch.rsqrt(x_flat.pow(2).mean(-1, keepdim=True) + norm_eps)
    mixes = F.linear(x_flat, fn.float()) * rsqrt
    pre, post, comb = sinkhorn(mixes, scale.float(), base.float(), hc_mult, iters, eps)
    y = (pre.unsqueeze(-1) * x.float()).sum(dim=-2)
    return y.to(x.dtype), post, comb


def hc_post(y, residual, post, comb):
    """y [..., D] (the sub-layer output), residual [..., hc, D] -> [..., hc, D] in residual's dtype."""
    out = post.unsqueeze(-1) * y.unsqueeze(-2).float() + torch.einsum("...mn,...nd->...md", comb, residual.float())
    return out.to(residual.dtype)
