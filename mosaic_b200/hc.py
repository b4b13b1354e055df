"""Hyper-connections and the ffn RMSNorm around the MoE, on the fused kernels.

Reference API mirrored (paths inside fazin-ahamed/Mosaic):

* ``HyperConnections`` <- ``mosaicvm/model/layers.py:237-271``: parameters
  ``fn`` [(2+hc)*hc, hc*D], ``base`` [(2+hc)*hc], ``scale`` [3];
  ``pre(x [b, s, hc, D]) -> (y [b, s, D], post [b, s, hc], comb [b, s, hc, hc])``
  and ``post(y, residual, post, comb) -> [b, s, hc, D]``.
* ``RMSNorm`` <- ``mosaicvm/model/layers.py:19-29``: ``weight`` [D], ``eps``;
  ``forward`` runs ``mosaic_rms_norm``.
* ``ffn_pre_norm`` is the fused form of ``y, post, comb = hc_ffn.pre(x);
  y = ffn_norm(y)`` in ``V4Block.forward`` (``layers.py:428-433``), optionally
  with ``act_quant_ref`` of y (the FP8 MoE input), in one kernel
  (``mosaic_hc_pre_norm``).

Activations are bf16 (the reference's residual dtype); nothing here computes
on the CPU.
"""
from __future__ import annotations

import torch
from torch import nn

from . import _capi as C
from . import ops


class RMSNorm(nn.Module):
    """RMSNorm (layers.py:19-29) on the GPU: ``mosaic_rms_norm``, one row per CTA.

    ``forward(x)`` takes bf16 ``[..., D]`` and returns bf16, as the reference
    does for bf16 activations (fp32 arithmetic, one rounding at the end).
    ``forward(x, quant=True)`` also returns ``act_quant_ref`` of the result
    (E4M3 ``[..., D]`` and fp32 scales ``[..., D/128]``), fused.  In front of
    the MoE the norm runs fused with the hyper-connection pre-mix instead
    (:func:`ffn_pre_norm`).
    """

    def __init__(self, dim: int, eps: float = 1e-6):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim), requires_grad=False)
        self.eps = eps

    def forward(self, x, quant: bool = False):
        if x.dtype != torch.bfloat16:
            raise TypeError(f"RMSNorm on the GPU path takes bf16 activations, got {x.dtype}")
        d = x.shape[-1]
        if d != self.weight.numel():
            raise ValueError(f"RMSNorm of width {self.weight.numel()} given rows of {d}")
        t = x.numel() // d
        xf = x.reshape(t, d).contiguous()
        ops._need_cuda(xf, what="RMSNorm")
        w = self.weight.detach().float().contiguous().to(xf.device)
        y = torch.empty_like(xf)
        q = torch.empty(t, d, dtype=torch.uint8, device=xf.device) if quant else None
        qs = torch.empty(t, d // 128, dtype=torch.float32, device=xf.device) if quant else None
        st = C.lib().mosaic_rms_norm(ops._ptr(xf), ops._ptr(w), t, d, float(self.eps), ops._ptr(y), ops._ptr(q),
                                     ops._ptr(qs), ops._stream())
        C.check(st, "mosaic_rms_norm")
        y = y.view(x.shape)
        if not quant:
            return y
        return y, q.view(torch.float8_e4m3fn).view(x.shape), qs.view(*x.shape[:-1], d // 128)


class HyperConnections(nn.Module):
    """hc_mult residual copies with the Sinkhorn mix (layers.py:237-271)."""

    def __init__(self, hidden_size: int, hc_mult: int = 4, sinkhorn_iters: int = 20, hc_eps: float = 1e-6,
                 rms_norm_eps: float = 1e-6):
        super().__init__()
        self.mult = hc_mult
        self.iters = sinkhorn_iters
        self.eps = hc_eps
        self.norm_eps = rms_norm_eps
        mix = (2 + hc_mult) * hc_mult
        self.fn = nn.Parameter(torch.empty(mix, hc_mult * hidden_size), requires_grad=False)
        self.base = nn.Parameter(torch.zeros(mix), requires_grad=False)
        self.scale = nn.Parameter(torch.ones(3), requires_grad=False)
        self.last_workspace = None  # the last fused call's workspace (error word at byte 0)
        nn.init.normal_(self.fn, std=0.01)

    def pre(self, x):
        y, post, comb = _pre_norm(self, None, x, quant=False)
        return y, post, comb

    def post(self, x, residual, post, comb):
        """x [..., D] (the sub-layer output), residual [..., hc, D] -> [..., hc, D] bf16."""
        if residual.dtype != torch.bfloat16 or x.dtype != torch.bfloat16:
            raise ValueError("HyperConnections.post expects bf16 x and residual")
        hc, d = residual.shape[-2:]
        t = residual.numel() // (hc * d)
        yf, rf = x.reshape(t, d).contiguous(), residual.reshape(t, hc, d).contiguous()
        pf = post.reshape(t, hc).float().contiguous()
        cf = comb.reshape(t, hc, hc).float().contiguous()
        ops._need_cuda(yf, rf, pf, cf, what="HyperConnections.post")
        out = torch.empty_like(rf)
        st = C.lib().mosaic_hc_post(ops._ptr(yf), ops._ptr(rf), ops._ptr(pf), ops._ptr(cf), t, d, hc, ops._ptr(out),
                                    ops._stream())
        C.check(st, "mosaic_hc_post")
        return out.view(residual.shape)


def _pre_norm(hc_mod: HyperConnections, norm: RMSNorm | None, x, *, quant: bool):
    if x.dtype != torch.bfloat16:
        raise ValueError("hyper-connection input must be bf16 [..., hc, D]")
    hc, d = x.shape[-2:]
    if hc != hc_mod.mult:
        raise ValueError(f"x has {hc} residual copies, the module {hc_mod.mult}")
    if norm is not None and norm.eps != hc_mod.norm_eps:
        raise ValueError("the fused kernel uses one epsilon for the pre-mix rsqrt and the RMSNorm")
    lead = x.shape[:-2]
    t = x.numel() // (hc * d)
    xf = x.reshape(t, hc, d).contiguous()
    ops._need_cuda(xf, what="hyper-connection pre-mix")
    dev = xf.device
    fn = hc_mod.fn.detach().float().contiguous().to(dev)
    base = hc_mod.base.detach().float().contiguous().to(dev)
    scale = hc_mod.scale.detach().float().contiguous().to(dev)
    w = None if norm is None else norm.weight.detach().float().contiguous().to(dev)
    y = torch.empty(t, d, dtype=torch.bfloat16, device=dev)
    post = torch.empty(t, hc, dtype=torch.float32, device=dev)
    comb = torch.empty(t, hc, hc, dtype=torch.float32, device=dev)
    q = torch.empty(t, d, dtype=torch.uint8, device=dev) if quant else None
    qs = torch.empty(t, d // 128, dtype=torch.float32, device=dev) if quant else None
    lib = C.lib()
    ws = torch.empty(max(lib.mosaic_hc_pre_norm_workspace_bytes(t, d, hc), 256), dtype=torch.uint8, device=dev)
    st = lib.mosaic_hc_pre_norm(ops._ptr(xf), ops._ptr(fn), ops._ptr(base), ops._ptr(scale), ops._ptr(w), t, d, hc,
                                hc_mod.iters, float(hc_mod.eps), float(hc_mod.norm_eps), ops._ptr(y), ops._ptr(post),
                                ops._ptr(comb), ops._ptr(q), ops._ptr(qs), ops._ptr(ws), ws.numel(), ops._stream())
    C.check(st, "mosaic_hc_pre_norm")
    hc_mod.last_workspace = ws  # its error word: ops.read_error(hc.last_workspace)
    out = (y.view(*lead, d), post.view(*lead, hc), comb.view(*lead, hc, hc))
    if quant:
        out += (q.view(torch.float8_e4m3fn).view(*lead, d), qs.view(*lead, d // 128))
    return out


def ffn_pre_norm(x, hc: HyperConnections, norm: RMSNorm, *, quant: bool = False):
    """``y, post, comb = hc.pre(x); y = norm(y)`` in one kernel (layers.py:428-433).

    Returns (y bf16 [..., D], post, comb), plus (q E4M3 [..., D], q_scale fp32
    [..., D/128]) = ``act_quant_ref(y)`` when ``quant``.
    """
    return _pre_norm(hc, norm, x, quant=quant)
