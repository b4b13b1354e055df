"""One MoE layer on the CPU: routed experts, shared expert, ordered combine (test oracle).

Two activation modes, both following the reference:

``mode="bf16"`` (decode configs, bf16 activations):
    ``mosaicvm/model/layers.py:329-373`` (``grouped_expert_forward``) on the
    dequantised weights (``runtime/fp8.py:19-34``): fp32 gate/up, optional
    clamp (gate max-only, up both sides, ``layers.py:357-360``), SiLU(gate)*up
    in fp32, times the route weight BEFORE the down projection
    (``layers.py:361-363``), cast to bf16, fp32 down projection, and a
    sequential fp32 sum of the per-slot partials in ascending expert-id order
    (``layers.py:367-373``), cast to bf16.  It is evaluated per expert (the
    loop order of the vendored ``MoE.forward``,
    ``.mosaicvm/source/inference_model.py:634-650``), which gives the same
    arithmetic without materialising per-token weight copies.
    The shared expert is ``ExpertMLP`` (``layers.py:200-221``) in bf16:
    gate/up outputs rounded to bf16, fp32 SwiGLU, bf16 down output; the
    layer output is ``bf16(shared + routed)`` (``layers.py:297``).

``mode="fp8"`` (prefill configs, E4M3 activations):
    ``exact_moe`` -> ``fused_moe_qpa`` (``mosaicvm/kernels/exact_moe.py:12-19``,
    ``mosaicvm/kernels/qpa_mma.py:681-784``): ``act_quant_ref`` on x, the
    source-exact FP4 linear (``fp4_source.py:132-156``) rounded to bf16 for
    gate|up, fp32 SwiGLU with the same clamps, route weight, bf16 cast,
    ``act_quant_ref`` again, the FP4 down linear rounded to bf16, then the
    same ordered fp32 combine.  The shared expert runs the same FP8 path at
    weight 1.0 and the output is ``bf16(shared + routed)``.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

from .formats import act_quant_ref, dequant_fp4, fp4_linear_source, to_bf16


def _silu(x: np.ndarray) -> np.ndarray:
    return F.silu(torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32))).numpy()


def _swiglu(gate, up, w, limit: float):
    if limit > 0:
        gate = np.minimum(gate, np.float32(limit))
        up = np.clip(up, np.float32(-limit), np.float32(limit))
    z = (_silu(gate) * up).astype(np.float32)
    return (z * w[:, None].astype(np.float32)).astype(np.float32)


def _linear_f32(x, packed, scale, fast):
    if fast is not None:
        return fast(x, packed, scale)
    return (x.astype(np.float32) @ dequant_fp4(packed, scale).T).astype(np.float32)


def expert_bf16(x, gu_packed, gu_scale, dn_packed, dn_scale, w, limit: float,
                shared: bool = False, fast=None) -> np.ndarray:
    """One expert on bf16 activations x [M, H] (fp32 values of bf16) -> fp32 [M, H].
    ``fast``: an ``oracle.cpu_path.F32LinearCPU`` for the two linears (the same
    products summed in double instead of numpy's fp32 order)."""
    inter = gu_packed.shape[0] // 2
    gu = _linear_f32(x, gu_packed, gu_scale, fast)
    if shared:
        gu = to_bf16(gu)
    z = _swiglu(gu[:, :inter], gu[:, inter:], w, limit)
    zd = to_bf16(z)
    y = _linear_f32(zd, dn_packed, dn_scale, fast)
    return to_bf16(y) if shared else y


def _linear_src(q, s, packed, scale, fast):
    if fast is not None:
        return fast(q, s, fast.prepare(packed, scale))
    return fp4_linear_source(q, s, packed, scale)


def expert_fp8(xq, xs, gu_packed, gu_scale, dn_packed, dn_scale, w, limit: float, fast=None) -> np.ndarray:
    """One expert on E4M3 activations (bytes [M, H], pow2 scales [M, H/128]) -> bf16-valued fp32 [M, H].
    ``fast``: an ``oracle.cpu_path.FP4LinearCPU`` (bit-equal to ``fp4_linear_source``)."""
    inter = gu_packed.shape[0] // 2
    gu = to_bf16(_linear_src(xq, xs, gu_packed, gu_scale, fast))
    z = _swiglu(gu[:, :inter], gu[:, inter:], w, limit)
    zd = to_bf16(z)
    zq, zs = act_quant_ref(zd)
    return to_bf16(_linear_src(zq, zs, dn_packed, dn_scale, fast))


def moe_layer(x, weights, idx, bank: dict, *, mode: str = "bf16", swiglu_limit: float = 0.0,
              with_shared: bool = True, return_parts: bool = False, fast: bool = False):
    """x [T, H] (bf16 values as fp32 or a bf16 tensor), weights fp32 [T, k], idx [T, k].

    bank: dict of numpy uint8 arrays ``gu_packed [E, 2I, H/2]``,
    ``gu_scale [E, 2I, H/32]``, ``dn_packed [E, H, I/2]``, ``dn_scale [E, H, I/32]``
    and, with ``with_shared``, ``sh_gu_packed [2I, H/2]``, ``sh_gu_scale``,
    ``sh_dn_packed [H, I/2]``, ``sh_dn_scale``.
    Returns the bf16-valued fp32 output [T, H] (and the parts if asked).
    ``fast`` runs the linears in the C checkers of ``oracle/cpu_path.py``
    (V3 sizes: the FP8 path bit-equal, the bf16 path summed in double).
    """
    lin = None
    if fast:
        from .cpu_path import F32LinearCPU, FP4LinearCPU

        lin = F32LinearCPU() if mode == "bf16" else FP4LinearCPU("port")
    if isinstance(x, torch.Tensor):
        x = x.detach().to(torch.float32).cpu().numpy()
    x = np.ascontiguousarray(x, dtype=np.float32)
    weights = np.asarray(torch.as_tensor(weights).float().cpu().numpy(), dtype=np.float32)
    idx = np.asarray(torch.as_tensor(idx).cpu().numpy(), dtype=np.int64)
    t, h = x.shape
    k = idx.shape[1]
    partials = np.zeros((t, k, h), dtype=np.float32)
    if mode == "fp8":
        xq, xs = act_quant_ref(x)
    for e in np.unique(idx):
        tok, slot = np.nonzero(idx == e)
        w = weights[tok, slot]
        args = (bank["gu_packed"][e], bank["gu_scale"][e], bank["dn_packed"][e], bank["dn_scale"][e])
        if mode == "bf16":
            y = expert_bf16(x[tok], *args, w, swiglu_limit, fast=lin)
        elif mode == "fp8":
            y = expert_fp8(xq[tok], xs[tok], *args, w, swiglu_limit, fast=lin)
        else:
            raise ValueError(f"unknown mode {mode}")
        partials[tok, slot] = y
    order = np.argsort(idx, axis=1, kind="stable")
    acc = np.zeros((t, h), dtype=np.float32)
    for s in range(k):
        acc = acc + partials[np.arange(t), order[:, s]]
    routed = to_bf16(acc)
    if not with_shared:
        return (routed, partials) if return_parts else routed
    one = np.ones(t, dtype=np.float32)
    sargs = (bank["sh_gu_packed"], bank["sh_gu_scale"], bank["sh_dn_packed"], bank["sh_dn_scale"])
    if mode == "bf16":
        shared = expert_bf16(x, *sargs, one, swiglu_limit, shared=True, fast=lin)
    else:
        shared = expert_fp8(xq, xs, *sargs, one, swiglu_limit, fast=lin)
    out = to_bf16(shared + routed)
    if return_parts:
        return out, partials, routed, shared
    return out
