"""Seeded synthetic MoE layers at the benchmark configurations (no dataset involved).

* Expert weights ~ N(0, 0.02), quantised to MXFP4 on the GPU by the packer
  (bit-identical to the reference ``pack_mxfp4_nk``); the shared expert is
  drawn the same way and stored as the bank's last expert.
* Router weight ~ U(-1/sqrt(H), 1/sqrt(H)) fp32; bias ~ N(0, 0.01) fp32, or
  calibrated so the per-expert load follows Zipf(alpha) (prefill config).
* Tokens ~ N(0, 1) in bf16.

Everything is drawn from ``torch.Generator`` seeded per tensor, on the device
the layer lives on.
"""
from __future__ import annotations

import math

import numpy as np
import torch

from .moe import ExpertBank, MoEConfig, MoELayer
from . import ops

V3 = dict(hidden_size=7168, moe_intermediate_size=2048, n_routed_experts=256, num_experts_per_tok=8,
          n_group=8, topk_group=4, routed_scaling_factor=2.5)


def _gen(seed: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def make_bank(hidden: int, inter: int, n_experts: int, seed: int, *, has_shared: bool = True, std: float = 0.02,
              device="cuda") -> ExpertBank:
    """MXFP4 bank of n_experts (+1 shared) experts with N(0, std) weights."""
    n = n_experts + (1 if has_shared else 0)
    gu_p = torch.empty(n, 2 * inter, hidden // 2, dtype=torch.uint8, device=device)
    gu_s = torch.empty(n, 2 * inter, hidden // 32, dtype=torch.uint8, device=device)
    dn_p = torch.empty(n, hidden, inter // 2, dtype=torch.uint8, device=device)
    dn_s = torch.empty(n, hidden, inter // 32, dtype=torch.uint8, device=device)
    g = _gen(seed, device)
    for e in range(n):
        w = torch.randn(2 * inter, hidden, generator=g, device=device) * std
        gu_p[e], gu_s[e] = ops.pack_mxfp4_nk(w)
        w = torch.randn(hidden, inter, generator=g, device=device) * std
        dn_p[e], dn_s[e] = ops.pack_mxfp4_nk(w)
        del w
    return ExpertBank(gu_p, gu_s, dn_p, dn_s, has_shared=has_shared)


def make_local_bank(hidden: int, inter: int, n_experts: int, seed: int, *, lo: int, hi: int, std: float = 0.02,
                    device="cuda") -> ExpertBank:
    """Experts [lo, hi) of an n_experts bank plus its shared expert (last), each
    drawn from a generator seeded by (seed, expert id): every rank of an
    expert-parallel group gets the same weights for an expert without
    generating the whole bank."""
    ids = list(range(lo, hi)) + [n_experts]
    n = len(ids)
    gu_p = torch.empty(n, 2 * inter, hidden // 2, dtype=torch.uint8, device=device)
    gu_s = torch.empty(n, 2 * inter, hidden // 32, dtype=torch.uint8, device=device)
    dn_p = torch.empty(n, hidden, inter // 2, dtype=torch.uint8, device=device)
    dn_s = torch.empty(n, hidden, inter // 32, dtype=torch.uint8, device=device)
    for i, e in enumerate(ids):
        g = _gen(seed * 1009 + e, device)
        w = torch.randn(2 * inter, hidden, generator=g, device=device) * std
        gu_p[i], gu_s[i] = ops.pack_mxfp4_nk(w)
        w = torch.randn(hidden, inter, generator=g, device=device) * std
        dn_p[i], dn_s[i] = ops.pack_mxfp4_nk(w)
        del w
    return ExpertBank(gu_p, gu_s, dn_p, dn_s, has_shared=True, keep_packed=False)


def make_router_weights(hidden: int, n_experts: int, seed: int, device="cuda"):
    """Router weight U(-1/sqrt(H), 1/sqrt(H)) and bias N(0, 0.01), seeded."""
    g = _gen(seed + 1, device)
    bound = 1.0 / math.sqrt(hidden)
    w = (torch.rand(n_experts, hidden, generator=g, device=device) * 2 - 1) * bound
    b = torch.randn(n_experts, generator=g, device=device) * 0.01
    return w, b


def make_router(layer: MoELayer, seed: int, device="cuda") -> None:
    cfg = layer.cfg
    g = _gen(seed + 1, device)
    bound = 1.0 / math.sqrt(cfg.hidden_size)
    w = (torch.rand(cfg.n_routed_experts, cfg.hidden_size, generator=g, device=device) * 2 - 1) * bound
    b = torch.randn(cfg.n_routed_experts, generator=g, device=device) * 0.01
    layer.router.weight.data = w
    layer.router.e_score_correction_bias.data = b


def make_tokens(t: int, hidden: int, seed: int, device="cuda") -> torch.Tensor:
    g = _gen(seed + 2, device)
    return torch.randn(t, hidden, generator=g, device=device).to(torch.bfloat16)


def make_layer(tokens: int, seed: int = 0, act_mode: str = "bf16", n_experts: int = 256, device="cuda",
               bank: ExpertBank | None = None, **overrides):
    """V3-dimension layer + tokens.  Returns (layer, x)."""
    kw = dict(V3)
    kw.update(overrides)
    kw["n_routed_experts"] = n_experts
    cfg = MoEConfig(act_mode=act_mode, **kw)
    if bank is None:
        bank = make_bank(cfg.hidden_size, cfg.moe_intermediate_size, n_experts, seed, device=device)
    layer = MoELayer(cfg, bank)
    make_router(layer, seed, device)
    x = make_tokens(tokens, cfg.hidden_size, seed, device)
    return layer, x


def zipf_targets(n_experts: int, alpha: float, assignments: int, seed: int, cap: float | None = None) -> np.ndarray:
    """Per-expert target loads proportional to rank^-alpha, ranks assigned by a seeded permutation.

    With ``cap`` (the token count: an expert takes at most one slot of a token)
    the loads above it are clipped and the excess is spread over the other
    experts in proportion to their Zipf shares, until none exceeds the cap
    (Zipf(1.2) over 256 experts asks 25 % of all slots of rank 1, more than
    one per token at top-8)."""
    rng = np.random.default_rng(seed)
    ranks = rng.permutation(n_experts) + 1
    share = ranks.astype(np.float64) ** (-alpha)
    t = share / share.sum() * assignments
    if cap is not None:
        for _ in range(n_experts):
            over = t > cap
            if not over.any():
                break
            excess = float((t[over] - cap).sum())
            t[over] = cap
            free = ~over & (t < cap)
            t[free] += excess * share[free] / share[free].sum()
    return t


def _fit_alpha(load: np.ndarray) -> float:
    srt = np.sort(load)[::-1]
    r = np.arange(1, len(srt) + 1)
    nz = srt > 0
    return float(-np.polyfit(np.log(r[nz]), np.log(srt[nz]), 1)[0]) if nz.sum() > 2 else float("nan")


def calibrate_zipf_bias(layer: MoELayer, alpha: float = 1.2, tokens: int = 8192, steps: int = 300,
                        seed: int = 0) -> dict:
    """Fit the selection bias so the per-expert load approaches the clipped
    Zipf(alpha) target of :func:`zipf_targets` on a separate calibration batch.

    Each step moves b_e by lr_i * clip(log((target_e + 1) / (load_e + 1)), -1, 1),
    with lr decaying from 0.05 to 0.002: large moves first (the bias has to
    span about the spread of the sigmoid scores), fine ones last.  Returns the
    final histogram's summary: fitted exponent, max / min load, the target's
    maximum and the relative L1 distance sum|load - target| / sum target.
    """
    cfg = layer.cfg
    dev = layer.router.weight.device
    xc = make_tokens(tokens, cfg.hidden_size, seed + 1000, dev)
    a = tokens * cfg.num_experts_per_tok
    target_np = zipf_targets(cfg.n_routed_experts, alpha, a, seed, cap=float(tokens))
    target = torch.from_numpy(target_np).to(dev)
    bias = layer.router.e_score_correction_bias.data
    for i in range(steps):
        _, idx = layer.router(xc)
        load = torch.bincount(idx.reshape(-1), minlength=cfg.n_routed_experts).double()
        lr = 0.048 * (0.985 ** i) + 0.002
        bias += (lr * torch.clamp(torch.log((target + 1.0) / (load + 1.0)), -1.0, 1.0)).float()
    _, idx = layer.router(xc)
    load = torch.bincount(idx.reshape(-1), minlength=cfg.n_routed_experts).double().cpu().numpy()
    return {"alpha": alpha, "target": "Zipf(alpha) clipped at one slot per token, excess re-spread",
            "load_max": float(load.max()), "load_min": float(load.min()), "target_max": float(target_np.max()),
            "fitted_alpha": _fit_alpha(load), "target_fitted_alpha": _fit_alpha(target_np),
            "l1_rel": float(np.abs(load - target_np).sum() / target_np.sum()), "steps": steps,
            "calibration_tokens": tokens}


def bank_to_oracle(bank: ExpertBank, experts) -> dict:
    """Copy the packed bytes of the given routed experts (+ the shared one) to host numpy
    in the oracle's bank layout (expert i of the dict = experts[i])."""
    experts = torch.as_tensor(np.asarray(experts), dtype=torch.long, device=bank.gu_packed.device)
    out = {"gu_packed": bank.gu_packed[experts].cpu().numpy(), "gu_scale": bank.gu_scale[experts].cpu().numpy(),
           "dn_packed": bank.dn_packed[experts].cpu().numpy(), "dn_scale": bank.dn_scale[experts].cpu().numpy()}
    if bank.has_shared:
        s = bank.n_bank - 1
        out.update({"sh_gu_packed": bank.gu_packed[s].cpu().numpy(), "sh_gu_scale": bank.gu_scale[s].cpu().numpy(),
                    "sh_dn_packed": bank.dn_packed[s].cpu().numpy(), "sh_dn_scale": bank.dn_scale[s].cpu().numpy()})
    return out
