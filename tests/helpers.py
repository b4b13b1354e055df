"""Shared test helpers: build oracle banks and GPU banks from the same seeded case."""
from __future__ import annotations

import numpy as np
import torch

from oracle import formats as fm


def pack_case(case):
    """Pack every expert of a recipe case with the oracle packer (pinned to the reference)."""
    e = case["cfg"]["E"]
    gu = [fm.pack_mxfp4_nk(w) for w in case["w_gu"]]
    dn = [fm.pack_mxfp4_nk(w) for w in case["w_dn"]]
    obank = {"gu_packed": np.stack([p for p, _ in gu[:e]]), "gu_scale": np.stack([s for _, s in gu[:e]]),
             "dn_packed": np.stack([p for p, _ in dn[:e]]), "dn_scale": np.stack([s for _, s in dn[:e]]),
             "sh_gu_packed": gu[e][0], "sh_gu_scale": gu[e][1], "sh_dn_packed": dn[e][0],
             "sh_dn_scale": dn[e][1]}
    full = (np.stack([p for p, _ in gu]), np.stack([s for _, s in gu]),
            np.stack([p for p, _ in dn]), np.stack([s for _, s in dn]))
    return obank, full


def gpu_bank(full, has_shared=True, device="cuda"):
    from mosaic_b200 import ExpertBank

    t = [torch.from_numpy(np.ascontiguousarray(a)).to(device) for a in full]
    if not has_shared:
        t = [a[:-1].contiguous() for a in t]
    return ExpertBank(*t, has_shared=has_shared)


def layer_for(case, bank, mode, device="cuda"):
    from mosaic_b200 import MoEConfig, MoELayer

    c = case["cfg"]
    cfg = MoEConfig(hidden_size=c["H"], moe_intermediate_size=c["I"], n_routed_experts=c["E"],
                    num_experts_per_tok=c["k"], n_group=c["n_group"], topk_group=c["topk_group"],
                    routed_scaling_factor=c["scale"], swiglu_limit=c["swiglu_limit"], act_mode=mode,
                    n_shared_experts=1 if bank.has_shared else 0)
    layer = MoELayer(cfg, bank)
    layer.router.weight.data = case["router_w"].to(device)
    layer.router.e_score_correction_bias.data = case["bias"].to(device)
    return layer


def rel_l2(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def oracle_subset(layer, x, y, sel, mode):
    """Relative L2 of the layer output y on the tokens ``sel`` against the CPU
    oracle, run with the routing the layer used (its last call) on a bank of
    just the experts those tokens touch (the C linears of oracle/cpu_path.py:
    V3-size experts in seconds)."""
    from mosaic_b200 import synthetic
    from oracle.moe import moe_layer

    sel = np.sort(np.asarray(sel))
    idx = layer.last_idx[torch.as_tensor(sel, device=layer.last_idx.device)].cpu()
    w = layer.last_weights[torch.as_tensor(sel, device=layer.last_idx.device)].cpu()
    experts = np.unique(idx.numpy())
    obank = synthetic.bank_to_oracle(layer.bank, experts)
    remap = {int(e): i for i, e in enumerate(experts)}
    idx_l = torch.tensor([[remap[int(v)] for v in row] for row in idx.numpy()])
    xs = x[torch.as_tensor(sel, device=x.device)].cpu()
    ref = moe_layer(xs, w, idx_l, obank, mode=mode, swiglu_limit=layer.cfg.swiglu_limit, fast=True)
    return rel_l2(y[torch.as_tensor(sel, device=y.device)].float().cpu().numpy(), ref)
