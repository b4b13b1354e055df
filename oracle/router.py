"""Sigmoid group-limited top-k router with a selection-only bias (test oracle).

Reference behaviour followed:

* ``mosaicvm/model/layers.py:127-150`` (``Router.forward``): fp32 logits
  ``F.linear(x.float(), W.float())``; scores; ``+ e_score_correction_bias``
  for selection only; ``torch.topk``; weights gathered from the UNBIASED
  scores; normalised by ``sum.clamp_min(1e-9)``; times
  ``routed_scaling_factor``.
* ``.mosaicvm/source/inference_model.py:569-589`` (vendored ``Gate``):
  the ``score_func == "sigmoid"`` branch (``scores.sigmoid()``).
* The group limit (n_group / topk_group) is absent from the reference.  It is
  restated from the published DeepSeek-V3 rule: each group's score is the sum
  of its two largest biased scores; the ``topk_group`` best groups survive;
  experts of the other groups are masked to -inf before the final top-k.
  With ``topk_group == n_group`` it is the identity and the router equals the
  reference ``Gate`` bit for bit (pinned in tests/test_oracle_golden.py).

``route_ties`` marks tokens whose selection is not decidable in fp32: it
recomputes the logits in float64 and bounds the error of an fp32 summation
of the K products by the probabilistic bound lam * u * sqrt(K/2) * ||x o w||_2
(u = 2^-24, lam = 10; Higham & Mary, "A new approach to probabilistic rounding
error analysis", SIAM J. Sci. Comput. 41(5), 2019).  The worst-case bound
gamma_K * sum|x_i w_i| is ~1e4 times larger than the errors fp32 summation
actually makes at K = 7168 (measured ~1e-6 on these inputs for both torch's
CPU GEMM and the GPU's split-K FMA chain, against a probabilistic bound of
~1.5e-5), and would declare most tokens ties.  The logit bound is propagated
through the sigmoid (Lipschitz 1/4) plus a few ulps of evaluation error, and
every token for which a group or expert decision boundary has a margin below
the combined bound is flagged.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F


def route(x, weight, bias, *, top_k: int, n_group: int = 1, topk_group: int = 1,
          route_scale: float = 1.0, norm_topk_prob: bool = True):
    """x [T, H] (bf16 or fp32 tensor), weight [E, H] fp32, bias [E] fp32
    -> (weights fp32 [T, k], idx int64 [T, k]) in torch.topk (descending) order."""
    x = torch.as_tensor(x)
    weight = torch.as_tensor(weight, dtype=torch.float32)
    bias = torch.as_tensor(bias, dtype=torch.float32)
    logits = F.linear(x.float(), weight.float())
    scores = logits.sigmoid()
    sel = scores + bias
    t, e = sel.shape
    if n_group > 1 and topk_group < n_group:
        g = sel.view(t, n_group, e // n_group)
        gscore = g.topk(2, dim=-1).values.sum(dim=-1)
        keep = gscore.topk(topk_group, dim=-1).indices
        mask = torch.ones(t, n_group, dtype=torch.bool).scatter_(1, keep, False)
        sel = g.masked_fill(mask.unsqueeze(-1), float("-inf")).view(t, e)
    idx = torch.topk(sel, top_k, dim=-1).indices
    w = scores.gather(-1, idx)
    if norm_topk_prob:
        w = w / w.sum(dim=-1, keepdim=True).clamp_min(1e-9)
    w = w * route_scale
    return w.float(), idx


def route_ties(x, weight, bias, *, top_k: int, n_group: int = 1, topk_group: int = 1,
               eval_ulps: float = 8.0, lam: float = 10.0):
    """Return (sel_tie [T] bool, order_tie [T] bool).

    sel_tie: the SET of selected experts is not decidable in fp32.
    order_tie: the set is decidable but the descending order of two selected
    experts is not (compare as sets there).
    """
    xd = torch.as_tensor(x).to(torch.float64).numpy()
    wd = torch.as_tensor(weight).to(torch.float64).numpy()
    b = torch.as_tensor(bias).to(torch.float64).numpy()
    k_dim = xd.shape[1]
    u = 2.0 ** -24
    logits = xd @ wd.T
    err = lam * u * np.sqrt(k_dim / 2.0) * np.sqrt((xd * xd) @ (wd * wd).T)
    s = 1.0 / (1.0 + np.exp(-logits))
    sel = s + b
    dsel = err / 4.0 + eval_ulps * np.spacing(np.abs(sel).astype(np.float32)).astype(np.float64)
    t, e = sel.shape
    sel_tie = np.zeros(t, dtype=bool)
    order_tie = np.zeros(t, dtype=bool)
    for ti in range(t):
        row = sel[ti].copy()
        drow = dsel[ti]
        if n_group > 1 and topk_group < n_group:
            gsz = e // n_group
            gs = np.empty(n_group)
            gd = np.empty(n_group)
            for gi in range(n_group):
                seg = row[gi * gsz:(gi + 1) * gsz]
                o = np.argsort(-seg, kind="stable")
                gs[gi] = seg[o[0]] + seg[o[1]]
                gd[gi] = drow[gi * gsz + o[0]] + drow[gi * gsz + o[1]] + 2 * drow[gi * gsz:(gi + 1) * gsz].max()
            og = np.argsort(-gs, kind="stable")
            a, bb = og[topk_group - 1], og[topk_group]
            if gs[a] - gs[bb] <= gd[a] + gd[bb]:
                sel_tie[ti] = True
                continue
            keep = np.zeros(n_group, dtype=bool)
            keep[og[:topk_group]] = True
            row = np.where(np.repeat(keep, gsz), row, -np.inf)
        o = np.argsort(-row, kind="stable")
        a, bb = o[top_k - 1], o[top_k]
        if np.isfinite(row[bb]) and row[a] - row[bb] <= drow[a] + drow[bb]:
            sel_tie[ti] = True
            continue
        for j in range(top_k - 1):
            p, q = o[j], o[j + 1]
            if row[p] - row[q] <= drow[p] + drow[q]:
                order_tie[ti] = True
                break
    return sel_tie, order_tie
