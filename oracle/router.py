"""Group-limited top-k router with a selection-only bias, and hash routing (test oracle).

Test infrastructure only: the tests, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU baseline use it as the checker; the product never calls it.

Reference behaviour followed:

* ``mosaicvm/model/layers.py:127-150`` (``Router.forward``): fp32 logits
  ``F.linear(x.float(), W.float())``; scores; ``+ e_score_correction_bias``
  for selection only; ``torch.topk``; weights gathered from the UNBIASED
  scores; normalised by ``sum.clamp_min(1e-9)``; times
  ``routed_scaling_factor``.
* Score functions: ``sigmoid`` and ``softmax`` from the vendored ``Gate``
  (``.mosaicvm/source/inference_model.py:571-574``), ``sqrtsoftplus`` from
  ``layers.py:110-115`` (``_router_scores``: ``F.softplus(l).sqrt()``).
* ``hash_route`` follows ``layers.py:171-197`` (``HashRouter.forward``): ids
  ``tid2eid[token_ids % V]``, weights the scores gathered there, normalised
  unless softmax, times the scale; without a table the salted hash of
  ``layers.py:180-184`` evaluated in torch's int32 tensor arithmetic.
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


SCORE_FUNCS = ("sigmoid", "sqrtsoftplus", "softmax")


def router_scores(logits: torch.Tensor, score_func: str) -> torch.Tensor:
    """fp32 scores of fp32 logits [T, E] (inference_model.py:571-576, layers.py:110-115)."""
    if score_func == "sigmoid":
        return logits.sigmoid()
    if score_func == "sqrtsoftplus":
        return F.softplus(logits.float()).sqrt()
    if score_func == "softmax":
        return logits.softmax(dim=-1)
    raise ValueError(f"unknown scoring_func {score_func}")


def route(x, weight, bias, *, top_k: int, n_group: int = 1, topk_group: int = 1,
          route_scale: float = 1.0, norm_topk_prob: bool = True, score_func: str = "sigmoid"):
    """x [T, H] (bf16 or fp32 tensor), weight [E, H] fp32, bias [E] fp32 (or None)
    -> (weights fp32 [T, k], idx int64 [T, k]) in torch.topk (descending) order."""
    x = torch.as_tensor(x)
    weight = torch.as_tensor(weight, dtype=torch.float32)
    logits = F.linear(x.float(), weight.float())
    scores = router_scores(logits, score_func)
    sel = scores if bias is None else scores + torch.as_tensor(bias, dtype=torch.float32)
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


def _scores_and_error(logits, err, score_func):
    """float64 scores and a first-order bound on their change for logit errors ``err``."""
    if score_func == "sigmoid":
        s = 1.0 / (1.0 + np.exp(-logits))
        return s, err * s * (1.0 - s)
    if score_func == "sqrtsoftplus":
        sp = np.where(logits > 20.0, logits, np.log1p(np.exp(np.minimum(logits, 20.0))))
        s = np.sqrt(sp)
        sig = 1.0 / (1.0 + np.exp(-logits))
        ds = np.where(logits > 20.0, 0.5 / np.maximum(s, 1e-300), sig / (2.0 * np.maximum(s, 1e-300)))
        return s, err * ds
    if score_func == "softmax":
        z = np.exp(logits - logits.max(axis=-1, keepdims=True))
        s = z / z.sum(axis=-1, keepdims=True)
        # d s_i = s_i (d l_i - sum_j s_j d l_j)
        return s, s * (err + (s * err).sum(axis=-1, keepdims=True))
    raise ValueError(f"unknown scoring_func {score_func}")


def route_ties(x, weight, bias, *, top_k: int, n_group: int = 1, topk_group: int = 1,
               eval_ulps: float = 8.0, lam: float = 10.0, score_func: str = "sigmoid"):
    """Return (sel_tie [T] bool, order_tie [T] bool).

    sel_tie: the SET of selected experts is not decidable in fp32.
    order_tie: the set is decidable but the descending order of two selected
    experts is not (compare as sets there).
    """
    xd = torch.as_tensor(x).to(torch.float64).numpy()
    wd = torch.as_tensor(weight).to(torch.float64).numpy()
    b = 0.0 if bias is None else torch.as_tensor(bias).to(torch.float64).numpy()
    k_dim = xd.shape[1]
    u = 2.0 ** -24
    logits = xd @ wd.T
    err = lam * u * np.sqrt(k_dim / 2.0) * np.sqrt((xd * xd) @ (wd * wd).T)
    s, ds = _scores_and_error(logits, err, score_func)
    sel = s + b
    dsel = ds + eval_ulps * np.spacing(np.abs(sel).astype(np.float32)).astype(np.float64)
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


def salted_hash_ids(token_ids, layer_idx: int, n_experts: int) -> np.ndarray:
    """Table-less hash routing ids (layers.py:180-184) as torch evaluates them.

    ``token_ids.int()`` truncates to int32; ``+ salt`` and ``* 2654435761``
    wrap modulo 2^32 on the int32 tensor; the literal ``2**31`` becomes the
    int32 scalar -2^31, and ``%`` is the floor modulo (sign of the divisor).
    Pinned against the reference's own outputs in tests/golden/routing.npz.
    """
    salt = layer_idx * 2654435761 % (2 ** 31)  # Python integers, as in the reference
    out = []
    for tid in np.asarray(token_ids, dtype=np.int64).reshape(-1).tolist():
        t32 = ((tid + 2 ** 31) % 2 ** 32) - 2 ** 31          # .int()
        a = ((t32 + salt + 2 ** 31) % 2 ** 32) - 2 ** 31      # int32 add
        h = ((a * 2654435761 + 2 ** 31) % 2 ** 32) - 2 ** 31  # int32 multiply
        r = h - (h // -(2 ** 31)) * -(2 ** 31)                # h % (-2^31), floor modulo
        out.append(r % n_experts)                              # floor modulo, E > 0
    return np.array(out, dtype=np.int64).reshape(-1, 1)


def hash_route(x, weight, tid2eid, token_ids=None, *, n_experts: int, layer_idx: int = 0,
               score_func: str = "sqrtsoftplus", route_scale: float = 1.0, norm_topk_prob=None):
    """HashRouter.forward (layers.py:171-197) -> (weights fp32 [T, k], idx int64 [T, k]).

    ``tid2eid`` None: the salted hash (k = 1, weight = route_scale).  Otherwise
    ``[V]`` or ``[V, k]``: ids ``tid2eid[token_ids mod V]``; weights the scores
    gathered at the ids, normalised (``clamp_min(1e-9)``) unless the score is
    softmax (``norm_topk_prob`` overrides), times ``route_scale``.
    """
    n = int(torch.as_tensor(x).shape[0])
    tok = np.arange(n, dtype=np.int64) if token_ids is None else np.asarray(token_ids, dtype=np.int64).reshape(-1)
    if tid2eid is None:
        idx = torch.from_numpy(salted_hash_ids(tok, layer_idx, n_experts))
        return torch.full((n, 1), float(route_scale), dtype=torch.float32), idx
    table = torch.as_tensor(np.asarray(tid2eid)).long()
    idx = table[torch.from_numpy(tok) % table.shape[0]].reshape(n, -1)
    logits = F.linear(torch.as_tensor(x).float(), torch.as_tensor(weight, dtype=torch.float32))
    s = router_scores(logits, score_func)
    w = s.gather(-1, idx)
    norm = score_func != "softmax" if norm_topk_prob is None else norm_topk_prob
    if norm:
        w = w / w.sum(-1, keepdim=True).clamp_min(1e-9)
    return (w * route_scale).float(), idx
