"""Test-only CPU restatement of the expert-parallel kernels, on the oracle.

``ExpertParallelMoELayer`` reaches its kernels through a ``kernels`` object.
These CPU versions of route / dispatch / per-row expert pass / combine follow
the CUDA kernels' data contracts (send-row layout with its 16-byte tail,
expert-sorted row order, partial dtypes), so ``gloo`` ranks on the CPU can
check the layer's host-side orchestration: split sizes, exchange order and
reassembly.  They are never used by the package.
"""
from __future__ import annotations

import numpy as np
import torch

from oracle.formats import act_quant_ref
from oracle.moe import expert_bf16, expert_fp8
from oracle.router import hash_route, route


class CpuEPKernels:
    """``local_bank``: oracle dict of this rank's experts (``gu_packed`` [n, 2I, H/2],
    ``gu_scale``, ``dn_packed``, ``dn_scale``), the shared expert last."""

    def __init__(self, router_w, bias, cfg, local_bank: dict):
        self.router_w = router_w
        self.bias = bias
        self.cfg = cfg
        self.bank = local_bank

    def route(self, router, x):
        c = self.cfg
        return route(x, self.router_w, self.bias, top_k=c.num_experts_per_tok, n_group=c.n_group,
                     topk_group=c.topk_group, route_scale=c.routed_scaling_factor, norm_topk_prob=c.norm_topk_prob)

    def route_hash(self, router, x, token_ids):
        c = self.cfg
        tok = None if token_ids is None else token_ids.reshape(-1).numpy()
        return hash_route(x, self.router_w, router.tid2eid, tok, n_experts=c.n_routed_experts,
                          layer_idx=router.layer_idx, score_func=c.scoring_func, route_scale=c.routed_scaling_factor)

    def dispatch(self, dims, world, x, idx, w):
        t, k = idx.shape
        h = dims.hidden
        el = dims.n_experts // world
        flat = idx.reshape(-1).numpy()
        tok = np.repeat(np.arange(t), k)
        order = np.lexsort((tok, flat))  # expert id, then token: the layout kernel's row order
        a = t * k
        send = torch.zeros(a, 2 * h + 16, dtype=torch.uint8)
        xb = x.contiguous().view(torch.uint8).reshape(t, 2 * h)
        send[:, :2 * h] = xb[torch.from_numpy(tok[order])]
        e_sorted = flat[order]
        dest = e_sorted // el
        tail = np.zeros((a, 4), dtype=np.int32)
        tail[:, 0] = e_sorted - dest * el
        tail[:, 1] = w.reshape(-1).float().numpy()[order].view(np.int32)
        tail[:, 2] = tok[order]
        tail[:, 3] = dest
        send[:, 2 * h:] = torch.from_numpy(tail.view(np.uint8).reshape(a, 16))
        counts = torch.from_numpy(np.bincount(dest, minlength=world).astype(np.int32))
        return send, counts, {"order": order, "t": t, "k": k}

    def _experts(self, x, ids, wts, out):
        n_routed = self.bank["gu_packed"].shape[0] - 1
        limit = self.cfg.swiglu_limit
        for e in np.unique(ids):
            rows = np.nonzero(ids == e)[0]
            args = (self.bank["gu_packed"][e], self.bank["gu_scale"][e], self.bank["dn_packed"][e],
                    self.bank["dn_scale"][e])
            if self.cfg.act_mode == "bf16":
                y = expert_bf16(x[rows], *args, wts[rows], limit, shared=(e == n_routed))
            else:
                xq, xs = act_quant_ref(x[rows])
                y = expert_fp8(xq, xs, *args, wts[rows], limit)
            out[torch.from_numpy(rows)] = torch.from_numpy(np.ascontiguousarray(y)).to(out.dtype)

    def expert_rows(self, dims_local, bank, recv, out):
        h = dims_local.hidden
        x = recv[:, :2 * h].contiguous().view(torch.bfloat16).float().numpy()
        tail = recv[:, 2 * h:].contiguous().view(torch.int32).numpy()
        self._experts(x, tail[:, 0].copy(), tail[:, 1].copy().view(np.float32), out)

    def shared_rows(self, dims_local, bank, x, out):
        n = x.shape[0]
        self._experts(x.float().numpy(), np.full(n, dims_local.n_experts), np.ones(n, dtype=np.float32), out)

    def combine(self, dims, partials, ws, y):
        order, t, k = ws["order"], ws["t"], ws["k"]
        row_of = np.empty(t * k, dtype=np.int64)
        row_of[order] = np.arange(t * k)
        rows = np.sort(row_of.reshape(t, k), axis=1)  # ascending row = ascending expert id
        p = partials.float().numpy()
        acc = np.zeros((t, dims.hidden), dtype=np.float32)
        for s in range(k):
            acc = acc + p[rows[:, s]]
        routed = torch.from_numpy(acc).to(torch.bfloat16).float()
        if dims.has_shared:
            routed = routed + partials[t * k:t * k + t].float()
        y.copy_(routed.to(torch.bfloat16))
