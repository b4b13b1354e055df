"""Generate the golden fixtures in this directory by running the REFERENCE itself.

Run in a container that has the reference checkout (read-only) at
``$MOSAIC_REFERENCE`` (default: a ``reference`` checkout beside this
repository):

    python tests/golden/gen_golden.py

It imports fazin-ahamed/Mosaic's own functions and records their outputs on
seeded inputs:

* ``mosaicvm/kernels/fp4_source.py``: ``pack_mxfp4_nk``, ``act_quant_ref``,
  ``reference_fp4_linear_source_semantics``;
* ``mosaicvm/runtime/fp8.py``: ``dequant_fp4``;
* ``.mosaicvm/source/inference_model.py``: ``Gate`` with ``score_func``
  "sigmoid", "softmax" and "sqrtsoftplus", score-based and on hash layers;
* ``mosaicvm/model/layers.py``: ``HyperConnections`` (pre / post) and ``RMSNorm``;
* ``mosaicvm/model/layers.py``: ``Router`` (sqrtsoftplus) and ``HashRouter``
  (with a table, and the salted fallback with ``MOSAICVM_EXACT_TARGET=0``);
* ``mosaicvm/model/layers.py``: ``grouped_expert_forward`` and
  ``SharedExpertMLP`` on dequantised MXFP4 weights (the bf16 MoE path).

The GPU box never runs this script; the tests only read the ``.npz`` files.
Large weight banks are not stored: the fixture stores the generator seed and
a SHA-256 of the packed bytes so the tests can regenerate and verify them.
"""
from __future__ import annotations

import hashlib
import importlib.util
import math
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REF = os.environ.get("MOSAIC_REFERENCE", str(HERE.parents[2] / "reference"))
sys.path.insert(0, REF)
sys.path.insert(0, str(HERE.parents[1]))

from mosaicvm.kernels.fp4_source import (  # noqa: E402
    act_quant_ref,
    pack_mxfp4_nk,
    reference_fp4_linear_source_semantics,
)
from mosaicvm.model.config import V4Config  # noqa: E402
from mosaicvm.model.layers import (  # noqa: E402
    HashRouter,
    HyperConnections,
    RMSNorm,
    Router,
    SharedExpertMLP,
    grouped_expert_forward,
)
from mosaicvm.runtime.fp8 import dequant_fp4  # noqa: E402

from tests.golden.recipes import (  # noqa: E402
    GATE_CASES,
    HC_ORACLE_CASES,
    MOE_CASES,
    ROUTING_CASES,
    SALTED_CASES,
    edge_weight_matrix,
    make_gate_case,
    make_hash_case,
    make_hc_case,
    make_moe_case,
    salted_token_ids,
)


def _sha(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def _vendored_gate_module():
    src = Path(REF) / ".mosaicvm" / "source"
    spec = importlib.util.spec_from_file_location("kernel", src / "inference_kernel.py")
    km = importlib.util.module_from_spec(spec)
    sys.modules["kernel"] = km
    spec.loader.exec_module(km)
    spec = importlib.util.spec_from_file_location("inference_model", src / "inference_model.py")
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


def gen_formats():
    g = torch.Generator().manual_seed(1234)
    out = {}
    w = torch.randn(64, 256, generator=g) * 0.02
    p, s = pack_mxfp4_nk(w)
    out["pack_w"] = w.numpy()
    out["pack_packed"] = p.numpy()
    out["pack_scale"] = s.view(torch.uint8).numpy()
    we = edge_weight_matrix()
    p, s = pack_mxfp4_nk(we)
    out["edge_w"] = we.numpy()
    out["edge_packed"] = p.numpy()
    out["edge_scale"] = s.view(torch.uint8).numpy()
    out["edge_dequant"] = dequant_fp4(p, s.view(torch.uint8).view(torch.float8_e8m0fnu),
                                      we.shape[0], we.shape[1]).float().numpy()
    # act_quant: random rows plus the reference's own pow2 boundary cases
    x = torch.randn(6, 512, generator=g).to(torch.bfloat16)
    q, sa = act_quant_ref(x)
    out["act_x"] = x.float().numpy()
    out["act_q"] = q.view(torch.uint8).numpy()
    out["act_s"] = sa.numpy()
    vals = [0.0, 1e-5, -1e-5, 1e-4, 448.0, -448.0, 1.0, 2.0 ** -60]
    vals += [2.0 ** e * 448.0 for e in (-10, -1, 0, 4)]
    vals += [2.0 ** e * 448.0 * 1.0000001 for e in (-10, -1, 0, 4)]
    xb = torch.zeros(1, 128 * len(vals))
    for i, v in enumerate(vals):
        if v != 0.0:
            xb[0, 128 * i + 7] = v
    xb = xb.to(torch.bfloat16)
    q, sa = act_quant_ref(xb)
    out["actb_x"] = xb.float().numpy()
    out["actb_q"] = q.view(torch.uint8).numpy()
    out["actb_s"] = sa.numpy()
    # source-exact FP4 linear
    for name, (m, k, n) in {"lin_a": (1, 128, 16), "lin_b": (8, 256, 32), "lin_c": (5, 512, 64)}.items():
        wl = (torch.randn(n, k, generator=g) / math.sqrt(k)).to(torch.bfloat16)
        xl = torch.randn(m, k, generator=g).to(torch.bfloat16)
        p, s = pack_mxfp4_nk(wl)
        y = reference_fp4_linear_source_semantics(xl, p, s)
        out[name + "_x"] = xl.float().numpy()
        out[name + "_packed"] = p.numpy()
        out[name + "_scale"] = s.view(torch.uint8).numpy()
        out[name + "_y"] = y.float().numpy()
    np.savez_compressed(HERE / "formats.npz", **out)


def gen_router():
    m = _vendored_gate_module()
    out = {}
    for name, (t, h, e, k, scale) in GATE_CASES.items():
        args = m.ModelArgs(dim=h, n_routed_experts=e, n_activated_experts=k,
                           score_func="sigmoid", route_scale=scale, n_hash_layers=0)
        gate = m.Gate(0, args)
        x, wt, bias = make_gate_case(t, h, e, seed=77 + e)
        with torch.no_grad():
            gate.weight.copy_(wt)
            gate.bias.copy_(bias)
            w, idx = gate(x, None)
        out[name + "_sha"] = np.frombuffer(_sha(x.float().numpy(), wt.numpy(), bias.numpy()).encode(),
                                           dtype=np.uint8)
        out[name + "_weights"] = w.float().numpy()
        out[name + "_idx"] = idx.numpy().astype(np.int64)
        out[name + "_meta"] = np.array([t, h, e, k, scale])
    np.savez_compressed(HERE / "router.npz", **out)


def gen_routing():
    m = _vendored_gate_module()
    out = {}
    for name, c in ROUTING_CASES.items():
        t, h, e, k = c["T"], c["H"], c["E"], c["k"]
        src = c["src"]
        with torch.no_grad():
            if src in ("router", "gate"):
                x, wt, bias = make_gate_case(t, h, e, seed=c["seed"])
                if src == "router":
                    cfg = V4Config(hidden_size=h, n_routed_experts=e, num_experts_per_tok=k,
                                   scoring_func=c["score"], routed_scaling_factor=c["scale"])
                    mod = Router(cfg)
                    mod.weight.copy_(wt)
                    mod.e_score_correction_bias.copy_(bias)
                    w, idx = mod(x)
                else:
                    args = m.ModelArgs(dim=h, n_routed_experts=e, n_activated_experts=k, score_func=c["score"],
                                       route_scale=c["scale"], n_hash_layers=0)
                    gate = m.Gate(0, args)
                    gate.weight.copy_(wt)
                    gate.bias.copy_(bias)
                    w, idx = gate(x, None)
                inputs = (x.float().numpy(), wt.numpy(), bias.numpy())
            else:
                x, wt, table, tok = make_hash_case(t, h, e, None if src == "hash1d" else k, c["vocab"], c["seed"],
                                                   in_table=src == "gate_hash")
                if src == "gate_hash":
                    args = m.ModelArgs(dim=h, n_routed_experts=e, n_activated_experts=k, score_func=c["score"],
                                       route_scale=c["scale"], n_hash_layers=1, vocab_size=c["vocab"])
                    gate = m.Gate(0, args)
                    gate.weight.copy_(wt)
                    gate.tid2eid.copy_(table)
                    w, idx = gate(x, tok)
                else:
                    cfg = V4Config(hidden_size=h, n_routed_experts=e, num_experts_per_tok=k,
                                   scoring_func=c["score"], routed_scaling_factor=c["scale"])
                    hr = HashRouter(cfg, 3)
                    hr.weight.copy_(wt)
                    hr.tid2eid = table
                    w, idx = hr(x, tok)
                inputs = (x.float().numpy(), wt.numpy(), table.numpy(), tok.numpy())
        out[name + "_sha"] = np.frombuffer(_sha(*inputs).encode(), dtype=np.uint8)
        out[name + "_weights"] = w.float().numpy()
        out[name + "_idx"] = idx.numpy().astype(np.int64)
    # table-less salted hash (the reference raises under the exact target)
    tok = salted_token_ids()
    os.environ["MOSAICVM_EXACT_TARGET"] = "0"
    try:
        for e, layer_idx in SALTED_CASES:
            cfg = V4Config(hidden_size=64, n_routed_experts=e, num_experts_per_tok=1)
            w, idx = HashRouter(cfg, layer_idx)(torch.zeros(tok.numel(), 64), tok)
            out[f"salted_{e}_{layer_idx}_idx"] = idx.numpy().astype(np.int64)
            out[f"salted_{e}_{layer_idx}_weights"] = w.float().numpy()
    finally:
        del os.environ["MOSAICVM_EXACT_TARGET"]
    out["salted_tokens"] = tok.numpy()
    np.savez_compressed(HERE / "routing.npz", **out)


def gen_hc():
    out = {}
    for name, (b, s_, hc, d, iters, seed) in HC_ORACLE_CASES.items():
        x, fn, base, scale, norm_w, y = make_hc_case(b, s_, hc, d, seed)
        cfg = V4Config(hidden_size=d, hc_mult=hc, hc_sinkhorn_iters=iters)
        mod = HyperConnections(cfg, "ffn")
        norm = RMSNorm(d, cfg.rms_norm_eps)
        with torch.no_grad():
            mod.fn.copy_(fn)
            mod.base.copy_(base)
            mod.scale.copy_(scale)
            norm.weight.copy_(norm_w)
            y_pre, post, comb = mod.pre(x)
            y_norm = norm(y_pre)
            q, qs = act_quant_ref(y_norm.reshape(-1, d))
            out_post = mod.post(y, x, post, comb)
        out[name + "_y_pre"] = y_pre.float().numpy()
        out[name + "_post"] = post.numpy()
        out[name + "_comb"] = comb.numpy()
        out[name + "_y_norm"] = y_norm.float().numpy()
        out[name + "_q"] = q.view(torch.uint8).numpy()
        out[name + "_qs"] = qs.numpy()
        out[name + "_out_post"] = out_post.float().numpy()
    np.savez_compressed(HERE / "hc.npz", **out)


def gen_moe():
    out = {}
    for name, spec in MOE_CASES.items():
        case = make_moe_case(**spec)
        cfg = case["cfg"]
        e, h, inter = cfg["E"], cfg["H"], cfg["I"]
        packs = []
        wg = torch.empty(e, h, inter)
        wu = torch.empty(e, h, inter)
        wd = torch.empty(e, inter, h)
        gu_p, gu_s, dn_p, dn_s = [], [], [], []
        for ei in range(e + 1):
            pg, sg = pack_mxfp4_nk(case["w_gu"][ei])
            pd, sd = pack_mxfp4_nk(case["w_dn"][ei])
            gu_p.append(pg)
            gu_s.append(sg)
            dn_p.append(pd)
            dn_s.append(sd)
            dgu = dequant_fp4(pg, sg, 2 * inter, h)
            ddn = dequant_fp4(pd, sd, h, inter)
            if ei < e:
                wg[ei] = dgu[:inter].float().T
                wu[ei] = dgu[inter:].float().T
                wd[ei] = ddn.float().T
            else:
                shared = SharedExpertMLP(h, inter, cfg["swiglu_limit"]).to(torch.bfloat16)
                with torch.no_grad():
                    shared.gate_proj.weight.copy_(dgu[:inter])
                    shared.up_proj.weight.copy_(dgu[inter:])
                    shared.down_proj.weight.copy_(ddn)
        packs = [torch.stack(gu_p).numpy(), torch.stack(gu_s).view(torch.uint8).numpy(),
                 torch.stack(dn_p).numpy(), torch.stack(dn_s).view(torch.uint8).numpy()]
        x = case["x"]
        w, idx = case["weights"], case["idx"]
        with torch.no_grad():
            routed = grouped_expert_forward(x, w, idx, (wg.to(torch.bfloat16), wu.to(torch.bfloat16)),
                                            wd.to(torch.bfloat16), e, swiglu_limit=cfg["swiglu_limit"])
            ysh = shared(x)
            y = ysh + routed
        out[name + "_sha"] = np.frombuffer(_sha(*packs).encode(), dtype=np.uint8)
        out[name + "_weights"] = w.float().numpy()
        out[name + "_idx"] = idx.numpy().astype(np.int64)
        out[name + "_routed"] = routed.float().numpy()
        out[name + "_shared"] = ysh.float().numpy()
        out[name + "_y"] = y.float().numpy()
    np.savez_compressed(HERE / "moe.npz", **out)


if __name__ == "__main__":
    gen_formats()
    gen_router()
    gen_routing()
    gen_hc()
    gen_moe()
    for f in sorted(HERE.glob("*.npz")):
        print(f.name, f.stat().st_size)
