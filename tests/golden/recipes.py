"""Seeded input recipes shared by the golden generator and the tests.

Everything is drawn from ``torch.Generator`` on the CPU, so the same seed gives
the same tensors here and on the GPU box.
"""
from __future__ import annotations

import math

import torch

# Small MoE cases (the BASELINE small config S and variants of it).
MOE_CASES = {
    # S: H 512, 32 routed + 1 shared, I 256, 4 groups / top-2 groups, top-4, 64 tokens
    "S": dict(T=64, H=512, I=256, E=32, k=4, n_group=4, topk_group=2, scale=2.5,
              swiglu_limit=0.0, seed=11),
    # same with the SwiGLU clamp the reference exercises (layers.py:213-216)
    "S_clamp": dict(T=24, H=512, I=256, E=32, k=4, n_group=4, topk_group=2, scale=2.5,
                    swiglu_limit=10.0, seed=12, x_mult=6.0, w_std=0.2),
    # tiny ragged case: few tokens, many experts
    "tiny": dict(T=3, H=256, I=128, E=16, k=2, n_group=1, topk_group=1, scale=1.0,
                 swiglu_limit=0.0, seed=13),
}


def edge_weight_matrix() -> torch.Tensor:
    """[16, 64] weights hitting E2M1 rounding ties, saturation and scale edges."""
    rows = []
    base = torch.tensor([0.0, 0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0,
                         6.0, 7.0, 0.1, 0.3, 0.6, 0.9, 1.1, 2.9])
    for r in range(16):
        v = torch.cat([base, -base]) * (2.0 ** (r - 8))
        if r == 3:
            v = torch.zeros(32)
        if r == 5:
            v = v * 1e-30
        rows.append(torch.cat([v, v.flip(0) * 3.0]))
    return torch.stack(rows).float()


GATE_CASES = {"gate_s": (64, 512, 32, 4, 2.5), "gate_v3": (16, 7168, 256, 8, 2.5)}


def make_gate_case(t, h, e, seed):
    """Seeded router inputs: W U(-1/sqrt(h), 1/sqrt(h)) fp32 [e, h], bias N(0, 0.01), x bf16 [t, h]."""
    g = torch.Generator().manual_seed(seed)
    bound = 1.0 / math.sqrt(h)
    wt = (torch.rand(e, h, generator=g) * 2 - 1) * bound
    bias = torch.randn(e, generator=g) * 0.01
    x = torch.randn(t, h, generator=g).to(torch.bfloat16)
    return x, wt, bias


def make_moe_case(T, H, I, E, k, n_group, topk_group, scale, swiglu_limit, seed,
                  x_mult: float = 1.0, w_std: float = 0.02):
    """Seeded MoE-layer inputs: router, expert weights (fp32, unpacked) and tokens.

    Returns a dict with ``cfg``, ``x`` (bf16 [T, H]), ``router_w`` (fp32 [E, H],
    U(-1/sqrt(H), 1/sqrt(H))), ``bias`` (fp32 [E], N(0, 0.01)), ``w_gu``
    (list of E+1 fp32 [2I, H], gate rows then up rows; index E is the shared
    expert), ``w_dn`` (list of E+1 fp32 [H, I]) and the routing ``weights``/``idx``
    computed by the oracle router.
    """
    g = torch.Generator().manual_seed(seed)
    bound = 1.0 / math.sqrt(H)
    router_w = (torch.rand(E, H, generator=g) * 2 - 1) * bound
    bias = torch.randn(E, generator=g) * 0.01
    w_gu = [torch.randn(2 * I, H, generator=g) * w_std for _ in range(E + 1)]
    w_dn = [torch.randn(H, I, generator=g) * w_std for _ in range(E + 1)]
    x = (torch.randn(T, H, generator=g) * x_mult).to(torch.bfloat16)
    from oracle.router import route

    weights, idx = route(x, router_w, bias, top_k=k, n_group=n_group, topk_group=topk_group,
                         route_scale=scale)
    cfg = dict(T=T, H=H, I=I, E=E, k=k, n_group=n_group, topk_group=topk_group, scale=scale,
               swiglu_limit=swiglu_limit)
    return dict(cfg=cfg, x=x, router_w=router_w, bias=bias, w_gu=w_gu, w_dn=w_dn,
                weights=weights, idx=idx)


# Router variants recorded from the reference into routing.npz:
#   src "router": mosaicvm/model/layers.py Router (scoring_func, norm_topk_prob, no groups)
#   src "gate":   vendored .mosaicvm/source/inference_model.py Gate (score-based)
#   src "gate_hash": the same Gate on a hash layer (tid2eid[input_ids], ids inside the table)
#   src "hash" / "hash1d": layers.py HashRouter with a [V, k] / [V] table, any token ids
ROUTING_CASES = {
    "router_v4_s": dict(src="router", T=64, H=512, E=32, k=6, score="sqrtsoftplus", scale=1.5, seed=21),
    "router_v4": dict(src="router", T=16, H=4096, E=256, k=6, score="sqrtsoftplus", scale=1.5, seed=22),
    "gate_softmax": dict(src="gate", T=48, H=512, E=64, k=6, score="softmax", scale=1.0, seed=23),
    "gate_sqrtsoftplus": dict(src="gate", T=48, H=512, E=64, k=6, score="sqrtsoftplus", scale=2.5, seed=24),
    "gate_hash_sqrtsoftplus": dict(src="gate_hash", T=40, H=512, E=32, k=6, score="sqrtsoftplus", scale=1.5,
                                   seed=25, vocab=97),
    "gate_hash_softmax": dict(src="gate_hash", T=40, H=512, E=32, k=4, score="softmax", scale=1.0, seed=26,
                              vocab=97),
    "hash_table": dict(src="hash", T=40, H=512, E=32, k=6, score="sqrtsoftplus", scale=1.5, seed=27, vocab=50),
    "hash_table_1d": dict(src="hash1d", T=40, H=512, E=32, k=1, score="sqrtsoftplus", scale=1.5, seed=28,
                          vocab=37),
    "hash_v4": dict(src="hash", T=16, H=4096, E=256, k=6, score="sqrtsoftplus", scale=1.5, seed=29, vocab=129280),
}

# Table-less hash routing (layers.py:180-184): (n_experts, layer_idx) pairs, one token-id vector.
SALTED_CASES = [(1, 0), (3, 1), (16, 2), (24, 7), (100, 42), (255, 1000), (256, 2), (256, 2 ** 31 - 1)]


def make_hash_case(T, H, E, k, vocab, seed, in_table: bool = False):
    """Router inputs of make_gate_case plus an int32 table [vocab, k] of ids in [0, E)
    (1-D when k is None) and int64 token ids [T]: inside [0, vocab) when
    ``in_table``, else spanning negatives, multiples of vocab and 2^40."""
    x, wt, _ = make_gate_case(T, H, E, seed)
    g = torch.Generator().manual_seed(seed + 500)
    shape = (vocab,) if k is None else (vocab, k)
    table = torch.randint(0, E, shape, generator=g, dtype=torch.int64).to(torch.int32)
    if in_table:
        tok = torch.randint(0, vocab, (T,), generator=g, dtype=torch.int64)
    else:
        tok = torch.randint(-3 * vocab, 3 * vocab, (T,), generator=g, dtype=torch.int64)
        edge = torch.tensor([0, vocab - 1, vocab, -1, -vocab, 2 ** 40 + 3, -(2 ** 40) - 5], dtype=torch.int64)
        tok[:edge.numel()] = edge
    return x, wt, table, tok


def salted_token_ids() -> torch.Tensor:
    """int64 token ids for the table-less hash: random 62-bit values plus int32 / int64 edges."""
    g = torch.Generator().manual_seed(31)
    rnd = torch.randint(-2 ** 62, 2 ** 62, (120,), generator=g, dtype=torch.int64)
    edge = torch.tensor([0, 1, -1, 2 ** 31 - 1, -2 ** 31, 2 ** 31, 2 ** 32 - 1, 2 ** 32, 2 ** 63 - 1, -2 ** 63],
                        dtype=torch.int64)
    return torch.cat([edge, rnd, torch.arange(64, dtype=torch.int64)])


# Hyper-connection + RMSNorm cases recorded from the reference into hc.npz:
# name: (batch, seq, hc_mult, D, sinkhorn iters, seed)
HC_CASES = {
    "hc_s": (2, 3, 4, 256, 20, 51),
    "hc_v4": (1, 4, 4, 4096, 20, 52),
    "hc_mult2": (1, 5, 2, 512, 7, 53),
}
# more residual-copy counts, pinning the oracle (CPU tests) on every hc the C ABI takes
HC_ORACLE_CASES = {
    **HC_CASES,
    "hc_mult1": (1, 3, 1, 256, 20, 54),
    "hc_mult3": (2, 2, 3, 384, 20, 55),
}


def make_hc_case(b, s, hc, d, seed):
    """Seeded hyper-connection inputs: x bf16 [b, s, hc, d] (~N(0,1)), fn fp32
    [(2+hc)*hc, hc*d] (~N(0, 0.01), the reference init), base ~N(0, 0.5), scale
    ~U(0.5, 1.5) [3], RMSNorm weight 1 + N(0, 0.1) [d], and a sub-layer output y
    bf16 [b, s, d] for the post-mix."""
    g = torch.Generator().manual_seed(seed)
    mix = (2 + hc) * hc
    x = torch.randn(b, s, hc, d, generator=g).to(torch.bfloat16)
    fn = torch.randn(mix, hc * d, generator=g) * 0.01
    base = torch.randn(mix, generator=g) * 0.5
    scale = torch.rand(3, generator=g) + 0.5
    norm_w = 1.0 + torch.randn(d, generator=g) * 0.1
    y = torch.randn(b, s, d, generator=g).to(torch.bfloat16)
    return x, fn, base, scale, norm_w, y
