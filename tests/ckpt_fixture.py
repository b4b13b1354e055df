"""Test-only writer of small safetensors checkpoints in the V4 tensor contract.

Names and formats follow mosaicvm/runtime/streaming_model.py:30-100,150-205:
``layers.<i>.ffn.experts.<e>.w{1,3,2}.{weight,scale}`` (packed E2M1 uint8
``[N, K/2]``, E8M0 ``[N, K/32]``), ``ffn.shared_experts.*`` (same format
here), ``ffn.gate.weight`` bf16 ``[E, H]``, ``ffn.gate.bias`` fp32 on routed
layers, ``ffn.gate.tid2eid`` int32 ``[V, k]`` on hash layers.  Weights are
packed with the oracle's packer (pinned to the reference's
``pack_mxfp4_nk``); files are written with the ``safetensors`` package, so
the loader's own header parser is checked against an independent writer.
"""
from __future__ import annotations

import json
import math
from pathlib import Path

import numpy as np
import torch

from oracle import formats as fm

CKPT = dict(H=256, I=128, E=8, k=2, layers=2, hash_layers=1, vocab=50)


def _packed(w: torch.Tensor):
    p, s = fm.pack_mxfp4_nk(w.numpy())
    return torch.from_numpy(p), torch.from_numpy(s).view(torch.float8_e8m0fnu)


def make_checkpoint(root: Path, *, seed: int = 0, shards: int = 2, shared_format: str = "fp4",
                    drop: tuple = (), extra: dict | None = None, config_extra: dict | None = None) -> dict:
    """Write a 2-layer checkpoint under ``root``; return the tensors written (CPU)."""
    from safetensors.torch import save_file

    c = CKPT
    h, inter, e = c["H"], c["I"], c["E"]
    g = torch.Generator().manual_seed(seed)
    tensors = {}
    for li in range(c["layers"]):
        pre = f"layers.{li}."
        experts = [f"{pre}ffn.experts.{i}." for i in range(e)] + [f"{pre}ffn.shared_experts."]
        for j, base in enumerate(experts):
            w1 = torch.randn(inter, h, generator=g) * 0.02
            w3 = torch.randn(inter, h, generator=g) * 0.02
            w2 = torch.randn(h, inter, generator=g) * 0.02
            for name, w in (("w1", w1), ("w3", w3), ("w2", w2)):
                if j == e and shared_format == "bf16":
                    tensors[base + name + ".weight"] = w.to(torch.bfloat16)
                    continue
                p, s = _packed(w)
                tensors[base + name + ".weight"] = p
                tensors[base + name + ".scale"] = s
        tensors[pre + "ffn.gate.weight"] = (torch.randn(e, h, generator=g) / math.sqrt(h)).to(torch.bfloat16)
        if li < c["hash_layers"]:
            tensors[pre + "ffn.gate.tid2eid"] = torch.randint(0, e, (c["vocab"], c["k"]), generator=g,
                                                              dtype=torch.int32)
        else:
            tensors[pre + "ffn.gate.bias"] = torch.randn(e, generator=g) * 0.01
    for name in drop:
        tensors.pop(name)
    tensors.update(extra or {})
    root.mkdir(parents=True, exist_ok=True)
    names = sorted(tensors)
    if shards == 1:
        save_file({n: tensors[n].contiguous() for n in names}, str(root / "model.safetensors"))
    else:
        weight_map = {}
        for s in range(shards):
            part = names[s::shards]
            fname = f"model-{s + 1:05d}-of-{shards:05d}.safetensors"
            save_file({n: tensors[n].contiguous() for n in part}, str(root / fname))
            weight_map.update({n: fname for n in part})
        (root / "model.safetensors.index.json").write_text(json.dumps({"metadata": {}, "weight_map": weight_map}))
    config = {"dim": h, "moe_inter_dim": inter, "n_routed_experts": e, "n_activated_experts": c["k"],
              "score_func": "sqrtsoftplus", "route_scale": 1.5, "num_hash_layers": c["hash_layers"],
              "n_layers": c["layers"], "swiglu_limit": 10.0, "vocab_size": c["vocab"]}
    config.update(config_extra or {})
    (root / "config.json").write_text(json.dumps(config))
    return tensors


def expected_bank(tensors: dict, layer: int):
    """Reference-layout bank arrays of a layer: (gu_packed, gu_scale, dn_packed, dn_scale), shared last."""
    e = CKPT["E"]
    pre = f"layers.{layer}."
    bases = [f"{pre}ffn.experts.{i}." for i in range(e)] + [f"{pre}ffn.shared_experts."]

    def u8(t):
        return t.view(torch.uint8).numpy()

    gu_p = np.stack([np.concatenate([u8(tensors[b + "w1.weight"]), u8(tensors[b + "w3.weight"])]) for b in bases])
    gu_s = np.stack([np.concatenate([u8(tensors[b + "w1.scale"]), u8(tensors[b + "w3.scale"])]) for b in bases])
    dn_p = np.stack([u8(tensors[b + "w2.weight"]) for b in bases])
    dn_s = np.stack([u8(tensors[b + "w2.scale"]) for b in bases])
    return gu_p, gu_s, dn_p, dn_s
