"""Checkpoint loader without a GPU: the safetensors header parser against an
independent writer, config aliases, and the exact tensor contract
(mosaicvm/runtime/streaming_model.py:30-100)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from mosaic_b200 import ExactContractError
from mosaic_b200.checkpoint import ShardIndex, moe_config_from_checkpoint, validate_exact_v4_tensors
from tests.ckpt_fixture import CKPT, make_checkpoint


@pytest.mark.parametrize("shards", [1, 3])
def test_index_reads_every_tensor_bit_exact(tmp_path, shards):
    tensors = make_checkpoint(tmp_path, shards=shards)
    idx = ShardIndex(tmp_path)
    assert sorted(idx.keys()) == sorted(tensors)
    for name, t in tensors.items():
        dt, shape = idx.meta(name)
        assert tuple(shape) == tuple(t.shape), name
        raw = idx.array(name)
        want = t.contiguous().view(torch.uint8).numpy().reshape(-1)
        assert np.array_equal(np.ascontiguousarray(raw).reshape(-1).view(np.uint8), want), name
        got = idx.tensor(name)
        if t.dtype == torch.float8_e8m0fnu:
            assert dt == "F8_E8M0" and torch.equal(got, t.view(torch.uint8))
        else:
            assert got.dtype == t.dtype and torch.equal(got, t), name


def test_index_missing_checkpoint(tmp_path):
    with pytest.raises(FileNotFoundError):
        ShardIndex(tmp_path)


def test_config_aliases(tmp_path):
    make_checkpoint(tmp_path, shards=1)
    cfg, n_hash, raw = moe_config_from_checkpoint(tmp_path)
    c = CKPT
    assert (cfg.hidden_size, cfg.moe_intermediate_size, cfg.n_routed_experts) == (c["H"], c["I"], c["E"])
    assert cfg.num_experts_per_tok == c["k"] and cfg.scoring_func == "sqrtsoftplus"
    assert cfg.routed_scaling_factor == 1.5 and cfg.swiglu_limit == 10.0 and cfg.norm_topk_prob
    assert (cfg.n_group, cfg.topk_group) == (1, 1) and n_hash == c["hash_layers"]


def test_exact_contract_accepts_the_fixture(tmp_path):
    make_checkpoint(tmp_path)
    idx = ShardIndex(tmp_path)
    cfg, n_hash, _ = moe_config_from_checkpoint(tmp_path)
    for li in range(CKPT["layers"]):
        validate_exact_v4_tensors(idx, f"layers.{li}.", li, cfg, n_hash)


@pytest.mark.parametrize("mutation,message", [
    (dict(extra={"layers.1.ffn.experts.0.w1.weight": torch.zeros(128, 256)}), "w1.weight: dtype F32, the exact path needs I8 or U8"),
    (dict(extra={"layers.1.ffn.experts.0.w2.weight": torch.zeros(256, 32, dtype=torch.uint8)}), "w2.weight: shape \\(256, 32\\), the exact path needs"),
    (dict(drop=("layers.1.ffn.experts.0.w3.scale",)), "layers.1.ffn.experts.0.w3.scale: not in the checkpoint"),
    (dict(extra={"layers.1.ffn.experts.0.w1.scale": torch.zeros(128, 8)}), "w1.scale: dtype F32, the exact path needs F8_E8M0"),
    (dict(drop=("layers.1.ffn.gate.bias",)), "layers.1.ffn.gate.bias: not in the checkpoint"),
    (dict(extra={"layers.0.ffn.gate.bias": torch.zeros(8)}), "hash-routed layer takes no score bias"),
    (dict(drop=("layers.0.ffn.gate.tid2eid",)), "layers.0.ffn.gate.tid2eid: not in the checkpoint"),
])
def test_exact_contract_violations(tmp_path, mutation, message):
    make_checkpoint(tmp_path, **mutation)
    idx = ShardIndex(tmp_path)
    cfg, n_hash, _ = moe_config_from_checkpoint(tmp_path)
    layer = 0 if "layers.0" in str(mutation) else 1
    with pytest.raises(ExactContractError, match=message):
        validate_exact_v4_tensors(idx, f"layers.{layer}.", layer, cfg, n_hash)


def test_exact_contract_missing_gate_weights(tmp_path):
    e = CKPT["E"]
    drop = tuple(f"layers.1.ffn.experts.{i}.w1.weight" for i in range(e))
    make_checkpoint(tmp_path, drop=drop)
    idx = ShardIndex(tmp_path)
    cfg, n_hash, _ = moe_config_from_checkpoint(tmp_path)
    with pytest.raises(ExactContractError, match=f"layers.1.ffn.experts.{e - 1}.w1.weight: not in the checkpoint"):
        validate_exact_v4_tensors(idx, "layers.1.", 1, cfg, n_hash)


def test_exact_contract_no_experts(tmp_path):
    e = CKPT["E"]
    drop = tuple(f"layers.1.ffn.experts.{i}.{w}.{t}" for i in range(e) for w in ("w1", "w2", "w3")
                 for t in ("weight", "scale"))
    make_checkpoint(tmp_path, drop=drop)
    idx = ShardIndex(tmp_path)
    cfg, n_hash, _ = moe_config_from_checkpoint(tmp_path)
    with pytest.raises(ExactContractError, match="no routed expert tensors") as info:
        validate_exact_v4_tensors(idx, "layers.1.", 1, cfg, n_hash)
    assert "experts.0.w1" not in str(info.value)
