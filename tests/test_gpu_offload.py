"""Expert offload on the GPU: layers whose experts stream from pinned host memory
through an LRU expert cache give outputs bit-identical to the resident layers
(logical ids in ascending global order, the resident combine order)."""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def _layers(n_layers, act_mode="bf16", hidden=512, inter=256, n_experts=32):
    from mosaic_b200 import MoEConfig, MoELayer
    from mosaic_b200 import synthetic

    cfg = MoEConfig(hidden_size=hidden, moe_intermediate_size=inter, n_routed_experts=n_experts,
                    num_experts_per_tok=4, n_group=4, topk_group=2, routed_scaling_factor=2.5, act_mode=act_mode)
    out = []
    for li in range(n_layers):
        layer = MoELayer(cfg, synthetic.make_bank(hidden, inter, n_experts, 100 + li))
        synthetic.make_router(layer, 100 + li)
        out.append(layer)
    return cfg, out


def _offloaded(cfg, resident, cache, layer_key):
    from mosaic_b200.offload import HostBank, OffloadedMoELayer

    off = OffloadedMoELayer(cfg, HostBank.from_bank(resident.bank), cache, layer_key=layer_key)
    off.router.weight.data = resident.router.weight.data
    off.router.e_score_correction_bias.data = resident.router.e_score_correction_bias.data
    return off


@pytest.mark.parametrize("act_mode", ["bf16", "fp8"])
def test_offloaded_layers_bit_identical(act_mode):
    from mosaic_b200 import ops
    from mosaic_b200 import synthetic
    from mosaic_b200.offload import ExpertCache

    cfg, res = _layers(3, act_mode)
    cache = ExpertCache(512, 256, capacity=40)  # < 3 layers x 33 experts: entries are replaced
    offs = [_offloaded(cfg, r, cache, li) for li, r in enumerate(res)]
    for step in range(2):
        x = synthetic.make_tokens(24, 512, 7 + step)
        for r, o in zip(res, offs):
            y_ref = r(x)
            y = o(x)
            torch.cuda.synchronize()
            assert torch.equal(o.last_idx, r.last_idx)
            assert torch.equal(y, y_ref)
            assert ops.read_error(o._ws.buf) == 0
    # each layer's experts replaced the previous layer's; the last layer's are still cached
    assert cache.misses > 0 and cache.hits == 0
    assert torch.equal(offs[-1](x), res[-1](x))
    assert cache.hits > 0


def test_offload_v3_decode_one_token():
    """V3 dimensions, one token (8 routed + the shared expert per layer), two layers
    sharing one host bank through a 12-expert cache."""
    from mosaic_b200 import synthetic
    from mosaic_b200.offload import ExpertCache, HostBank, OffloadedMoELayer

    layer, _ = synthetic.make_layer(tokens=1, seed=5, act_mode="bf16", n_experts=64)
    host = HostBank.from_bank(layer.bank)
    cache = ExpertCache(7168, 2048, capacity=12)
    offs = []
    for key in range(2):
        o = OffloadedMoELayer(layer.cfg, host, cache, layer_key=key)
        o.router.weight.data = layer.router.weight.data
        o.router.e_score_correction_bias.data = layer.router.e_score_correction_bias.data
        offs.append(o)
    for seed in range(3):
        x = synthetic.make_tokens(1, 7168, 50 + seed)
        y_ref = layer(x)
        for o in offs:
            assert torch.equal(o(x), y_ref)


def test_offload_hash_layer_and_capacity_check():
    from mosaic_b200 import HashMoELayer, MoEConfig
    from mosaic_b200 import synthetic
    from mosaic_b200.offload import ExpertCache, HostBank, OffloadedMoELayer

    cfg = MoEConfig(hidden_size=512, moe_intermediate_size=256, n_routed_experts=32, num_experts_per_tok=4,
                    n_group=1, topk_group=1, routed_scaling_factor=1.5, scoring_func="sqrtsoftplus")
    res = HashMoELayer(cfg, 2, synthetic.make_bank(512, 256, 32, 9))
    g = torch.Generator().manual_seed(3)
    res.hash_router.weight.data = (torch.randn(32, 512, generator=g) / 512 ** 0.5).cuda()
    res.hash_router.tid2eid = torch.randint(0, 32, (100, 4), generator=g, dtype=torch.int32)
    cache = ExpertCache(512, 256, capacity=33)
    off = OffloadedMoELayer(cfg, HostBank.from_bank(res.bank), cache, layer_idx=2)
    off.hash_router.weight.data = res.hash_router.weight.data
    off.hash_router.tid2eid = res.hash_router.tid2eid
    x = synthetic.make_tokens(16, 512, 3)
    tok = torch.randint(0, 1000, (16,), generator=g).cuda()
    assert torch.equal(off(x, tok), res(x, tok))
    small = ExpertCache(512, 256, capacity=3)
    off2 = OffloadedMoELayer(cfg, HostBank.from_bank(res.bank), small, layer_idx=2)
    off2.hash_router.weight.data = res.hash_router.weight.data
    off2.hash_router.tid2eid = res.hash_router.tid2eid
    with pytest.raises(ValueError, match="cache holds 3"):
        off2(x, tok)
