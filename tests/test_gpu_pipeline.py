"""HostPipeline: layer steps over pinned host batches with the uploads and
downloads of neighbouring steps overlapping the layer.  Every output equals the
layer's own output on that batch bit for bit, in graph and eager mode, for an
odd number of batches (both slots, a last step on slot 0) and with batches
that repeat."""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def _layer(act_mode):
    from mosaic_b200 import MoEConfig, MoELayer, synthetic

    cfg = MoEConfig(hidden_size=512, moe_intermediate_size=256, n_routed_experts=32, num_experts_per_tok=4,
                    n_group=4, topk_group=2, routed_scaling_factor=2.5, act_mode=act_mode)
    layer = MoELayer(cfg, synthetic.make_bank(512, 256, 32, 4))
    synthetic.make_router(layer, 4)
    return layer


@pytest.mark.parametrize("graph", [True, False])
@pytest.mark.parametrize("act_mode", ["fp8", "bf16"])
def test_host_pipeline_outputs_equal_the_layer(graph, act_mode):
    from mosaic_b200 import synthetic
    from mosaic_b200.pipeline import HostPipeline

    layer = _layer(act_mode)
    t = 96
    xs = [synthetic.make_tokens(t, 512, 100 + i) for i in range(5)]
    refs = [layer(x).cpu() for x in xs]
    pipe = HostPipeline(layer, t, 512, graph=graph)
    xh = [x.cpu().pin_memory() for x in xs]
    order = [0, 1, 2, 3, 4, 2, 2]  # 7 steps: both slots, repeats
    yh = [torch.empty_like(xh[0]).pin_memory() for _ in order]
    pipe.run([xh[i] for i in order], yh)
    torch.cuda.synchronize()
    for j, i in enumerate(order):
        assert torch.equal(yh[j], refs[i]), (j, i)
    # a second run reuses the slots and their events
    pipe.run([xh[4], xh[0]], yh[:2])
    torch.cuda.synchronize()
    assert torch.equal(yh[0], refs[4]) and torch.equal(yh[1], refs[0])
    pipe.close()


def test_host_pipeline_rejects_unpinned_or_misshaped_batches():
    from mosaic_b200.pipeline import HostPipeline

    layer = _layer("fp8")
    pipe = HostPipeline(layer, 32, 512, graph=False)
    good = torch.zeros(32, 512, dtype=torch.bfloat16).pin_memory()
    with pytest.raises(ValueError, match="pinned"):
        pipe.run([torch.zeros(32, 512, dtype=torch.bfloat16)], [good])
    with pytest.raises(ValueError, match="shape"):
        pipe.run([torch.zeros(16, 512, dtype=torch.bfloat16).pin_memory()], [good])
    with pytest.raises(ValueError, match="one output"):
        pipe.run([good], [])
    pipe.close()
