"""GPU layout kernels against the oracle and the reference's known answers (bit-exact)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.layout import emit_tiles as emit_ref
from oracle.layout import layout_assignments as layout_ref

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    from mosaic_b200 import ops as o

    return o


def test_layout_known_answer(ops):
    # tests/test_moe_layout.py:13-24 of the reference
    sorted_ids, perm, offsets, counts = ops.layout_assignments(torch.tensor([3, 0, 3, 1], device="cuda"), 4)
    assert counts.tolist() == [1, 1, 0, 2]
    assert int(offsets[-1].item()) == 4
    for e in range(4):
        lo, hi = int(offsets[e]), int(offsets[e + 1])
        assert (sorted_ids[lo:hi] == e).all()
    assert perm.tolist() == [1, 3, 0, 2]


@pytest.mark.parametrize("a,e", [(1, 1), (256, 32), (1024, 256), (65536, 256), (5000, 7)])
def test_layout_random_stable(ops, a, e):
    g = torch.Generator().manual_seed(a + e)
    ids = torch.randint(0, e, (a,), generator=g)
    s, p, o, c = ops.layout_assignments(ids.cuda(), e)
    sr, pr, orf, cr = layout_ref(ids.numpy(), e)
    assert np.array_equal(c.cpu().numpy(), cr)
    assert np.array_equal(o.cpu().numpy(), orf)
    assert np.array_equal(p.cpu().numpy(), pr)
    assert np.array_equal(s.cpu().numpy(), sr)


def test_layout_rejects_cpu(ops):
    with pytest.raises(ValueError):
        ops.layout_assignments(torch.tensor([0, 1]), 2)


@pytest.mark.parametrize("block_m", [1, 8, 16])
def test_emit_tiles_known_answer(ops, block_m):
    # tests/test_emit_tiles.py:15-34 of the reference
    counts = torch.tensor([0, 1, block_m - 1, block_m, block_m + 1, 3 * block_m + 2], dtype=torch.int32)
    ei, ms, nt, rows = ops.emit_tiles(counts.cuda(), block_m=block_m, max_tiles=64)
    n = int(nt.item())
    exp = emit_ref(counts.tolist(), block_m)
    assert n == len(exp)
    assert list(zip(ei[:n].tolist(), ms[:n].tolist(), rows[:n].tolist())) == exp


@pytest.mark.parametrize("block_m", [1, 8, 16])
def test_emit_tiles_all_empty(ops, block_m):
    ei, ms, nt, rows = ops.emit_tiles(torch.zeros(5, dtype=torch.int32, device="cuda"), block_m=block_m, max_tiles=8)
    assert int(nt.item()) == 0


def test_layout_repeated_expert_per_token(ops):
    """A token may name an expert more than once (a hash table row can): every
    assignment keeps its own row, in flat order, as the reference's argsort groups them."""
    g = torch.Generator().manual_seed(12)
    ids = torch.randint(0, 8, (700, 3), generator=g)  # most tokens repeat an expert
    ids[0] = torch.tensor([5, 5, 5])
    sid, perm, off, cnt = ops.layout_assignments(ids.reshape(-1).cuda(), 8)
    r_sid, r_perm, r_off, r_cnt = layout_ref(ids.reshape(-1).numpy(), 8)
    assert np.array_equal(perm.cpu().numpy(), r_perm) and np.array_equal(sid.cpu().numpy(), r_sid)
    assert np.array_equal(off.cpu().numpy(), r_off) and np.array_equal(cnt.cpu().numpy(), r_cnt)


@pytest.mark.parametrize("mode", ["bf16", "fp8"])
def test_moe_routed_with_repeated_experts(mode):
    """The expert path with repeated ids per token (all assignments computed, the
    equal partials summed) matches the oracle layer."""
    from oracle.moe import moe_layer
    from tests.golden.recipes import MOE_CASES, make_moe_case
    from tests.helpers import gpu_bank, layer_for, pack_case, rel_l2

    case = make_moe_case(**MOE_CASES["S"])
    obank, full = pack_case(case)
    c = case["cfg"]
    g = torch.Generator().manual_seed(3)
    idx = torch.randint(0, c["E"], (c["T"], c["k"]), generator=g)
    idx[:, 1] = idx[:, 0]  # every token names its first expert twice
    w = torch.rand(c["T"], c["k"], generator=g)
    layer = layer_for(case, gpu_bank(full), mode)
    from mosaic_b200.moe import _routed

    y = _routed(layer.cfg, case["x"].cuda(), idx.cuda(), w.cuda(), layer.bank, include_shared=True)
    torch.cuda.synchronize()
    ref = moe_layer(case["x"], w, idx, obank, mode=mode, swiglu_limit=c["swiglu_limit"])
    tol = {"bf16": 5e-3, "fp8": 2e-3}[mode]
    assert rel_l2(y.float().cpu().numpy(), ref) <= tol
