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
