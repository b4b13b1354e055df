"""Assignment layout (histogram / prefix scan / permutation) and tile list (test oracle).

Reference behaviour followed:

* ``mosaicvm/kernels/moe_layout.py:8-27`` (``layout_assignments``):
  ``counts = bincount(ids)``, ``offsets = [0, cumsum(counts)]`` (int32), and a
  permutation that groups assignments by expert.  The reference uses the
  default (unstable) ``torch.argsort``; this build fixes the order inside an
  expert segment to ascending flat index (token-major, then slot), i.e. the
  stable argsort.  Counts, offsets and segment contents are what the
  reference's own test pins (``tests/test_moe_layout.py:13-24``); they are
  identical under either order.
* ``mosaicvm/kernels/w4a16_grouped.py:151-169`` and the Triton kernel at
  ``:41-61`` (``emit_tiles``): for every expert e, tiles
  (e, m_start = t*block_m, rows = min(block_m, count - m_start)) in expert
  order; the tile count stays on the device.
"""
from __future__ import annotations

import numpy as np


def layout_assignments(expert_ids, n_experts: int):
    """ids [A] -> (sorted_ids int64 [A], perm int64 [A], offsets int32 [E+1], counts int32 [E])."""
    ids = np.asarray(expert_ids, dtype=np.int64).reshape(-1)
    perm = np.argsort(ids, kind="stable").astype(np.int64)
    counts = np.bincount(ids, minlength=n_experts).astype(np.int32)
    offsets = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
    return ids[perm], perm, offsets, counts


def emit_tiles(counts, block_m: int):
    """counts [E] -> list of (expert, m_start, rows) in expert order."""
    out = []
    for e, c in enumerate(np.asarray(counts).tolist()):
        n = (c + block_m - 1) // block_m
        for t in range(n):
            out.append((e, t * block_m, min(block_m, c - t * block_m)))
    return out


def moe_rows(idx, n_experts: int, with_shared: bool = True):
    """Row map of one MoE layer's packed (expert-sorted) activation matrix.

    idx [T, k] routed expert ids.  Routed assignments are ordered by
    (expert, token, slot); when ``with_shared`` the shared expert is expert
    ``n_experts`` and owns the last T rows, one per token in token order.

    Returns (counts int32 [E(+1)], offsets int32 [E(+1)+1], row_of int32 [T, k],
    row_token int32 [R], row_slot int32 [R]).
    """
    idx = np.asarray(idx, dtype=np.int64)
    t, k = idx.shape
    _, perm, offsets, counts = layout_assignments(idx.reshape(-1), n_experts)
    a = t * k
    row_of = np.empty(a, dtype=np.int32)
    row_of[perm] = np.arange(a, dtype=np.int32)
    row_token = (perm // k).astype(np.int32)
    row_slot = (perm % k).astype(np.int32)
    if with_shared:
        counts = np.concatenate([counts, [t]]).astype(np.int32)
        offsets = np.concatenate([offsets, [a + t]]).astype(np.int32)
        row_token = np.concatenate([row_token, np.arange(t, dtype=np.int32)])
        row_slot = np.concatenate([row_slot, np.full(t, k, dtype=np.int32)])
    return counts, offsets, row_of.reshape(t, k), row_token, row_slot
