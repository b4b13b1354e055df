"""Expert cache bookkeeping without a GPU: byte sizes of the bank layouts and the
LRU replacement order (the copies themselves need a device)."""
from __future__ import annotations

from mosaic_b200.offload import _expert_bytes


def test_expert_bytes_match_the_bank_layouts():
    gu_t, gu_sf, dn_t, dn_sf = _expert_bytes(7168, 2048)
    assert gu_t + dn_t == 2 * 2048 * 7168 // 2 + 7168 * 2048 // 2
    assert gu_sf == 2 * 2048 * 7168 // 32 and dn_sf == 7168 * 2048 // 32
    # one V3 expert: codes + E8M0 scales
    assert sum(_expert_bytes(7168, 2048)) == 23_396_352
