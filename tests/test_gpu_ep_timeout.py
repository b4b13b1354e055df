"""A device-side wait of the peer-memory exchange that runs out, on one GPU.

The exchange of rank 0 of a world of 2 is opened in one process with the
second rank's region allocated but never served: nothing stamps rank 0's
flags for rank 1, so the count exchange and the data wait each run out after
the 1 ms budget (``mosaic_ep_peers.wait_us``).  The kernels return, the
region's error word reads MOSAIC_ERR_TIMEOUT, and the device keeps working
(a MoE layer call afterwards gives the same output as before).  No GPU fault,
trap or endless wait is involved: the wait is bounded and the flag simply
never changes.
"""
from __future__ import annotations

import ctypes
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_peer_exchange_wait_runs_out_and_the_device_stays_usable():
    from mosaic_b200 import _capi as C
    from mosaic_b200 import ops
    from tests.test_gpu_ep import _small_layer

    layer, x = _small_layer("bf16", seed=9, t=32)
    y_before = layer(x)
    torch.cuda.synchronize()

    lib = C.lib()
    pe = C.EpPeersC()
    pe.world, pe.rank = 2, 0
    pe.max_tokens, pe.hidden, pe.partial_f32 = 8, 512, 1
    pe.max_send_rows = 8 * 4
    pe.max_recv_rows = 2 * 8 * 4
    pe.wait_us = 1000
    nbytes = lib.mosaic_ep_region_bytes(ctypes.byref(pe))
    assert nbytes > 0
    regions = []
    for _ in range(2):  # rank 0's region and the region of a rank 1 that never runs
        ptr, handle = ctypes.c_void_p(), (ctypes.c_uint8 * 64)()
        C.check(lib.mosaic_ep_region_alloc(nbytes, ctypes.byref(ptr), handle), "mosaic_ep_region_alloc")
        regions.append(ptr.value)
    try:
        pe.regions[0], pe.regions[1] = regions
        send = torch.zeros(2, C.ep_row_bytes(512), dtype=torch.uint8, device="cuda")
        counts = torch.tensor([1, 1], dtype=torch.int32, device="cuda")  # one row to each rank
        t0 = time.perf_counter()
        st = lib.mosaic_ep_exchange_rows(ctypes.byref(pe), ops._ptr(send), ops._ptr(counts), ops._stream())
        torch.cuda.synchronize()
        elapsed = time.perf_counter() - t0
        assert st == C.MOSAIC_OK
        assert elapsed < 1.0, elapsed  # two 1 ms waits, not the 2 s default
        code = ctypes.c_int32(0)
        C.check(lib.mosaic_read_error(ctypes.c_void_p(regions[0]), 1, ctypes.byref(code), ops._stream()),
                "mosaic_read_error")
        assert code.value == C.MOSAIC_ERR_TIMEOUT
        # the context is intact: the same layer call gives the same output
        y_after = layer(x)
        torch.cuda.synchronize()
        assert torch.equal(y_after, y_before)
        assert ops.read_error(layer.workspace(x.shape[0], x.device)) == 0
    finally:
        for r in regions:
            lib.mosaic_ep_region_free(ctypes.c_void_p(r))


def test_peer_exchange_rejects_a_negative_wait_budget():
    from mosaic_b200 import _capi as C

    pe = C.EpPeersC()
    pe.world, pe.rank, pe.max_tokens, pe.hidden, pe.partial_f32 = 2, 0, 8, 512, 1
    pe.max_send_rows, pe.max_recv_rows, pe.wait_us = 32, 64, -1
    assert C.lib().mosaic_ep_region_bytes(ctypes.byref(pe)) == 0
