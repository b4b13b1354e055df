"""C ABI checks that need no GPU: the library loads, exports every symbol the
header declares, and host-side validation rejects bad calls before any launch."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from mosaic_b200 import _capi as C

HEADER = Path(__file__).resolve().parents[1] / "include" / "mosaic_moe.h"


def _declared():
    text = HEADER.read_text()
    return set(re.findall(r"MOSAIC_API[^;(]*?\b(mosaic_\w+)\s*\(", text, flags=re.S))


def test_library_loads_and_exports_all_declared_symbols():
    lib = C.lib()
    declared = _declared()
    assert declared == set(C.EXPORTED)
    for name in declared:
        assert hasattr(lib, name), name
    assert lib.mosaic_version() >= 1


def test_status_strings():
    lib = C.lib()
    for code in range(0, 9):
        assert lib.mosaic_status_string(code)
    assert lib.mosaic_status_string(0) == b"ok"


def _dims(**kw):
    d = C.MoEDims()
    base = dict(tokens=8, hidden=512, inter=256, n_experts=32, top_k=4, n_group=4, topk_group=2, act_mode=0,
                norm_topk_prob=1, has_shared=1, route_scale=2.5, swiglu_limit=0.0)
    base.update(kw)
    for k, v in base.items():
        setattr(d, k, v)
    return d


@pytest.mark.parametrize("bad", [dict(hidden=500), dict(hidden=384), dict(inter=100), dict(n_experts=300), dict(top_k=9),
                                 dict(n_group=3), dict(topk_group=5), dict(n_group=8, topk_group=1, top_k=8),
                                 dict(act_mode=7), dict(tokens=0)])
def test_workspace_bytes_rejects_bad_dims(bad):
    assert C.lib().mosaic_moe_workspace_bytes(ctypes.byref(_dims(**bad))) == 0


def test_workspace_bytes_grows_with_tokens():
    lib = C.lib()
    a = lib.mosaic_moe_workspace_bytes(ctypes.byref(_dims(tokens=8)))
    b = lib.mosaic_moe_workspace_bytes(ctypes.byref(_dims(tokens=64)))
    assert 0 < a < b


def test_forward_validation_before_launch():
    lib = C.lib()
    bank = C.ExpertBankC()
    fake = 1 << 20  # aligned, never dereferenced: validation fails first
    bank.gu_tiled = bank.gu_sf = bank.dn_tiled = bank.dn_sf = fake
    d = _dims()
    args = [ctypes.byref(d), fake, fake, fake, ctypes.byref(bank), fake, fake, fake, fake, 1 << 40, None]
    # null x
    a = list(args)
    a[1] = None
    assert lib.mosaic_moe_forward(*a) == C.MOSAIC_ERR_SHAPE
    # misaligned y
    a = list(args)
    a[5] = fake + 2
    assert lib.mosaic_moe_forward(*a) == C.MOSAIC_ERR_ALIGN
    # misaligned weight bank (TMA needs 32 B)
    bank.gu_tiled = fake + 16
    assert lib.mosaic_moe_forward(*args) == C.MOSAIC_ERR_ALIGN
    bank.gu_tiled = fake
    # workspace too small
    a = list(args)
    a[9] = 16
    assert lib.mosaic_moe_forward(*a) == C.MOSAIC_ERR_WORKSPACE
    # bad dims
    bad = _dims(n_group=3)
    a = list(args)
    a[0] = ctypes.byref(bad)
    assert lib.mosaic_moe_forward(*a) == C.MOSAIC_ERR_SHAPE


def test_split_expert_gemm_validation_before_launch():
    lib = C.lib()
    bank = C.ExpertBankC()
    fake = 1 << 20  # aligned, never dereferenced: validation fails first
    bank.gu_tiled = bank.gu_sf = bank.dn_tiled = bank.dn_sf = fake
    d = _dims()
    gu = [ctypes.byref(d), fake, fake, fake, ctypes.byref(bank), fake, 1 << 40, None]
    dn = [ctypes.byref(d), ctypes.byref(bank), fake, fake, 1 << 40, None]
    for fn, args, x_at, ws_at, size_at in ((lib.mosaic_expert_gemm_gu, gu, 1, 5, 6),
                                            (lib.mosaic_expert_gemm_down, dn, 2, 3, 4)):
        a = list(args)
        a[x_at] = None  # null x (gate/up) or y (down)
        assert fn(*a) == C.MOSAIC_ERR_SHAPE
        a = list(args)
        a[x_at] = fake + 2
        assert fn(*a) == C.MOSAIC_ERR_ALIGN
        a = list(args)
        a[ws_at] = fake + 128  # the workspace needs 256-B alignment
        assert fn(*a) == C.MOSAIC_ERR_ALIGN
        a = list(args)
        a[size_at] = 16
        assert fn(*a) == C.MOSAIC_ERR_WORKSPACE
        a = list(args)
        a[0] = None
        assert fn(*a) == C.MOSAIC_ERR_SHAPE
        bank.dn_sf = fake + 4
        assert fn(*args) == C.MOSAIC_ERR_ALIGN
        bank.dn_sf = fake
    # the two calls size their workspace exactly as the fused call does
    assert lib.mosaic_moe_workspace_bytes(ctypes.byref(d)) > 16


def test_router_validation_before_launch():
    lib = C.lib()
    fake = 1 << 20
    st = lib.mosaic_router(fake, fake, None, 4, 512, 32, 9, 1, 1, 1.0, 1, fake, fake, fake, 1 << 30, None)
    assert st == C.MOSAIC_ERR_SHAPE
    st = lib.mosaic_router(fake + 4, fake, None, 4, 512, 32, 4, 1, 1, 1.0, 1, fake, fake, fake, 1 << 30, None)
    assert st == C.MOSAIC_ERR_ALIGN


def test_check_maps_status_to_reference_exceptions():
    with pytest.raises(ValueError):
        C.check(C.MOSAIC_ERR_SHAPE, "x")
    with pytest.raises(TypeError):
        C.check(C.MOSAIC_ERR_DTYPE, "x")
    with pytest.raises(C.MosaicError):
        C.check(C.MOSAIC_ERR_TIMEOUT, "x")
    C.check(C.MOSAIC_OK, "x")


def test_host_api_mirrors_reference_names():
    import mosaic_b200 as m

    for name in ("MoELayer", "Router", "grouped_expert_forward", "exact_moe", "exact_target", "ExactContractError"):
        assert hasattr(m, name)
    from mosaic_b200 import ops

    for name in ("layout_assignments", "emit_tiles", "act_quant", "pack_mxfp4_nk"):
        assert hasattr(ops, name)


def test_ops_reject_cpu_tensors():
    import torch

    from mosaic_b200 import ops

    with pytest.raises(ValueError):
        ops.layout_assignments(torch.tensor([0, 1, 2]), 4)
    with pytest.raises(ValueError):
        ops.act_quant(torch.zeros(2, 100))


def test_router_noalloc_constant_matches_header():
    m = re.search(r"#define MOSAIC_ROUTER_NOALLOC_SCRATCH_BYTES \((\d+)u << (\d+)\)", HEADER.read_text())
    assert m and int(m.group(1)) << int(m.group(2)) == C.MOSAIC_ROUTER_NOALLOC_SCRATCH_BYTES


def test_router_noalloc_validation_before_launch():
    """Bad shapes, misalignment and inputs larger than the fixed scratch are
    rejected on the host, before any device call."""
    lib = C.lib()
    fake = 1 << 20
    st = lib.mosaic_router_noalloc(fake, fake, None, 4, 512, 32, 9, 1, 1, 1.0, 1, fake, fake, None)
    assert st == C.MOSAIC_ERR_SHAPE
    st = lib.mosaic_router_noalloc(fake + 4, fake, None, 4, 512, 32, 4, 1, 1, 1.0, 1, fake, fake, None)
    assert st == C.MOSAIC_ERR_ALIGN
    # T = 32768 tokens over 256 experts: 32 MiB of logits + the W parts of the tensor-core path
    assert lib.mosaic_router_workspace_bytes(32768, 7168, 256) > C.MOSAIC_ROUTER_NOALLOC_SCRATCH_BYTES
    st = lib.mosaic_router_noalloc(fake, fake, None, 32768, 7168, 256, 8, 8, 4, 2.5, 1, fake, fake, None)
    assert st == C.MOSAIC_ERR_WORKSPACE


def test_router_workspace_follows_the_split_plan():
    """Without a device the plan assumes 148 SMs.  V3 router (H 7168, E 256):
    the tensor-core logits take one wave of 128 x 128 tiles, up to 64 K splits
    (the partials are [splits][T][E] fp32 after a 256-byte error block); from
    T = 129 on W's three bf16 parts (3·E·H·2 B) follow them."""
    lib = C.lib()
    h, e = 7168, 256
    up = lambda n: (n + 255) // 256 * 256  # noqa: E731
    parts = up(3 * e * h * 2)
    assert lib.mosaic_router_workspace_bytes(1, h, e) == 256 + up(64 * 1 * e * 4)
    assert lib.mosaic_router_workspace_bytes(128, h, e) == 256 + up(64 * 128 * e * 4)
    assert lib.mosaic_router_workspace_bytes(2048, h, e) == 256 + up(4 * 2048 * e * 4) + parts
    assert lib.mosaic_router_workspace_bytes(8192, h, e) == 256 + up(1 * 8192 * e * 4) + parts
    # H % 64 != 0 keeps the FMA kernels: no parts
    assert lib.mosaic_router_workspace_bytes(128, 992, e) % 256 == 0
    assert lib.mosaic_router_workspace_bytes(128, 992, e) < 256 + up(64 * 128 * e * 4)


def test_hc_workspace_follows_the_split_plan():
    """Error block, split-K mixing partials [splits][T][25] (one wave of 128-token
    tiles over 148 SMs, at most 32 splits and one 64-wide slice per split), fn's
    parts [3][32][hc·D], the tokens' pre-mix weights [T][4]."""
    lib = C.lib()
    d, hc = 7168, 4
    up = lambda n: (n + 255) // 256 * 256  # noqa: E731
    parts = up(3 * 32 * hc * d * 2)
    ws = lib.mosaic_hc_pre_norm_workspace_bytes
    assert ws(128, d, hc) == 256 + up(32 * 128 * 25 * 4) + parts + up(128 * 16)
    assert ws(8192, d, hc) == 256 + up(2 * 8192 * 25 * 4) + parts + up(8192 * 16)
    assert ws(1, 128, 1) == 256 + up(2 * 1 * 25 * 4) + up(3 * 32 * 128 * 2) + up(16)


def test_rms_norm_validation_before_launch():
    """Shape, pairing of q / q_scale, epsilon and alignment are checked on the host."""
    lib = C.lib()
    fake = 1 << 20
    st = lib.mosaic_rms_norm(fake, fake, 4, 12, 1e-6, fake, None, None, None)  # D % 8
    assert st == C.MOSAIC_ERR_SHAPE
    st = lib.mosaic_rms_norm(fake, fake, 4, 65544, 1e-6, fake, None, None, None)  # D above the maximum
    assert st == C.MOSAIC_ERR_SHAPE
    st = lib.mosaic_rms_norm(fake, fake, 4, 256, 1e-6, fake, fake, None, None)  # q without q_scale
    assert st == C.MOSAIC_ERR_SHAPE
    st = lib.mosaic_rms_norm(fake, fake, 4, 136, 1e-6, fake, fake, fake, None)  # act_quant needs D % 128
    assert st == C.MOSAIC_ERR_SHAPE
    st = lib.mosaic_rms_norm(fake, fake, 4, 256, -1.0, fake, None, None, None)
    assert st == C.MOSAIC_ERR_RANGE
    st = lib.mosaic_rms_norm(fake + 8, fake, 4, 256, 1e-6, fake, None, None, None)
    assert st == C.MOSAIC_ERR_ALIGN


def test_ep_row_sizes_match_header_and_region_geometry():
    """MOSAIC_EP_ROW_BYTES(_E4M3) as the header defines them; an E4M3 region
    holds max_recv_rows E4M3 rows; E4M3 rows with fp32 partials (a bf16
    layer), unit slots outside 0..8 or without E4M3 rows, or H > 16384 are
    refused (0 bytes); unit rows add 16 bytes per slot to an E4M3 row."""
    text = HEADER.read_text()
    assert "#define MOSAIC_EP_ROW_BYTES_E4M3(H) ((size_t)(H) + ((((size_t)(H) / 128u) + 15u) & ~(size_t)15u) + 16u)" \
        in text
    assert C.ep_row_bytes_e4m3(7168) == 7248 and C.ep_row_bytes(7168) == 14352
    assert C.ep_row_bytes_e4m3(512) == 544 and C.ep_row_bytes_e4m3(2048 + 128) == 2176 + 32 + 16
    lib = C.lib()

    def region(**kw):
        pe = C.EpPeersC()
        pe.world, pe.rank, pe.max_tokens, pe.hidden, pe.partial_f32 = 2, 0, 8, 7168, 0
        pe.max_send_rows, pe.max_recv_rows = 64, 128
        for k, v in kw.items():
            setattr(pe, k, v)
        return lib.mosaic_ep_region_bytes(ctypes.byref(pe))

    bf16_rows, e4m3_rows = region(), region(row_e4m3=1)
    assert bf16_rows - e4m3_rows == 128 * (C.ep_row_bytes(7168) - C.ep_row_bytes_e4m3(7168))
    assert region(row_e4m3=1, partial_f32=1) == 0
    assert region(row_e4m3=2) == 0 and region(unit_slots=9) == 0 and region(unit_slots=2) == 0
    assert C.ep_row_bytes_e4m3_units(7168, 8) == 7248 + 128
    assert region(row_e4m3=1, unit_slots=8) - e4m3_rows == 128 * 128
    assert region(row_e4m3=1, hidden=16384 + 256) == 0 and region(hidden=16384 + 256) > 0


def test_ep_dispatch_exchange_validation_before_launch():
    """The fused E4M3 dispatch refuses a bf16 layer, a bf16-row exchange and a
    rank's tokens above the exchange capacity before any device call."""
    from mosaic_b200 import MoEConfig

    lib = C.lib()
    fake = 1 << 20
    pe = C.EpPeersC()
    pe.world, pe.rank, pe.max_tokens, pe.hidden, pe.partial_f32, pe.row_e4m3 = 1, 0, 8, 512, 0, 1
    pe.max_send_rows, pe.max_recv_rows = 32, 32
    pe.regions[0] = fake
    cfg = MoEConfig(hidden_size=512, moe_intermediate_size=256, n_routed_experts=32, num_experts_per_tok=4,
                    n_group=1, topk_group=1, act_mode="fp8")

    def call(d, p):
        return lib.mosaic_ep_dispatch_exchange(ctypes.byref(d), ctypes.byref(p), fake, fake, fake, fake, 1 << 40,
                                               None)

    assert call(cfg.dims(9, True), pe) == C.MOSAIC_ERR_SHAPE  # 9 tokens > max_tokens 8
    d_bf16 = MoEConfig(hidden_size=512, moe_intermediate_size=256, n_routed_experts=32, num_experts_per_tok=4,
                       n_group=1, topk_group=1, act_mode="bf16").dims(8, True)
    assert call(d_bf16, pe) == C.MOSAIC_ERR_SHAPE
    pe.row_e4m3 = 0
    assert call(cfg.dims(8, True), pe) == C.MOSAIC_ERR_SHAPE
