"""ctypes binding of ``libmosaic_moe.so`` (declared in ``include/mosaic_moe.h``).

The library is built in-tree by ``mosaic_b200/build.py`` (nvcc, sm_100a).  There
is no fallback: if the shared object is missing or fails to load, every
operator raises.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libmosaic_moe.so"

MOSAIC_OK = 0
MOSAIC_ERR_SHAPE = 1
MOSAIC_ERR_DTYPE = 2
MOSAIC_ERR_ALIGN = 3
MOSAIC_ERR_RANGE = 4
MOSAIC_ERR_CUDA = 5
MOSAIC_ERR_TIMEOUT = 6
MOSAIC_ERR_UNSUPPORTED = 7
MOSAIC_ERR_WORKSPACE = 8

def ep_row_bytes(hidden: int) -> int:
    """include/mosaic_moe.h MOSAIC_EP_ROW_BYTES: H bf16 values + a 16-byte tail."""
    return 2 * hidden + 16


def ep_row_bytes_e4m3(hidden: int) -> int:
    """include/mosaic_moe.h MOSAIC_EP_ROW_BYTES_E4M3: H E4M3 codes, the H/128 scale
    exponents padded to 16 bytes, the 16-byte tail."""
    return hidden + ((hidden // 128 + 15) & ~15) + 16


def ep_row_bytes_e4m3_units(hidden: int, slots: int) -> int:
    """include/mosaic_moe.h MOSAIC_EP_ROW_BYTES_E4M3_UNITS: the E4M3 row (its tail
    the unit header) and 16 bytes per slot."""
    return ep_row_bytes_e4m3(hidden) + 16 * slots


# include/mosaic_moe.h MOSAIC_ROUTER_NOALLOC_SCRATCH_BYTES
MOSAIC_ROUTER_NOALLOC_SCRATCH_BYTES = 32 << 20

MOSAIC_ACT_BF16 = 0
MOSAIC_ACT_FP8 = 1

# enum mosaic_score_func
MOSAIC_SCORE_SIGMOID = 0
MOSAIC_SCORE_SQRTSOFTPLUS = 1
MOSAIC_SCORE_SOFTMAX = 2
SCORE_FUNCS = {"sigmoid": MOSAIC_SCORE_SIGMOID, "sqrtsoftplus": MOSAIC_SCORE_SQRTSOFTPLUS,
               "softmax": MOSAIC_SCORE_SOFTMAX}

# Every symbol the header declares; tests check the library exports all of them.
EXPORTED = (
    "mosaic_version",
    "mosaic_status_string",
    "mosaic_device_sm_count",
    "mosaic_router_workspace_bytes",
    "mosaic_router",
    "mosaic_router_noalloc",
    "mosaic_router_ext",
    "mosaic_layout_assignments",
    "mosaic_emit_tiles",
    "mosaic_act_quant",
    "mosaic_pack_mxfp4",
    "mosaic_repack_weights",
    "mosaic_prepack_scales",
    "mosaic_hc_pre_norm_workspace_bytes",
    "mosaic_hc_pre_norm",
    "mosaic_hc_post",
    "mosaic_rms_norm",
    "mosaic_moe_workspace_bytes",
    "mosaic_moe_forward",
    "mosaic_moe_forward_profiled",
    "mosaic_moe_forward_ext",
    "mosaic_moe_routed",
    "mosaic_moe_routed_slots",
    "mosaic_expert_gemm_gu",
    "mosaic_expert_gemm_down",
    "mosaic_ep_dispatch",
    "mosaic_moe_expert_rows_workspace_bytes",
    "mosaic_moe_expert_rows",
    "mosaic_ep_combine",
    "mosaic_ep_region_bytes",
    "mosaic_ep_region_alloc",
    "mosaic_ep_region_open",
    "mosaic_ep_region_close",
    "mosaic_ep_region_free",
    "mosaic_ep_region_view",
    "mosaic_ep_exchange_rows",
    "mosaic_ep_dispatch_exchange",
    "mosaic_ep_expert_rows_workspace_bytes",
    "mosaic_ep_return_partials",
    "mosaic_ep_expert_rows_return",
    "mosaic_moe_expert_rows_dev",
    "mosaic_read_error",
)


class MoEDims(ctypes.Structure):
    _fields_ = [
        ("tokens", ctypes.c_int32),
        ("hidden", ctypes.c_int32),
        ("inter", ctypes.c_int32),
        ("n_experts", ctypes.c_int32),
        ("top_k", ctypes.c_int32),
        ("n_group", ctypes.c_int32),
        ("topk_group", ctypes.c_int32),
        ("act_mode", ctypes.c_int32),
        ("norm_topk_prob", ctypes.c_int32),
        ("has_shared", ctypes.c_int32),
        ("route_scale", ctypes.c_float),
        ("swiglu_limit", ctypes.c_float),
    ]


class ExpertBankC(ctypes.Structure):
    _fields_ = [
        ("gu_tiled", ctypes.c_void_p),
        ("gu_sf", ctypes.c_void_p),
        ("dn_tiled", ctypes.c_void_p),
        ("dn_sf", ctypes.c_void_p),
    ]


class RouteExtC(ctypes.Structure):
    _fields_ = [
        ("score_func", ctypes.c_int32),
        ("hash", ctypes.c_int32),
        ("layer_idx", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
        ("table_rows", ctypes.c_int64),
        ("tid2eid", ctypes.c_void_p),
        ("token_ids", ctypes.c_void_p),
    ]


EP_MAX_WORLD = 8  # include/mosaic_moe.h MOSAIC_EP_MAX_WORLD


class EpPeersC(ctypes.Structure):
    _fields_ = [
        ("world", ctypes.c_int32),
        ("rank", ctypes.c_int32),
        ("max_recv_rows", ctypes.c_int32),
        ("max_send_rows", ctypes.c_int32),
        ("max_tokens", ctypes.c_int32),
        ("hidden", ctypes.c_int32),
        ("partial_f32", ctypes.c_int32),
        ("wait_us", ctypes.c_int32),
        ("row_e4m3", ctypes.c_int32),
        ("unit_slots", ctypes.c_int32),
        ("regions", ctypes.c_void_p * EP_MAX_WORLD),
    ]


class MosaicError(RuntimeError):
    """A MOSAIC_ERR_* status that has no closer Python exception class."""


_P = ctypes.c_void_p
_I = ctypes.c_int32
_SZ = ctypes.c_size_t

_SIGS = {
    "mosaic_version": ([], ctypes.c_int),
    "mosaic_status_string": ([ctypes.c_int], ctypes.c_char_p),
    "mosaic_device_sm_count": ([], ctypes.c_int),
    "mosaic_router_workspace_bytes": ([_I, _I, _I], _SZ),
    "mosaic_router": ([_P, _P, _P, _I, _I, _I, _I, _I, _I, ctypes.c_float, _I, _P, _P, _P, _SZ, _P], ctypes.c_int),
    "mosaic_router_noalloc": ([_P, _P, _P, _I, _I, _I, _I, _I, _I, ctypes.c_float, _I, _P, _P, _P], ctypes.c_int),
    "mosaic_router_ext": ([ctypes.POINTER(RouteExtC), _P, _P, _P, _I, _I, _I, _I, _I, _I, ctypes.c_float, _I, _P, _P,
                           _P, _SZ, _P], ctypes.c_int),
    "mosaic_layout_assignments": ([_P, _I, _I, _P, _P, _P, _P, _P], ctypes.c_int),
    "mosaic_emit_tiles": ([_P, _I, _I, _I, _P, _P, _P, _P, _P], ctypes.c_int),
    "mosaic_act_quant": ([_P, _I, _I, _P, _P, _P], ctypes.c_int),
    "mosaic_pack_mxfp4": ([_P, _I, _I, _P, _P, _P], ctypes.c_int),
    "mosaic_repack_weights": ([_P, _I, _I, _I, _I, _P, _P], ctypes.c_int),
    "mosaic_prepack_scales": ([_P, _I, _I, _I, _I, _P, _P], ctypes.c_int),
    "mosaic_hc_pre_norm_workspace_bytes": ([_I, _I, _I], _SZ),
    "mosaic_hc_pre_norm": ([_P, _P, _P, _P, _P, _I, _I, _I, _I, ctypes.c_float, ctypes.c_float, _P, _P, _P, _P, _P,
                            _P, _SZ, _P], ctypes.c_int),
    "mosaic_hc_post": ([_P, _P, _P, _P, _I, _I, _I, _P, _P], ctypes.c_int),
    "mosaic_rms_norm": ([_P, _P, _I, _I, ctypes.c_float, _P, _P, _P, _P], ctypes.c_int),
    "mosaic_moe_workspace_bytes": ([ctypes.POINTER(MoEDims)], _SZ),
    "mosaic_moe_forward": ([ctypes.POINTER(MoEDims), _P, _P, _P, ctypes.POINTER(ExpertBankC), _P, _P, _P, _P, _SZ, _P],
                           ctypes.c_int),
    "mosaic_moe_forward_profiled": ([ctypes.POINTER(MoEDims), _P, _P, _P, ctypes.POINTER(ExpertBankC), _P, _P, _P, _P,
                                     _SZ, _P, ctypes.POINTER(ctypes.c_void_p)], ctypes.c_int),
    "mosaic_moe_forward_ext": ([ctypes.POINTER(MoEDims), ctypes.POINTER(RouteExtC), _P, _P, _P,
                                ctypes.POINTER(ExpertBankC), _P, _P, _P, _P, _SZ, _P], ctypes.c_int),
    "mosaic_moe_routed": ([ctypes.POINTER(MoEDims), _P, _P, _P, ctypes.POINTER(ExpertBankC), _P, _P, _SZ, _P],
                          ctypes.c_int),
    "mosaic_moe_routed_slots": ([ctypes.POINTER(MoEDims), _P, _P, _P, ctypes.POINTER(ExpertBankC), _P, _I, _P, _P, _SZ,
                                 _P], ctypes.c_int),
    "mosaic_expert_gemm_gu": ([ctypes.POINTER(MoEDims), _P, _P, _P, ctypes.POINTER(ExpertBankC), _P, _SZ, _P],
                              ctypes.c_int),
    "mosaic_expert_gemm_down": ([ctypes.POINTER(MoEDims), ctypes.POINTER(ExpertBankC), _P, _P, _SZ, _P],
                                ctypes.c_int),
    "mosaic_ep_dispatch": ([ctypes.POINTER(MoEDims), _I, _P, _P, _P, _P, _P, _P, _SZ, _P], ctypes.c_int),
    "mosaic_moe_expert_rows_workspace_bytes": ([ctypes.POINTER(MoEDims), _I], _SZ),
    "mosaic_moe_expert_rows": ([ctypes.POINTER(MoEDims), _I, _P, _I, _P, _P, _I, _I, ctypes.POINTER(ExpertBankC), _P,
                                _P, _SZ, _P], ctypes.c_int),
    "mosaic_ep_combine": ([ctypes.POINTER(MoEDims), _P, _P, _P, _P], ctypes.c_int),
    "mosaic_ep_region_bytes": ([ctypes.POINTER(EpPeersC)], _SZ),
    "mosaic_ep_region_alloc": ([_SZ, ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_uint8)], ctypes.c_int),
    "mosaic_ep_region_open": ([ctypes.POINTER(ctypes.c_uint8), ctypes.POINTER(ctypes.c_void_p)], ctypes.c_int),
    "mosaic_ep_region_close": ([_P], ctypes.c_int),
    "mosaic_ep_region_free": ([_P], ctypes.c_int),
    "mosaic_ep_region_view": ([ctypes.POINTER(EpPeersC), ctypes.POINTER(ctypes.c_void_p),
                               ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_void_p)], ctypes.c_int),
    "mosaic_ep_exchange_rows": ([ctypes.POINTER(EpPeersC), _P, _P, _P], ctypes.c_int),
    "mosaic_ep_dispatch_exchange": ([ctypes.POINTER(MoEDims), ctypes.POINTER(EpPeersC), _P, _P, _P, _P, _SZ, _P],
                                    ctypes.c_int),
    "mosaic_ep_expert_rows_workspace_bytes": ([ctypes.POINTER(MoEDims), ctypes.POINTER(EpPeersC)], _SZ),
    "mosaic_ep_return_partials": ([ctypes.POINTER(EpPeersC), _P, _P], ctypes.c_int),
    "mosaic_ep_expert_rows_return": ([ctypes.POINTER(MoEDims), ctypes.POINTER(EpPeersC), ctypes.POINTER(ExpertBankC),
                                      _P, _SZ, _P], ctypes.c_int),
    "mosaic_moe_expert_rows_dev": ([ctypes.POINTER(MoEDims), _I, _P, _P, _I, _P, _P, _I, _I,
                                    ctypes.POINTER(ExpertBankC), _P, _P, _SZ, _P], ctypes.c_int),
    "mosaic_read_error": ([_P, _I, ctypes.POINTER(ctypes.c_int32), _P], ctypes.c_int),
}

_LIB = None


def lib():
    """Load the CUDA library once; raise if it is not built."""
    global _LIB
    if _LIB is None:
        path = os.environ.get("MOSAIC_LIB", str(LIB_PATH))
        if not os.path.exists(path):
            raise RuntimeError(
                f"mosaic_b200 CUDA library not found at {path}; build it with "
                "`python -m mosaic_b200.build` (nvcc, sm_100a). There is no CPU fallback.")
        handle = ctypes.CDLL(path)
        for name, (args, res) in _SIGS.items():
            fn = getattr(handle, name)
            fn.argtypes = args
            fn.restype = res
        _LIB = handle
    return _LIB


def check(status: int, what: str) -> None:
    """Map a MOSAIC_ERR_* status to the exception class the reference raises."""
    if status == MOSAIC_OK:
        return
    msg = f"{what}: {lib().mosaic_status_string(status).decode()} (status {status})"
    if status in (MOSAIC_ERR_SHAPE, MOSAIC_ERR_ALIGN, MOSAIC_ERR_RANGE, MOSAIC_ERR_WORKSPACE):
        raise ValueError(msg)
    if status == MOSAIC_ERR_DTYPE:
        raise TypeError(msg)
    if status == MOSAIC_ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    raise MosaicError(msg)
