"""Tensor-level operators over the C ABI (torch supplies device memory and streams).

Each function validates its tensors the way the reference operator does
(``ValueError`` for shape / device contracts), passes raw device pointers and
the current CUDA stream to ``libmosaic_moe.so`` and returns freshly allocated
outputs.  Nothing here computes on the CPU.
"""
from __future__ import annotations

import ctypes

import torch

from . import _capi as C


def _stream() -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _ptr(t: torch.Tensor | None) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr() if t is not None else 0)


def _need_cuda(*ts: torch.Tensor, what: str) -> None:
    for t in ts:
        if t is None:
            continue
        if t.device.type != "cuda":
            raise ValueError(f"{what} requires CUDA tensors")
        if not t.is_contiguous():
            raise ValueError(f"{what} requires contiguous tensors")


def _u8(t: torch.Tensor) -> torch.Tensor:
    if t.dtype == torch.uint8:
        return t
    if t.dtype in (torch.int8, torch.float8_e8m0fnu, torch.float8_e4m3fn):
        return t.view(torch.uint8)
    raise TypeError(f"expected uint8-compatible tensor, got {t.dtype}")


def router(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None, *, top_k: int, n_group: int = 1,
           topk_group: int = 1, route_scale: float = 1.0, norm_topk_prob: bool = True):
    """Sigmoid (group-limited) top-k router -> (weights fp32 [T, k], idx int64 [T, k])."""
    _need_cuda(x, weight, bias, what="router")
    if x.dtype != torch.bfloat16 or x.dim() != 2:
        raise ValueError("router expects bf16 x [T, H]")
    if weight.dtype != torch.float32 or bias is not None and bias.dtype != torch.float32:
        raise ValueError("router expects fp32 weight [E, H] and bias [E]")
    t, h = x.shape
    e = weight.shape[0]
    if weight.shape != (e, h) or (bias is not None and bias.shape != (e,)):
        raise ValueError("router weight/bias shape mismatch")
    lib = C.lib()
    ws_bytes = lib.mosaic_router_workspace_bytes(t, h, e)
    ws = torch.empty(max(ws_bytes, 256), dtype=torch.uint8, device=x.device)
    w = torch.empty(t, top_k, dtype=torch.float32, device=x.device)
    idx = torch.empty(t, top_k, dtype=torch.int64, device=x.device)
    st = lib.mosaic_router(_ptr(x), _ptr(weight), _ptr(bias), t, h, e, top_k, n_group, topk_group,
                           float(route_scale), int(bool(norm_topk_prob)), _ptr(w), _ptr(idx), _ptr(ws), ws.numel(),
                           _stream())
    C.check(st, "mosaic_router")
    return w, idx


def router_noalloc(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None, weights_out: torch.Tensor,
                   idx_out: torch.Tensor, *, top_k: int, n_group: int = 1, topk_group: int = 1,
                   route_scale: float = 1.0, norm_topk_prob: bool = True) -> None:
    """:func:`router` into caller-owned outputs through ``mosaic_router_noalloc``.

    Neither this wrapper nor the library allocates device memory: inputs must
    already be contiguous CUDA tensors of the right dtypes (no conversion), the
    split-K scratch is the library's fixed per-device array, and calls that
    overlap on one device race on it.  No counterpart in the reference.
    """
    _need_cuda(x, weight, bias, weights_out, idx_out, what="router_noalloc")
    if x.dtype != torch.bfloat16 or x.dim() != 2:
        raise ValueError("router_noalloc expects bf16 x [T, H]")
    if weight.dtype != torch.float32 or bias is not None and bias.dtype != torch.float32:
        raise ValueError("router_noalloc expects fp32 weight [E, H] and bias [E]")
    t, h = x.shape
    e = weight.shape[0]
    if weight.shape != (e, h) or (bias is not None and bias.shape != (e,)):
        raise ValueError("router weight/bias shape mismatch")
    if weights_out.dtype != torch.float32 or weights_out.shape != (t, top_k):
        raise ValueError("weights_out must be fp32 [T, top_k]")
    if idx_out.dtype != torch.int64 or idx_out.shape != (t, top_k):
        raise ValueError("idx_out must be int64 [T, top_k]")
    st = C.lib().mosaic_router_noalloc(_ptr(x), _ptr(weight), _ptr(bias), t, h, e, top_k, n_group, topk_group,
                                       float(route_scale), int(bool(norm_topk_prob)), _ptr(weights_out),
                                       _ptr(idx_out), _stream())
    C.check(st, "mosaic_router_noalloc")


def layout_assignments(expert_ids: torch.Tensor, n_experts: int):
    """ids [A] -> (sorted_ids int64 [A], perm int64 [A], offsets int32 [E+1], counts int32 [E]).

    Same contract as mosaicvm/kernels/moe_layout.py:8-27 (ValueError off CUDA);
    the permutation is the stable one.
    """
    if expert_ids.device.type != "cuda":
        raise ValueError("layout_assignments requires CUDA expert_ids")
    ids = expert_ids.reshape(-1).to(torch.int64).contiguous()
    a = ids.numel()
    sorted_ids = torch.empty(a, dtype=torch.int64, device=ids.device)
    perm = torch.empty(a, dtype=torch.int64, device=ids.device)
    offsets = torch.empty(n_experts + 1, dtype=torch.int32, device=ids.device)
    counts = torch.empty(n_experts, dtype=torch.int32, device=ids.device)
    st = C.lib().mosaic_layout_assignments(_ptr(ids), a, n_experts, _ptr(sorted_ids), _ptr(perm), _ptr(offsets),
                                           _ptr(counts), _stream())
    C.check(st, "mosaic_layout_assignments")
    return sorted_ids, perm, offsets, counts


def emit_tiles(counts: torch.Tensor, block_m: int = 8, max_tiles: int | None = None):
    """counts [E] int32 -> (expert_index, m_start, n_tiles [1], tile_rows) on the GPU
    (mosaicvm/kernels/w4a16_grouped.py:151-169)."""
    _need_cuda(counts, what="emit_tiles")
    c = counts.to(torch.int32).contiguous()
    e = c.numel()
    cap = int(max_tiles) if max_tiles is not None else max(e, 1)
    ei = torch.empty(cap, dtype=torch.int32, device=c.device)
    ms = torch.empty(cap, dtype=torch.int32, device=c.device)
    nt = torch.empty(1, dtype=torch.int32, device=c.device)
    tr = torch.empty(cap, dtype=torch.int32, device=c.device)
    st = C.lib().mosaic_emit_tiles(_ptr(c), e, block_m, cap, _ptr(ei), _ptr(ms), _ptr(nt), _ptr(tr), _stream())
    C.check(st, "mosaic_emit_tiles")
    return ei, ms, nt, tr


def act_quant(x: torch.Tensor, block: int = 128):
    """act_quant_ref on the GPU: x [M, K] bf16 -> (e4m3fn [M, K], fp32 pow2 scales [M, K/128])."""
    if x.dim() != 2:
        raise ValueError(f"act_quant expects [M, K], got {tuple(x.shape)}")
    if block != 128 or x.shape[1] % 128:
        raise ValueError(f"K={x.shape[1]} must be a multiple of act block 128")
    _need_cuda(x, what="act_quant")
    x = x.to(torch.bfloat16).contiguous()
    m, k = x.shape
    q = torch.empty(m, k, dtype=torch.uint8, device=x.device)
    s = torch.empty(m, k // 128, dtype=torch.float32, device=x.device)
    C.check(C.lib().mosaic_act_quant(_ptr(x), m, k, _ptr(q), _ptr(s), _stream()), "mosaic_act_quant")
    return q.view(torch.float8_e4m3fn), s


def pack_mxfp4_nk(w: torch.Tensor):
    """w [N, K] -> (packed uint8 [N, K/2], E8M0 scale uint8 [N, K/32]) on the GPU
    (bit-identical to mosaicvm/kernels/fp4_source.py:35-64)."""
    if w.dim() != 2:
        raise ValueError(f"pack_mxfp4_nk expects [N, K], got {tuple(w.shape)}")
    n, k = w.shape
    if k % 32:
        raise ValueError(f"K={k} must be a multiple of MX_BLOCK=32")
    _need_cuda(w, what="pack_mxfp4_nk")
    w = w.to(torch.float32).contiguous()
    packed = torch.empty(n, k // 2, dtype=torch.uint8, device=w.device)
    scale = torch.empty(n, k // 32, dtype=torch.uint8, device=w.device)
    C.check(C.lib().mosaic_pack_mxfp4(_ptr(w), n, k, _ptr(packed), _ptr(scale), _stream()), "mosaic_pack_mxfp4")
    return packed, scale


def prepack_scales(scale: torch.Tensor, halves: int = 1) -> torch.Tensor:
    """E8M0 [n_mats, rows, K/32] -> MMA scale chunks [n_mats, rows/128/halves, K/128, halves, 512] (uint8).

    halves=2 interleaves the two row halves (gate rows, up rows) per K-tile."""
    scale = _u8(scale).contiguous()
    if scale.dim() == 2:
        scale = scale.unsqueeze(0)
    _need_cuda(scale, what="prepack_scales")
    n, rows, kb = scale.shape
    if rows % (128 * halves) or (kb * 32) % 128:
        raise ValueError("prepack_scales needs rows % (128 * halves) == 0 and K % 128 == 0")
    out = torch.empty(n, rows // 128 // halves, kb // 4, halves, 512, dtype=torch.uint8, device=scale.device)
    C.check(C.lib().mosaic_prepack_scales(_ptr(scale), n, rows, kb * 32, halves, _ptr(out), _stream()),
            "mosaic_prepack_scales")
    return out


def repack_weights(packed: torch.Tensor, halves: int = 1) -> torch.Tensor:
    """Packed E2M1 codes [n_mats, rows, K/2] -> contiguous 8 KB MMA tiles
    [n_mats, rows/128/halves, K/128, halves, 128, 64] (halves=2: gate/up interleave)."""
    packed = _u8(packed).contiguous()
    if packed.dim() == 2:
        packed = packed.unsqueeze(0)
    _need_cuda(packed, what="repack_weights")
    n, rows, half_k = packed.shape
    k = half_k * 2
    if rows % (128 * halves) or k % 128:
        raise ValueError("repack_weights needs rows % (128 * halves) == 0 and K % 128 == 0")
    out = torch.empty(n, rows // 128 // halves, k // 128, halves, 128, 64, dtype=torch.uint8, device=packed.device)
    C.check(C.lib().mosaic_repack_weights(_ptr(packed), n, rows, k, halves, _ptr(out), _stream()),
            "mosaic_repack_weights")
    return out


def read_error(workspace: torch.Tensor, reset: bool = True) -> int:
    """Device error word of a layer workspace (synchronises the stream)."""
    code = ctypes.c_int32(0)
    C.check(C.lib().mosaic_read_error(_ptr(workspace), int(reset), ctypes.byref(code), _stream()),
            "mosaic_read_error")
    return int(code.value)
