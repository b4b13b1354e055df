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


def score_func_code(score_func: str) -> int:
    """``scoring_func`` name (V4Config / ModelArgs.score_func) -> enum mosaic_score_func."""
    try:
        return C.SCORE_FUNCS[score_func]
    except KeyError:
        raise ValueError(f"unknown scoring_func {score_func}") from None


def route_ext(score_func: str = "sigmoid", *, tid2eid: torch.Tensor | None = None,
              token_ids: torch.Tensor | None = None, hash_routing: bool = False,
              layer_idx: int = 0) -> C.RouteExtC:
    """The ``mosaic_route_ext`` of a router call (the tensors must outlive the call)."""
    ext = C.RouteExtC()
    ext.score_func = score_func_code(score_func)
    ext.hash = int(bool(hash_routing))
    ext.layer_idx = int(layer_idx)
    ext.table_rows = 0 if tid2eid is None else int(tid2eid.shape[0])
    ext.tid2eid = None if tid2eid is None else tid2eid.data_ptr()
    ext.token_ids = None if token_ids is None else token_ids.data_ptr()
    return ext


def router(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None, *, top_k: int, n_group: int = 1,
           topk_group: int = 1, route_scale: float = 1.0, norm_topk_prob: bool = True,
           score_func: str = "sigmoid"):
    """(Group-limited) top-k router -> (weights fp32 [T, k], idx int64 [T, k]).

    ``score_func``: "sigmoid" (mosaic_router), "sqrtsoftplus" or "softmax"
    (mosaic_router_ext).
    """
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
    if score_func == "sigmoid":
        st = lib.mosaic_router(_ptr(x), _ptr(weight), _ptr(bias), t, h, e, top_k, n_group, topk_group,
                               float(route_scale), int(bool(norm_topk_prob)), _ptr(w), _ptr(idx), _ptr(ws),
                               ws.numel(), _stream())
        C.check(st, "mosaic_router")
    else:
        ext = route_ext(score_func)
        st = lib.mosaic_router_ext(ctypes.byref(ext), _ptr(x), _ptr(weight), _ptr(bias), t, h, e, top_k, n_group,
                                   topk_group, float(route_scale), int(bool(norm_topk_prob)), _ptr(w), _ptr(idx),
                                   _ptr(ws), ws.numel(), _stream())
        C.check(st, "mosaic_router_ext")
    return w, idx


def hash_table(tid2eid: torch.Tensor, device) -> torch.Tensor:
    """tid2eid [V] or [V, k] (any integer dtype) -> contiguous int32 [V, k] on ``device``."""
    if tid2eid.dtype.is_floating_point or tid2eid.dtype == torch.bool:
        raise ValueError("tid2eid must be an integer tensor")
    table = tid2eid.reshape(tid2eid.shape[0], -1) if tid2eid.dim() != 1 else tid2eid.reshape(-1, 1)
    if table.dim() != 2 or table.shape[0] < 1:
        raise ValueError("tid2eid must be [V] or [V, k] with V >= 1")
    if table.dtype != torch.int32:
        lo, hi = int(table.min()), int(table.max())
        if lo < -2 ** 31 or hi >= 2 ** 31:
            raise ValueError("tid2eid entries do not fit int32")
        table = table.to(torch.int32)
    return table.to(device).contiguous()


def hash_router(x: torch.Tensor, weight: torch.Tensor | None, tid2eid: torch.Tensor | None,
                token_ids: torch.Tensor | None = None, *, n_experts: int, layer_idx: int = 0,
                score_func: str = "sqrtsoftplus", route_scale: float = 1.0, norm_topk_prob: bool | None = None):
    """Hash routing (mosaicvm/model/layers.py:171-197) -> (weights fp32 [T, k], idx int64 [T, k]).

    With ``tid2eid`` ([V] or [V, k]): ids = tid2eid[token_ids mod V], weights
    the scores gathered there, normalised unless ``score_func`` is softmax
    (``norm_topk_prob`` overrides), times ``route_scale``.  Without it: the
    salted hash of ``layer_idx``, one expert per token, weight ``route_scale``
    (the caller enforces the exact-target contract).
    """
    _need_cuda(x, what="hash_router")
    if x.dim() != 2:
        raise ValueError("hash_router expects x [T, H]")
    t, h = x.shape
    if token_ids is None:
        tok = None
    else:
        tok = token_ids.reshape(-1)
        if tok.numel() != t:
            raise ValueError(f"token_ids has {tok.numel()} entries for {t} tokens")
        if tok.dtype.is_floating_point or tok.dtype == torch.bool:
            raise ValueError("token_ids must be an integer tensor")
        tok = tok.to(device=x.device, dtype=torch.int64).contiguous()
    if norm_topk_prob is None:
        norm_topk_prob = score_func != "softmax"
    lib = C.lib()
    if tid2eid is None:
        if layer_idx < 0:
            raise ValueError("layer_idx must be >= 0")
        ext = route_ext(score_func, token_ids=tok, hash_routing=True, layer_idx=layer_idx)
        w = torch.empty(t, 1, dtype=torch.float32, device=x.device)
        idx = torch.empty(t, 1, dtype=torch.int64, device=x.device)
        st = lib.mosaic_router_ext(ctypes.byref(ext), None, None, None, t, h, n_experts, 1, 1, 1, float(route_scale),
                                   int(bool(norm_topk_prob)), _ptr(w), _ptr(idx), None, 0, _stream())
        C.check(st, "mosaic_router_ext")
        return w, idx
    if x.dtype != torch.bfloat16:
        raise ValueError("hash_router expects bf16 x [T, H]")
    _need_cuda(weight, what="hash_router")
    if weight is None or weight.dtype != torch.float32 or weight.shape != (n_experts, h):
        raise ValueError("hash_router expects fp32 weight [E, H]")
    table = hash_table(tid2eid, x.device)
    k = table.shape[1]
    ext = route_ext(score_func, tid2eid=table, token_ids=tok, hash_routing=True, layer_idx=layer_idx)
    ws = torch.empty(max(lib.mosaic_router_workspace_bytes(t, h, n_experts), 256), dtype=torch.uint8,
                     device=x.device)
    w = torch.empty(t, k, dtype=torch.float32, device=x.device)
    idx = torch.empty(t, k, dtype=torch.int64, device=x.device)
    st = lib.mosaic_router_ext(ctypes.byref(ext), _ptr(x), _ptr(weight), None, t, h, n_experts, k, 1, 1,
                               float(route_scale), int(bool(norm_topk_prob)), _ptr(w), _ptr(idx), _ptr(ws),
                               ws.numel(), _stream())
    C.check(st, "mosaic_router_ext")
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
