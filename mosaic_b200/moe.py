"""MoE module / operator API mirroring the reference, running on the B200 kernels.

Reference API mirrored (paths inside fazin-ahamed/Mosaic):

* ``Router`` <- ``mosaicvm/model/layers.py:118-150``: parameters ``weight`` [E, H]
  and ``e_score_correction_bias`` [E]; ``forward(x) -> (weights fp32 [bt, k],
  idx int64 [bt, k])``.  ``scoring_func`` "sigmoid" (vendored ``Gate``,
  ``.mosaicvm/source/inference_model.py:573-574``), "sqrtsoftplus"
  (``layers.py:110-115``) or "softmax" (``Gate``, ``:571-572``), plus the
  DeepSeek-V3 group limit (``n_group`` / ``topk_group``).
* ``HashRouter`` <- ``mosaicvm/model/layers.py:153-197``: ``weight``,
  ``tid2eid`` (None = salted fallback, an ``ExactContractError`` under the
  exact target), ``forward(x, token_ids=None)``.
* ``HashMoELayer`` <- ``mosaicvm/model/layers.py:376-405``:
  ``.hash_router``, ``forward(x, token_ids=None)``.
* ``MoELayer`` <- ``mosaicvm/model/layers.py:274-306``: ``.router``,
  ``.shared_expert`` (here the bank's last expert), ``.experts_gate_up()``,
  ``.experts_down()``, ``forward(x [b, t, H]) -> [b, t, H]`` in x's dtype.
* ``grouped_expert_forward`` <- ``mosaicvm/model/layers.py:329-373``.
* ``exact_moe`` <- ``mosaicvm/kernels/exact_moe.py:12-19`` (raises unless
  ``exact_target()``), with the tensor contract of ``fused_moe_qpa``
  (``mosaicvm/kernels/qpa_mma.py:681-691``): packed_gate_up uint8 [E, 2I, H/2],
  scale_gate_up E8M0 [E, 2I, H/32], packed_down [E, H, I/2], scale_down
  [E, H, I/32]; returns the routed output only.

Expert weights are MXFP4 banks (E2M1 codes + E8M0 per-32 scales) instead of
the reference's dense bf16 ``[E, H, I]`` test layers; everything else keeps the
reference names, argument meanings and exceptions.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass

import torch
from torch import nn

from . import _capi as C
from . import ops

_FALSE = ("0", "false", "False", "no", "")


def exact_target() -> bool:
    """True unless ``MOSAICVM_EXACT_TARGET`` is explicitly disabled (runtime/exact.py:19-20)."""
    return os.environ.get("MOSAICVM_EXACT_TARGET", "1") not in _FALSE


class ExactContractError(RuntimeError):
    """Raised when a configuration violates the exact contract (runtime/exact.py:23)."""


@dataclass
class MoEConfig:
    """MoE fields of the reference ``V4Config`` (mosaicvm/model/config.py:30-34, 51-55)
    plus the DeepSeek-V3 group limit and the expert activation format."""

    hidden_size: int = 7168
    moe_intermediate_size: int = 2048
    n_routed_experts: int = 256
    num_experts_per_tok: int = 8
    n_group: int = 8
    topk_group: int = 4
    routed_scaling_factor: float = 2.5
    scoring_func: str = "sigmoid"
    norm_topk_prob: bool = True
    swiglu_limit: float = 0.0
    n_shared_experts: int = 1
    act_mode: str = "bf16"  # "bf16" (decode) or "fp8" (reference act_quant semantics)

    def validate(self) -> None:
        if self.scoring_func not in C.SCORE_FUNCS:
            raise ValueError(f"unknown scoring_func {self.scoring_func}")
        if self.n_shared_experts not in (0, 1):
            raise ExactContractError("n_shared_experts must be 0 or 1")
        if self.act_mode not in ("bf16", "fp8"):
            raise ValueError(f"act_mode must be 'bf16' or 'fp8', got {self.act_mode}")

    def dims(self, tokens: int, has_shared: bool | None = None) -> C.MoEDims:
        self.validate()
        d = C.MoEDims()
        d.tokens = tokens
        d.hidden = self.hidden_size
        d.inter = self.moe_intermediate_size
        d.n_experts = self.n_routed_experts
        d.top_k = self.num_experts_per_tok
        d.n_group = self.n_group
        d.topk_group = self.topk_group
        d.act_mode = C.MOSAIC_ACT_BF16 if self.act_mode == "bf16" else C.MOSAIC_ACT_FP8
        d.norm_topk_prob = int(bool(self.norm_topk_prob))
        d.has_shared = int(self.n_shared_experts > 0 if has_shared is None else has_shared)
        d.route_scale = float(self.routed_scaling_factor)
        d.swiglu_limit = float(self.swiglu_limit)
        return d


class ExpertBank:
    """MXFP4 experts resident on one GPU.

    ``gu_packed`` uint8 [n, 2I, H/2] (gate rows then up rows), ``gu_scale`` E8M0
    bytes [n, 2I, H/32], ``dn_packed`` [n, H, I/2], ``dn_scale`` [n, H, I/32];
    with a shared expert it is the last of the n.  The layouts the MMA reads
    are built once here, invertibly (the bank re-layout of
    mosaicvm/kernels/qpa_mma.py:577-613): codes in contiguous 8 KB tiles
    (``gu_tiled``, ``dn_tiled``), scales in 512-byte chunks (``gu_sf``,
    ``dn_sf``).  ``keep_packed=False`` drops the reference-layout copies.
    """

    def __init__(self, gu_packed, gu_scale, dn_packed, dn_scale, *, has_shared: bool, keep_packed: bool = True):
        for t in (gu_packed, gu_scale, dn_packed, dn_scale):
            if t.device.type != "cuda":
                raise ValueError("ExpertBank tensors must be on a CUDA device")
        self.gu_packed = ops._u8(gu_packed).contiguous()
        self.gu_scale = ops._u8(gu_scale).contiguous()
        self.dn_packed = ops._u8(dn_packed).contiguous()
        self.dn_scale = ops._u8(dn_scale).contiguous()
        n, two_i, h_half = self.gu_packed.shape
        self.n_bank, self.inter, self.hidden = n, two_i // 2, h_half * 2
        if self.gu_scale.shape != (n, two_i, self.hidden // 32):
            raise ValueError("scale_gate_up must be [E, 2I, H/32]")
        if self.dn_packed.shape != (n, self.hidden, self.inter // 2):
            raise ValueError("packed_down must be [E, H, I/2]")
        if self.dn_scale.shape != (n, self.hidden, self.inter // 32):
            raise ValueError("scale_down must be [E, H, I/32]")
        self.has_shared = bool(has_shared)
        if self.hidden % 256:
            raise ValueError("hidden size must be a multiple of 256 (pairs of 128-row down blocks)")
        # gate rows / up rows, and the two hidden halves of down, interleaved per
        # (128-row block, K-tile): each GEMM stage loads a pair of adjacent tiles
        self.gu_sf = ops.prepack_scales(self.gu_scale, halves=2)
        self.dn_sf = ops.prepack_scales(self.dn_scale, halves=2)
        self.gu_tiled = ops.repack_weights(self.gu_packed, halves=2)
        self.dn_tiled = ops.repack_weights(self.dn_packed, halves=2)
        if not keep_packed:
            self.gu_packed = self.dn_packed = None

    @classmethod
    def from_dense(cls, w_gu, w_dn, *, has_shared: bool, device="cuda"):
        """Quantise dense fp32 weights (lists of [2I, H] and [H, I]) to MXFP4 on the GPU."""
        gu = [ops.pack_mxfp4_nk(w.to(device)) for w in w_gu]
        dn = [ops.pack_mxfp4_nk(w.to(device)) for w in w_dn]
        return cls(torch.stack([p for p, _ in gu]), torch.stack([s for _, s in gu]),
                   torch.stack([p for p, _ in dn]), torch.stack([s for _, s in dn]), has_shared=has_shared)

    def c_struct(self) -> C.ExpertBankC:
        b = C.ExpertBankC()
        b.gu_tiled = self.gu_tiled.data_ptr()
        b.gu_sf = self.gu_sf.data_ptr()
        b.dn_tiled = self.dn_tiled.data_ptr()
        b.dn_sf = self.dn_sf.data_ptr()
        return b

    def nbytes(self) -> int:
        """Device bytes the kernels read from (tiled codes + scale chunks)."""
        return sum(t.numel() for t in (self.gu_tiled, self.gu_sf, self.dn_tiled, self.dn_sf))


class _Workspace:
    """Caller-owned workspace of the C ABI, cached per dims."""

    def __init__(self):
        self._key = None
        self.buf = None

    def get(self, dims: C.MoEDims, device) -> torch.Tensor:
        device = torch.device(device)
        if device.type == "cuda" and device.index is None:  # "cuda" and "cuda:<current>" are one workspace
            device = torch.device("cuda", torch.cuda.current_device())
        key = (bytes(dims), device)
        if key != self._key:
            n = C.lib().mosaic_moe_workspace_bytes(ctypes.byref(dims))
            if n == 0:
                C.check(C.MOSAIC_ERR_SHAPE, "mosaic_moe_workspace_bytes")
            self.buf = torch.empty(n, dtype=torch.uint8, device=device)
            self._key = key
        return self.buf


class Router(nn.Module):
    """Linear + scores + bias-corrected (group-limited) top-k (layers.py:118-150)."""

    def __init__(self, cfg: MoEConfig):
        super().__init__()
        self.cfg = cfg
        self.weight = nn.Parameter(torch.zeros(cfg.n_routed_experts, cfg.hidden_size), requires_grad=False)
        self.e_score_correction_bias = nn.Parameter(torch.zeros(cfg.n_routed_experts), requires_grad=False)

    def forward(self, x):
        c = self.cfg
        return ops.router(x.to(torch.bfloat16).contiguous(), self.weight.float().contiguous(),
                          self.e_score_correction_bias.float().contiguous(), top_k=c.num_experts_per_tok,
                          n_group=c.n_group, topk_group=c.topk_group, route_scale=c.routed_scaling_factor,
                          norm_topk_prob=c.norm_topk_prob, score_func=c.scoring_func)


class HashRouter(nn.Module):
    """Hash-routed layers (layers.py:153-197): ids from ``tid2eid``, weights the
    router scores gathered there, normalised unless the score is softmax, times
    ``routed_scaling_factor``.  Without a table: ``ExactContractError`` under the
    exact target, else the salted hash (one expert per token, weight
    ``routed_scaling_factor``)."""

    def __init__(self, cfg: MoEConfig, layer_idx: int):
        super().__init__()
        cfg.validate()
        self.cfg = cfg
        self.layer_idx = layer_idx
        self.weight = nn.Parameter(torch.zeros(cfg.n_routed_experts, cfg.hidden_size), requires_grad=False)
        self.tid2eid = None
        self._table = (None, None)  # (source tensor, checked device int32 table)

    def table(self, device):
        """The int32 [V, k] device table, range-checked once per ``tid2eid`` tensor.

        An id outside [0, E) raises ``IndexError``, as the reference's gather would."""
        src, tab = self._table
        if src is not self.tid2eid or tab is None or tab.device != torch.device(device):
            tab = ops.hash_table(self.tid2eid, device)
            if int(tab.min()) < 0 or int(tab.max()) >= self.cfg.n_routed_experts:
                raise IndexError(f"HashRouter layer {self.layer_idx}: tid2eid holds an id outside "
                                 f"[0, {self.cfg.n_routed_experts})")
            self._table = (self.tid2eid, tab)
        return tab

    def route_ext(self, x, token_ids):
        """(mosaic_route_ext, tensors it points at, top_k) of one call."""
        c = self.cfg
        n = x.shape[0]
        tok = None
        if token_ids is not None:
            tok = token_ids.reshape(-1)
            if tok.numel() != n:
                raise ValueError(f"token_ids has {tok.numel()} entries for {n} tokens")
            tok = tok.to(device=x.device, dtype=torch.int64).contiguous()
        if self.tid2eid is None:
            if exact_target():
                raise ExactContractError(f"HashRouter layer {self.layer_idx}: tid2eid required under exact target")
            ext = ops.route_ext(c.scoring_func, token_ids=tok, hash_routing=True, layer_idx=self.layer_idx)
            return ext, (tok,), 1
        tab = self.table(x.device)
        ext = ops.route_ext(c.scoring_func, tid2eid=tab, token_ids=tok, hash_routing=True, layer_idx=self.layer_idx)
        return ext, (tok, tab), tab.shape[1]

    def forward(self, x, token_ids=None):
        c = self.cfg
        if self.tid2eid is None and exact_target():
            raise ExactContractError(f"HashRouter layer {self.layer_idx}: tid2eid required under exact target")
        tab = None if self.tid2eid is None else self.table(x.device)
        return ops.hash_router(x.to(torch.bfloat16).contiguous(), self.weight.float().contiguous(), tab, token_ids,
                               n_experts=c.n_routed_experts, layer_idx=self.layer_idx, score_func=c.scoring_func,
                               route_scale=c.routed_scaling_factor)


class MoELayer(nn.Module):
    """Shared expert + routed experts of one layer (layers.py:274-306) on MXFP4 banks."""

    def __init__(self, cfg: MoEConfig, bank: ExpertBank | None = None):
        super().__init__()
        cfg.validate()
        self.cfg = cfg
        self.router = Router(cfg)
        self.bank = bank
        self._ws = _Workspace()
        self.last_weights = None
        self.last_idx = None

    @property
    def shared_expert(self):
        """Index of the shared expert inside the bank (the last one), or None."""
        if self.bank is None or not self.bank.has_shared:
            return None
        return self.bank.n_bank - 1

    def experts_gate_up(self):
        if self.bank is None:
            raise NotImplementedError("MoELayer has no expert bank")
        return self.bank.gu_packed, self.bank.gu_scale

    def experts_down(self):
        if self.bank is None:
            raise NotImplementedError("MoELayer has no expert bank")
        return self.bank.dn_packed, self.bank.dn_scale

    def workspace(self, tokens: int, device) -> torch.Tensor:
        return self._ws.get(self.cfg.dims(tokens, self.bank.has_shared), device)

    def forward(self, x):
        if self.bank is None:
            raise NotImplementedError("MoELayer has no expert bank")
        shape = x.shape
        xf = x.reshape(-1, shape[-1]).to(torch.bfloat16).contiguous()
        if xf.device.type != "cuda":
            raise ValueError("MoELayer.forward requires a CUDA input (no CPU path)")
        ext = None if self.cfg.scoring_func == "sigmoid" else ops.route_ext(self.cfg.scoring_func)
        y = self._forward(xf, ext, self.cfg.num_experts_per_tok, self.cfg.norm_topk_prob,
                          self.router.weight.data, self.router.e_score_correction_bias.data)
        return y.to(x.dtype).view(shape)

    def _forward(self, xf, ext, top_k, norm, router_weight, router_bias):
        """One mosaic_moe_forward(_ext) call on bf16 rows ``xf`` [T, H]."""
        t = xf.shape[0]
        dims = self.cfg.dims(t, self.bank.has_shared)
        dims.top_k = top_k
        dims.norm_topk_prob = int(bool(norm))
        ws = self._ws.get(dims, xf.device)
        y = torch.empty_like(xf)
        w = torch.empty(t, top_k, dtype=torch.float32, device=xf.device)
        idx = torch.empty(t, top_k, dtype=torch.int64, device=xf.device)
        bank = self.bank.c_struct()
        rw = None if router_weight is None else router_weight.float().contiguous()
        rb = None if router_bias is None else router_bias.float().contiguous()
        if ext is None:
            st = C.lib().mosaic_moe_forward(ctypes.byref(dims), ops._ptr(xf), ops._ptr(rw), ops._ptr(rb),
                                            ctypes.byref(bank), ops._ptr(y), ops._ptr(w), ops._ptr(idx), ops._ptr(ws),
                                            ws.numel(), ops._stream())
            C.check(st, "mosaic_moe_forward")
        else:
            st = C.lib().mosaic_moe_forward_ext(ctypes.byref(dims), ctypes.byref(ext), ops._ptr(xf), ops._ptr(rw),
                                                ops._ptr(rb), ctypes.byref(bank), ops._ptr(y), ops._ptr(w),
                                                ops._ptr(idx), ops._ptr(ws), ws.numel(), ops._stream())
            C.check(st, "mosaic_moe_forward_ext")
        self.last_weights, self.last_idx = w, idx
        return y


class HashMoELayer(MoELayer):
    """MoE layer with hash routing (layers.py:376-405) on an MXFP4 bank:
    ``.hash_router`` (a :class:`HashRouter`), ``forward(x, token_ids=None)``."""

    def __init__(self, cfg: MoEConfig, layer_idx: int, bank: ExpertBank | None = None):
        super().__init__(cfg, bank)
        self.router = None
        self.hash_router = HashRouter(cfg, layer_idx)

    def forward(self, x, token_ids=None):
        if self.bank is None:
            raise NotImplementedError("MoELayer has no expert bank")
        shape = x.shape
        xf = x.reshape(-1, shape[-1]).to(torch.bfloat16).contiguous()
        if xf.device.type != "cuda":
            raise ValueError("HashMoELayer.forward requires a CUDA input (no CPU path)")
        ext, keep, k = self.hash_router.route_ext(xf, token_ids)
        y = self._forward(xf, ext, k, self.cfg.scoring_func != "softmax", self.hash_router.weight.data, None)
        del keep
        return y.to(x.dtype).view(shape)


def _routed(cfg: MoEConfig, x, expert_ids, expert_weights, bank: ExpertBank, *, include_shared: bool,
            workspace: _Workspace | None = None, split: bool = False):
    """Routed experts through ``mosaic_moe_routed``; ``split`` runs the same
    work as ``mosaic_expert_gemm_gu`` then ``mosaic_expert_gemm_down`` (the
    reference's gate/up and down ``_run_two_queues`` calls, qpa_mma.py:750-772)."""
    if x.device.type != "cuda":
        raise ValueError("MoE expert path requires CUDA tensors")
    xf = x.reshape(-1, x.shape[-1]).to(torch.bfloat16).contiguous()
    t = xf.shape[0]
    ids = expert_ids.reshape(t, -1).to(torch.int64).contiguous()
    if ids.shape[1] != cfg.num_experts_per_tok:
        raise ValueError(f"expert_ids must be [T, {cfg.num_experts_per_tok}]")
    w = None if expert_weights is None else expert_weights.reshape(t, -1).to(torch.float32).contiguous()
    dims = cfg.dims(t, include_shared)
    ws = (workspace or _Workspace()).get(dims, xf.device)
    y = torch.empty_like(xf)
    b = bank.c_struct()
    if split:
        st = C.lib().mosaic_expert_gemm_gu(ctypes.byref(dims), ops._ptr(xf), ops._ptr(ids), ops._ptr(w),
                                           ctypes.byref(b), ops._ptr(ws), ws.numel(), ops._stream())
        C.check(st, "mosaic_expert_gemm_gu")
        st = C.lib().mosaic_expert_gemm_down(ctypes.byref(dims), ctypes.byref(b), ops._ptr(y), ops._ptr(ws),
                                             ws.numel(), ops._stream())
        C.check(st, "mosaic_expert_gemm_down")
        return y
    st = C.lib().mosaic_moe_routed(ctypes.byref(dims), ops._ptr(xf), ops._ptr(ids), ops._ptr(w), ctypes.byref(b),
                                   ops._ptr(y), ops._ptr(ws), ws.numel(), ops._stream())
    C.check(st, "mosaic_moe_routed")
    return y


def grouped_expert_forward(x, scores, idx, gate_up, down=None, n_experts=None, swiglu_limit: float = 0.0,
                           act_mode: str = "bf16"):
    """Routed experts with the reference semantics (layers.py:329-373) on the GPU.

    ``gate_up`` is an :class:`ExpertBank` (``down`` ignored) or the reference's
    packed pair ``(packed_gate_up, scale_gate_up)`` with ``down =
    (packed_down, scale_down)``.  Route weight before the down projection,
    ordered fp32 combine in ascending expert id, output in x's dtype.
    """
    if isinstance(gate_up, ExpertBank):
        bank = gate_up
    else:
        (pgu, sgu), (pdn, sdn) = gate_up, down
        bank = ExpertBank(pgu, sgu, pdn, sdn, has_shared=False)
    e = n_experts if n_experts is not None else bank.n_bank - (1 if bank.has_shared else 0)
    cfg = MoEConfig(hidden_size=bank.hidden, moe_intermediate_size=bank.inter, n_routed_experts=e,
                    num_experts_per_tok=idx.shape[-1], n_group=1, topk_group=1, swiglu_limit=swiglu_limit,
                    act_mode=act_mode, n_shared_experts=0)
    return _routed(cfg, x, idx, scores, bank, include_shared=False).to(x.dtype)


def exact_moe(x, expert_ids, expert_weights, packed_gate_up, scale_gate_up, packed_down, scale_down,
              swiglu_limit: float = 0.0, act_mode: str = "fp8"):
    """Routed MoE with the reference exact contract (mosaicvm/kernels/exact_moe.py:12-19).

    Requires ``exact_target()``.  ``act_mode="fp8"`` is the reference's source
    semantics (act_quant_ref activations, bf16-rounded linears).
    """
    if not exact_target():
        raise RuntimeError("exact_moe requires MOSAICVM_EXACT_TARGET=1")
    bank = ExpertBank(packed_gate_up, scale_gate_up, packed_down, scale_down, has_shared=False)
    ids = expert_ids if expert_ids.dim() == 2 else expert_ids.reshape(-1, 1)
    cfg = MoEConfig(hidden_size=bank.hidden, moe_intermediate_size=bank.inter, n_routed_experts=bank.n_bank,
                    num_experts_per_tok=ids.shape[1], n_group=1, topk_group=1, swiglu_limit=swiglu_limit,
                    act_mode=act_mode, n_shared_experts=0)
    return _routed(cfg, x, ids, expert_weights, bank, include_shared=False).to(x.dtype)
