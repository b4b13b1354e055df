"""Expert-parallel MoE layer: one process per GPU, experts sharded by rank.

Rank d of W owns the contiguous routed experts [d*E/W, (d+1)*E/W) and a
replica of the shared expert (the expert-sharded ``MoE`` of
``.mosaicvm/source/inference_model.py:614-650``, whose cross-rank
``all_reduce`` becomes a dispatch / combine all-to-all here).  Every rank
routes its own tokens with the replicated router.  One layer step:

1. ``mosaic_router`` on the local tokens;
2. ``mosaic_ep_dispatch``: assignments sorted by expert id (hence grouped by
   destination rank) and gathered into send rows (token values + local expert
   id + route weight), with per-destination row counts;
3. all-to-all of the counts, then of the send rows (NCCL over NVLink);
4. the shared expert on the local tokens, overlapping the exchange;
5. ``mosaic_moe_expert_rows`` on the received rows: one partial per row;
6. all-to-all of the partials back to their source ranks, in send order;
7. ``mosaic_ep_combine``: each token's partials summed in ascending expert id.

Because the order of every fp32 sum is the single-GPU layer's, the output is
bit-identical to ``MoELayer`` on the same tokens.  The exchange sizes are read
on the host after the count exchange (one synchronisation per layer).

The kernels are reached through a ``kernels`` object; the default is the CUDA
library and there is no CPU path in this package.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist
from torch import nn

from . import _capi as C
from . import ops
from .moe import ExpertBank, HashRouter, MoEConfig, Router


def expert_range(n_experts: int, world: int, rank: int) -> tuple[int, int]:
    """Routed experts [lo, hi) owned by ``rank``."""
    if world < 1 or n_experts % world:
        raise ValueError(f"{n_experts} experts do not split evenly over {world} ranks")
    per = n_experts // world
    return rank * per, (rank + 1) * per


def shard_bank(gu_packed, gu_scale, dn_packed, dn_scale, *, rank: int, world: int, n_experts: int,
               has_shared: bool, keep_packed: bool = False) -> ExpertBank:
    """Local bank of ``rank`` from a reference-layout bank of E routed experts
    (+ the shared expert as expert E): its expert range, then the shared expert."""
    lo, hi = expert_range(n_experts, world, rank)
    sel = list(range(lo, hi)) + ([n_experts] if has_shared else [])
    sel_t = torch.tensor(sel, device=gu_packed.device)
    pick = [t.index_select(0, sel_t) for t in (gu_packed, gu_scale, dn_packed, dn_scale)]
    return ExpertBank(*pick, has_shared=has_shared, keep_packed=keep_packed)


class _Buffer:
    """Device byte buffer that grows to the largest size asked for."""

    def __init__(self):
        self.t = None

    def get(self, nbytes: int, device) -> torch.Tensor:
        nbytes = max(int(nbytes), 256)
        if self.t is None or self.t.numel() < nbytes or self.t.device != torch.device(device):
            self.t = torch.empty(nbytes, dtype=torch.uint8, device=device)
        return self.t


class _RawOut:
    """A raw device address passed where a tensor output is expected."""

    def __init__(self, ptr: int):
        self._ptr = ptr

    def data_ptr(self) -> int:
        return self._ptr


class CudaEPKernels:
    """The CUDA kernels of one expert-parallel rank, through the C ABI."""

    def __init__(self):
        self._ws_dispatch = _Buffer()
        self._ws_rows = _Buffer()
        self._ws_shared = _Buffer()

    def route(self, router: Router, x: torch.Tensor):
        return router(x)

    def route_hash(self, router: HashRouter, x: torch.Tensor, token_ids):
        return router(x, token_ids)

    def dispatch(self, dims: C.MoEDims, world: int, x, idx, w):
        lib = C.lib()
        ws = self._ws_dispatch.get(lib.mosaic_moe_workspace_bytes(ctypes.byref(dims)), x.device)
        a = dims.tokens * dims.top_k
        send = torch.empty(a, C.ep_row_bytes(dims.hidden), dtype=torch.uint8, device=x.device)
        counts = torch.empty(world, dtype=torch.int32, device=x.device)
        C.check(lib.mosaic_ep_dispatch(ctypes.byref(dims), world, ops._ptr(x), ops._ptr(idx), ops._ptr(w),
                                       ops._ptr(send), ops._ptr(counts), ops._ptr(ws), ws.numel(), ops._stream()),
                "mosaic_ep_dispatch")
        return send, counts, ws

    def _rows(self, dims_local: C.MoEDims, bank: ExpertBank, rows: int, x_ptr: int, ldx: int, ids_ptr, w_ptr,
              stride: int, default_id: int, out: torch.Tensor, buf: _Buffer, device):
        lib = C.lib()
        if rows == 0:
            return
        ws = buf.get(lib.mosaic_moe_expert_rows_workspace_bytes(ctypes.byref(dims_local), rows), device)
        b = bank.c_struct()
        C.check(lib.mosaic_moe_expert_rows(ctypes.byref(dims_local), rows, ctypes.c_void_p(x_ptr), ldx,
                                           ctypes.c_void_p(ids_ptr), ctypes.c_void_p(w_ptr), stride, default_id,
                                           ctypes.byref(b), ops._ptr(out), ops._ptr(ws), ws.numel(), ops._stream()),
                "mosaic_moe_expert_rows")

    def expert_rows(self, dims_local: C.MoEDims, bank: ExpertBank, recv: torch.Tensor, out: torch.Tensor):
        """Partials of received send rows (uint8 [R, row bytes]) into out [R, H]."""
        h = dims_local.hidden
        rb = C.ep_row_bytes(h)
        base = recv.data_ptr()
        self._rows(dims_local, bank, recv.shape[0], base, rb // 2, base + 2 * h, base + 2 * h + 4, rb // 4, 0, out,
                   self._ws_rows, recv.device)

    def shared_rows(self, dims_local: C.MoEDims, bank: ExpertBank, x: torch.Tensor, out: torch.Tensor):
        """Shared-expert partials of the local tokens x [T, H] into out [T, H]."""
        self._rows(dims_local, bank, x.shape[0], x.data_ptr(), x.shape[1], None, None, 1, dims_local.n_experts, out,
                   self._ws_shared, x.device)

    def combine(self, dims: C.MoEDims, partials: torch.Tensor, ws: torch.Tensor, y: torch.Tensor):
        C.check(C.lib().mosaic_ep_combine(ctypes.byref(dims), ops._ptr(partials), ops._ptr(ws), ops._ptr(y),
                                          ops._stream()), "mosaic_ep_combine")

    def read_error(self, ws: torch.Tensor) -> int:
        return ops.read_error(ws)


class PeerExchange:
    """Exchange regions of every rank of a group, mapped into this process.

    Each rank allocates one region (``mosaic_ep_region_alloc``), the 64-byte
    CUDA IPC handles are shared with ``all_gather_object`` and the peers'
    regions are opened (plain IPC mappings, no multicast).  The regions hold
    the flags, the count matrix, the receive rows and the return partials of
    the device-driven exchange (``mosaic_ep_exchange_rows`` /
    ``mosaic_ep_return_partials``).  With ``row_e4m3`` (FP8 layers) the rows
    are E4M3 rows quantised by the sender (``mosaic_ep_dispatch_exchange``);
    with ``unit_rows`` a token's row goes once to each rank that owns one of
    its experts, listing those experts (E4M3 unit rows).
    Capacity: ``max_tokens`` tokens per rank;
    the receive side is sized for any routing.  ``wait_us`` bounds every
    device-side wait on another rank's flag; a wait that runs out records
    MOSAIC_ERR_TIMEOUT in this rank's region (``error()``) and the kernel returns.
    """

    def __init__(self, *, group=None, max_tokens: int, top_k: int, n_experts: int, hidden: int,
                 partial_f32: bool, wait_us: int = 0, row_e4m3: bool = False, unit_rows: bool = False):
        lib = C.lib()
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if self.world > C.EP_MAX_WORLD:
            raise ValueError(f"peer exchange supports at most {C.EP_MAX_WORLD} ranks")
        e_local = n_experts // self.world
        self.max_tokens = max_tokens
        self.hidden = hidden
        pe = C.EpPeersC()
        pe.world, pe.rank = self.world, self.rank
        # unit rows: one per (token, owning rank), each with min(top_k, e_local) slots
        self.unit_slots = min(top_k, e_local) if unit_rows else 0
        pe.max_recv_rows = self.world * max_tokens * (1 if unit_rows else min(top_k, e_local))
        pe.max_send_rows = max_tokens * top_k
        pe.max_tokens = max_tokens
        pe.hidden = hidden
        pe.partial_f32 = int(bool(partial_f32))
        pe.wait_us = int(wait_us)  # budget of each device-side wait on a peer (0: about 2 s)
        pe.row_e4m3 = int(bool(row_e4m3 or unit_rows))  # E4M3 exchange rows (FP8 layers): half the bytes of bf16
        pe.unit_slots = self.unit_slots
        self.row_e4m3 = bool(row_e4m3 or unit_rows)
        nbytes = lib.mosaic_ep_region_bytes(ctypes.byref(pe))
        if nbytes == 0:
            raise ValueError("invalid peer-exchange geometry")
        region = ctypes.c_void_p()
        handle = (ctypes.c_uint8 * 64)()
        C.check(lib.mosaic_ep_region_alloc(nbytes, ctypes.byref(region), handle), "mosaic_ep_region_alloc")
        self._own = region.value
        self._opened = []
        handles = [bytes(handle)]
        if self.world > 1:
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(handle), group=group)
        for r in range(self.world):
            if r == self.rank:
                pe.regions[r] = self._own
                continue
            h = (ctypes.c_uint8 * 64).from_buffer_copy(handles[r])
            ptr = ctypes.c_void_p()
            C.check(lib.mosaic_ep_region_open(h, ctypes.byref(ptr)), "mosaic_ep_region_open")
            pe.regions[r] = ptr.value
            self._opened.append(ptr.value)
        if self.world > 1:
            dist.barrier(group=group)
        self.peers = pe
        recv, cnt, ret = ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_void_p()
        C.check(lib.mosaic_ep_region_view(ctypes.byref(pe), ctypes.byref(recv), ctypes.byref(cnt), ctypes.byref(ret)),
                "mosaic_ep_region_view")
        self.recv_rows, self.recv_count, self.ret_partials = recv.value, cnt.value, ret.value
        self.max_recv_rows = pe.max_recv_rows

    def error(self) -> int:
        """Device error word of this rank's region (synchronises the stream)."""
        code = ctypes.c_int32(0)
        C.check(C.lib().mosaic_read_error(ctypes.c_void_p(self._own), 1, ctypes.byref(code), ops._stream()),
                "mosaic_read_error")
        return int(code.value)

    def close(self) -> None:
        if self._own is None:
            return
        torch.cuda.synchronize()
        if self.world > 1:
            dist.barrier(group=self.group)  # no rank may still write into a region being released
        lib = C.lib()
        for ptr in self._opened:
            lib.mosaic_ep_region_close(ctypes.c_void_p(ptr))
        lib.mosaic_ep_region_free(ctypes.c_void_p(self._own))
        self._own, self._opened = None, []


class PeerFailure(RuntimeError):
    """A rank of the expert-parallel group left it, or a step's exchange with the
    other ranks failed (a peer that is gone, or the process group's timeout)."""


class PeerHealth:
    """Host-side liveness of the ranks of an expert-parallel group, kept in a
    c10d store the ranks share (``torch.distributed.TCPStore`` or any other
    ``Store``).

    A rank that stops between steps calls ``leave()``.  ``ExpertParallelMoELayer``
    with ``health=`` calls ``check()`` before it launches a step, which raises
    ``PeerFailure`` naming the ranks that left: the others stop before their
    next collective instead of waiting for its timeout.  A rank that stops
    without ``leave()`` is found by the process group's timeout, which ends the
    step's next collective with an error (also raised as ``PeerFailure``).
    """

    def __init__(self, store, world: int, rank: int, *, prefix: str = "mosaic_ep"):
        self.store, self.world, self.rank, self.prefix = store, world, rank, prefix

    def _key(self, r: int) -> str:
        return f"{self.prefix}/left/{r}"

    def leave(self) -> None:
        self.store.set(self._key(self.rank), "1")

    def left(self) -> list:
        return [r for r in range(self.world) if r != self.rank and self.store.check([self._key(r)])]

    def check(self) -> None:
        gone = self.left()
        if gone:
            raise PeerFailure(f"rank(s) {gone} left the expert-parallel group")


class ExpertParallelMoELayer(nn.Module):
    """``MoELayer`` with its routed experts sharded over the ranks of ``group``.

    ``local_bank`` holds this rank's experts (``expert_range``) followed by the
    shared expert when ``cfg.n_shared_experts``; ``shard_bank`` builds it from
    the full reference-layout bank.  ``forward`` takes this rank's tokens and
    returns their layer output; every rank of the group must call it.  With
    ``layer_idx`` the layer is hash-routed (``HashMoELayer``,
    mosaicvm/model/layers.py:376-405): ``.hash_router`` replaces ``.router``
    and ``forward(x, token_ids)`` routes by token id.  With ``health``
    (a ``PeerHealth``) every step first checks that no rank has left.  A failed
    collective of the NCCL / gloo exchange raises ``PeerFailure``.
    """

    def __init__(self, cfg: MoEConfig, local_bank, *, group=None, kernels=None, exchange: str = "nccl",
                 max_tokens: int | None = None, peer_exchange: "PeerExchange | None" = None,
                 layer_idx: int | None = None, health: "PeerHealth | None" = None, unit_rows: bool = True):
        super().__init__()
        self.health = health
        # p2p exchange of an FP8 layer: a row per (token, owning rank) instead of one per assignment
        self.unit_rows = unit_rows
        if exchange not in ("nccl", "p2p"):
            raise ValueError("exchange must be 'nccl' or 'p2p'")
        self.exchange = exchange
        self.max_tokens = max_tokens if peer_exchange is None else peer_exchange.max_tokens
        # layers that run one after the other on a stream may share one exchange
        self._px = peer_exchange
        self._owns_px = peer_exchange is None
        self._side = None
        cfg.validate()
        self.cfg = cfg
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.e_lo, self.e_hi = expert_range(cfg.n_routed_experts, self.world, self.rank)
        self.bank = local_bank
        self.has_shared = cfg.n_shared_experts > 0
        self.router = Router(cfg) if layer_idx is None else None
        self.hash_router = HashRouter(cfg, layer_idx) if layer_idx is not None else None
        self.kernels = kernels if kernels is not None else CudaEPKernels()
        self.last_weights = None
        self.last_idx = None
        self.last_counts = None

    def peer_exchange(self) -> PeerExchange:
        """The peer-memory exchange of this layer (created on first use; every
        rank of the group must reach this point together)."""
        if self._px is None:
            if self.max_tokens is None:
                raise ValueError("exchange='p2p' needs max_tokens")
            self._px = PeerExchange(group=self.group, max_tokens=self.max_tokens,
                                    top_k=max(self.cfg.num_experts_per_tok, self._k()),
                                    n_experts=self.cfg.n_routed_experts,
                                    hidden=self.cfg.hidden_size, partial_f32=self.cfg.act_mode == "bf16",
                                    row_e4m3=self.cfg.act_mode == "fp8",
                                    unit_rows=self.unit_rows and self.cfg.act_mode == "fp8")
        return self._px

    def close(self) -> None:
        if self._px is not None and self._owns_px:
            self._px.close()
        self._px = None

    @classmethod
    def from_layer(cls, layer, *, group=None, kernels=None, exchange: str = "nccl", max_tokens: int | None = None,
                   unit_rows: bool = True):
        """EP layer of this rank from a full single-GPU ``MoELayer`` (same config,
        router weights and experts; the bank keeps its reference-layout copies)."""
        world = dist.get_world_size(group) if dist.is_initialized() else 1
        rank = dist.get_rank(group) if dist.is_initialized() else 0
        b = layer.bank
        local = shard_bank(b.gu_packed, b.gu_scale, b.dn_packed, b.dn_scale, rank=rank, world=world,
                           n_experts=layer.cfg.n_routed_experts, has_shared=b.has_shared)
        hr = getattr(layer, "hash_router", None)
        ep = cls(layer.cfg, local, group=group, kernels=kernels, exchange=exchange, max_tokens=max_tokens,
                 layer_idx=None if hr is None else hr.layer_idx, unit_rows=unit_rows)
        if hr is not None:
            ep.hash_router.weight.data = hr.weight.data
            ep.hash_router.tid2eid = hr.tid2eid
        else:
            ep.router.weight.data = layer.router.weight.data
            ep.router.e_score_correction_bias.data = layer.router.e_score_correction_bias.data
        return ep

    def _k(self) -> int:
        """Experts per token: the config's, or a hash table's width (1 without a table)."""
        hr = self.hash_router
        if hr is None:
            return self.cfg.num_experts_per_tok
        if hr.tid2eid is None:
            return 1
        return 1 if hr.tid2eid.dim() == 1 else int(hr.tid2eid.shape[1])

    def _route(self, xf, token_ids):
        if self.hash_router is not None:
            return self.kernels.route_hash(self.hash_router, xf, token_ids)
        return self.kernels.route(self.router, xf)

    def _dims(self, tokens: int) -> C.MoEDims:
        d = self.cfg.dims(tokens, self.has_shared)
        d.top_k = self._k()
        return d

    def _local_dims(self, tokens: int) -> C.MoEDims:
        d = self._dims(tokens)
        d.n_experts = self.e_hi - self.e_lo
        return d

    def _a2a(self, out, inp, out_splits, in_splits, async_op=False):
        if self.world == 1:  # no process group needed: the exchange is a copy
            out.copy_(inp)
            return None
        try:
            return dist.all_to_all_single(out, inp, output_split_sizes=out_splits, input_split_sizes=in_splits,
                                          group=self.group, async_op=async_op)
        except RuntimeError as e:  # DistBackendError, timeouts
            raise PeerFailure(f"expert-parallel exchange failed on rank {self.rank}: {e}") from e

    def _wait(self, work) -> None:
        if work is None:
            return
        try:
            work.wait()
        except RuntimeError as e:
            raise PeerFailure(f"expert-parallel exchange failed on rank {self.rank}: {e}") from e

    def _forward_p2p(self, xf: torch.Tensor, token_ids=None) -> torch.Tensor:
        """One step with the device-driven peer-memory exchange: no host
        synchronisation, so the step can be captured in a CUDA graph."""
        t, h = xf.shape
        k = self._k()
        px = self.peer_exchange()
        if t > px.max_tokens:
            raise ValueError(f"{t} tokens exceed the exchange capacity {px.max_tokens}")
        if t == 0:
            raise ValueError("exchange='p2p' needs at least one token per rank")
        lib = C.lib()
        kern = self.kernels
        main = torch.cuda.current_stream()
        if self._side is None:
            self._side = torch.cuda.Stream()
        side = self._side
        # fork: the shared expert needs only this step's tokens, and the previous
        # step's combine (which read the same return rows) is before this point
        side.wait_stream(main)
        dl = self._local_dims(t)
        elem = 4 if self.cfg.act_mode == "bf16" else 2
        if self.has_shared:  # overlaps the exchange; writes return rows [t*k, t*k + t)
            with torch.cuda.stream(side):
                out = px.ret_partials + t * k * h * elem
                kern._rows(dl, self.bank, t, xf.data_ptr(), h, None, None, 1, dl.n_experts, _RawOut(out),
                           kern._ws_shared, xf.device)
        w, idx = self._route(xf, token_ids)
        dims = self._dims(t)
        pe = ctypes.byref(px.peers)
        if px.row_e4m3:  # layout, counts, rows quantised straight into the owners' buffers
            ws = kern._ws_dispatch.get(lib.mosaic_moe_workspace_bytes(ctypes.byref(dims)), xf.device)
            C.check(lib.mosaic_ep_dispatch_exchange(ctypes.byref(dims), pe, ops._ptr(xf), ops._ptr(idx), ops._ptr(w),
                                                    ops._ptr(ws), ws.numel(), ops._stream()),
                    "mosaic_ep_dispatch_exchange")
        else:
            send, counts, ws = kern.dispatch(dims, self.world, xf, idx, w)
            C.check(lib.mosaic_ep_exchange_rows(pe, ops._ptr(send), ops._ptr(counts), ops._stream()),
                    "mosaic_ep_exchange_rows")
        # expert pass on the received rows; the down epilogue stores every partial
        # straight into its source's return buffer
        ws_rows = kern._ws_rows.get(lib.mosaic_ep_expert_rows_workspace_bytes(ctypes.byref(dl), pe), xf.device)
        b = self.bank.c_struct()
        C.check(lib.mosaic_ep_expert_rows_return(ctypes.byref(dl), pe, ctypes.byref(b), ops._ptr(ws_rows),
                                                 ws_rows.numel(), ops._stream()), "mosaic_ep_expert_rows_return")
        main.wait_stream(side)  # join: the shared expert's rows are in the return buffer
        y = torch.empty_like(xf)
        C.check(lib.mosaic_ep_combine(ctypes.byref(dims), ctypes.c_void_p(px.ret_partials), ops._ptr(ws), ops._ptr(y),
                                      ops._stream()), "mosaic_ep_combine")
        self.last_weights, self.last_idx, self.last_counts = w, idx, None
        return y

    def forward(self, x: torch.Tensor, token_ids: torch.Tensor | None = None) -> torch.Tensor:
        shape = x.shape
        if token_ids is not None and self.hash_router is None:
            raise ValueError("token_ids are only used by a hash-routed layer")
        if self.health is not None:
            self.health.check()  # before anything is launched
        if self.exchange == "p2p":
            xf = x.reshape(-1, shape[-1]).to(torch.bfloat16).contiguous()
            return self._forward_p2p(xf, token_ids).to(x.dtype).view(shape)
        xf = x.reshape(-1, shape[-1]).to(torch.bfloat16).contiguous()
        t, h = xf.shape
        k = self._k()
        kern = self.kernels
        dims = self._dims(t)
        if t > 0:
            w, idx = self._route(xf, token_ids)
            send, counts, ws = kern.dispatch(dims, self.world, xf, idx, w)
        else:  # no tokens here, but this rank still serves its experts in every exchange
            w = torch.empty(0, k, dtype=torch.float32, device=xf.device)
            idx = torch.empty(0, k, dtype=torch.int64, device=xf.device)
            send = torch.empty(0, C.ep_row_bytes(h), dtype=torch.uint8, device=xf.device)
            counts = torch.zeros(self.world, dtype=torch.int32, device=xf.device)
            ws = None
        # row counts: rows this rank sends to each rank, rows it receives from each
        recv_counts = torch.empty_like(counts)
        self._a2a(recv_counts, counts, None, None)
        sc = counts.tolist()
        rc = recv_counts.tolist()
        n_send, n_recv = sum(sc), sum(rc)
        recv = torch.empty(n_recv, send.shape[1], dtype=torch.uint8, device=xf.device)
        work = self._a2a(recv, send[:n_send], rc, sc, async_op=True)
        pdt = torch.float32 if self.cfg.act_mode == "bf16" else torch.bfloat16
        # rows [0, n_send) come back from the owners, [t*k, t*k + t) are the shared
        # expert's; rows of assignments with invalid ids are never read
        partials = torch.empty(t * k + (t if self.has_shared else 0), h, dtype=pdt, device=xf.device)
        dl = self._local_dims(t)
        if self.has_shared and t > 0:  # overlaps the exchange
            kern.shared_rows(dl, self.bank, xf, partials[t * k:])
        self._wait(work)
        recv_part = torch.empty(n_recv, h, dtype=pdt, device=xf.device)
        kern.expert_rows(dl, self.bank, recv, recv_part)
        self._a2a(partials[:n_send], recv_part, sc, rc)
        y = torch.empty_like(xf)
        if t > 0:
            kern.combine(dims, partials, ws, y)
        self.last_weights, self.last_idx, self.last_counts = w, idx, (sc, rc)
        return y.to(x.dtype).view(shape)
