"""Expert offload: MoE layers whose experts live in pinned host memory and
stream into a device-resident expert cache.

Reference behaviour (paths inside fazin-ahamed/Mosaic):

* ``ExpertLRU`` ``mosaicvm/runtime/loader.py:48-71``: routed experts are loaded
  on demand into an LRU charged against a device byte budget;
* ``_make_streaming_moe_forward`` ``mosaicvm/runtime/streaming_model.py:209-257``:
  route, take the unique selected experts (a host sync), load them, remap the
  ids to the loaded set in ascending order, run the experts.

Here the cache holds experts in the MMA layouts the grouped GEMM reads
(tiled E2M1 codes and 512-byte scale chunks), so a miss is four contiguous
``cudaMemcpyAsync`` from pinned host memory on a copy stream and nothing is
re-laid out per step.  The selected experts get logical ids in ascending
global order (as the reference's remap does), and ``mosaic_moe_routed_slots``
reads logical expert j from cache slot ``expert_slot[j]``: the combine order
and every row's arithmetic are those of the resident layer, so an offloaded
layer's output is bit-identical to the resident one.  The shared expert is a
cache entry like the others.
"""
from __future__ import annotations

import ctypes
from collections import OrderedDict

import torch
from torch import nn

from . import _capi as C
from . import ops
from .moe import ExpertBank, HashRouter, MoEConfig, Router, _Workspace


def _expert_bytes(hidden: int, inter: int):
    """Bytes per expert of (gu_tiled, gu_sf, dn_tiled, dn_sf) in the bank layouts."""
    return (2 * inter * hidden // 2, 2 * inter * (hidden // 128) * 4,
            hidden * inter // 2, hidden * (inter // 128) * 4)


class HostBank:
    """An expert bank's MMA layouts in pinned host memory, one row per expert
    (``[n_bank, bytes]`` per tensor); the shared expert, when present, last."""

    def __init__(self, gu_tiled, gu_sf, dn_tiled, dn_sf, *, hidden: int, inter: int, has_shared: bool):
        self.hidden, self.inter, self.has_shared = hidden, inter, has_shared
        sizes = _expert_bytes(hidden, inter)
        self.parts = []
        for t, nb in zip((gu_tiled, gu_sf, dn_tiled, dn_sf), sizes):
            t = t.reshape(t.shape[0], -1)
            if t.shape[1] != nb:
                raise ValueError(f"expert rows of {t.shape[1]} bytes, expected {nb}")
            self.parts.append(t)
        self.n_bank = self.parts[0].shape[0]

    @classmethod
    def from_bank(cls, bank: ExpertBank) -> "HostBank":
        """Pinned host copy of a device bank's layouts (one device-to-host pass)."""
        n = bank.n_bank
        parts = []
        for t in (bank.gu_tiled, bank.gu_sf, bank.dn_tiled, bank.dn_sf):
            h = torch.empty(n, t.numel() // n, dtype=torch.uint8, pin_memory=True)
            h.copy_(t.reshape(n, -1))
            parts.append(h)
        return cls(*parts, hidden=bank.hidden, inter=bank.inter, has_shared=bank.has_shared)

    def expert(self, e: int):
        return [p[e] for p in self.parts]


class ExpertCache:
    """``capacity`` expert slots on the device in the bank layouts, least recently
    used replaced first.  Keys are any hashable (e.g. (layer, expert))."""

    def __init__(self, hidden: int, inter: int, capacity: int, device="cuda"):
        if capacity < 1:
            raise ValueError("capacity must be >= 1")
        self.hidden, self.inter, self.capacity = hidden, inter, capacity
        self.device = torch.device(device)
        self.parts = [torch.empty(capacity, nb, dtype=torch.uint8, device=self.device)
                      for nb in _expert_bytes(hidden, inter)]
        self.slot_of: OrderedDict = OrderedDict()
        self.copy_stream = torch.cuda.Stream(device=self.device)
        self.hits = self.misses = 0
        self.bytes_copied = 0

    @classmethod
    def for_budget(cls, hidden: int, inter: int, budget_bytes: int, device="cuda") -> "ExpertCache":
        """As many slots as ``budget_bytes`` of HBM holds (the reference sizes its LRU in bytes)."""
        return cls(hidden, inter, max(1, int(budget_bytes) // sum(_expert_bytes(hidden, inter))), device)

    def c_struct(self) -> C.ExpertBankC:
        b = C.ExpertBankC()
        b.gu_tiled, b.gu_sf, b.dn_tiled, b.dn_sf = (p.data_ptr() for p in self.parts)
        return b

    def ensure(self, keys, source) -> list:
        """Slots of ``keys`` (loaded from ``source(key) -> 4 host tensors`` on a miss).

        Copies run on the cache's copy stream after everything already queued on
        the current stream (a replaced slot may still be read by earlier work);
        the current stream then waits for them.
        """
        keys = list(keys)
        if len(set(keys)) > self.capacity:
            raise ValueError(f"{len(set(keys))} experts requested, cache holds {self.capacity}")
        want = set(keys)
        cur = torch.cuda.current_stream(self.device)
        missing = [k for k in dict.fromkeys(keys) if k not in self.slot_of]
        if missing:
            self.copy_stream.wait_stream(cur)
        used = set(self.slot_of.values())
        free = [s for s in range(self.capacity) if s not in used]
        with torch.cuda.stream(self.copy_stream):
            for k in missing:
                if free:
                    slot = free.pop()
                else:  # least recently used entry not needed now
                    victim = next(v for v in self.slot_of if v not in want)
                    slot = self.slot_of.pop(victim)
                for dst, src in zip(self.parts, source(k)):
                    dst[slot].copy_(src, non_blocking=True)
                    self.bytes_copied += src.numel()
                self.slot_of[k] = slot
        if missing:
            cur.wait_stream(self.copy_stream)
        self.misses += len(missing)
        self.hits += len(set(keys)) - len(missing)
        out = []
        for k in keys:
            self.slot_of.move_to_end(k)
            out.append(self.slot_of[k])
        return out


class OffloadedMoELayer(nn.Module):
    """A MoE layer (``MoELayer`` / ``HashMoELayer`` semantics) whose experts come
    through an :class:`ExpertCache` from a :class:`HostBank`.

    ``forward(x[, token_ids])`` routes on the device, reads the selected ids back
    (one host sync, as the reference's streaming forward does), makes sure the
    selected experts and the shared one are cached, and runs the expert path
    through the slot table.  ``layer_key`` keeps the layers sharing a cache apart.
    """

    def __init__(self, cfg: MoEConfig, host_bank: HostBank, cache: ExpertCache, *, layer_key=0,
                 layer_idx: int | None = None):
        super().__init__()
        cfg.validate()
        if (host_bank.hidden, host_bank.inter) != (cfg.hidden_size, cfg.moe_intermediate_size):
            raise ValueError("host bank and config sizes differ")
        if (cache.hidden, cache.inter) != (host_bank.hidden, host_bank.inter):
            raise ValueError("cache and host bank sizes differ")
        self.cfg, self.host, self.cache, self.layer_key = cfg, host_bank, cache, layer_key
        self.has_shared = host_bank.has_shared and cfg.n_shared_experts > 0
        self.router = Router(cfg) if layer_idx is None else None
        self.hash_router = HashRouter(cfg, layer_idx) if layer_idx is not None else None
        self._ws = _Workspace()
        self.last_weights = self.last_idx = None

    def _source(self, key):
        _, e = key
        return self.host.expert(self.host.n_bank - 1 if e == "shared" else e)

    def forward(self, x, token_ids=None):
        shape = x.shape
        xf = x.reshape(-1, shape[-1]).to(torch.bfloat16).contiguous()
        if xf.device.type != "cuda":
            raise ValueError("OffloadedMoELayer.forward requires a CUDA input (no CPU path)")
        w, idx = self.hash_router(xf, token_ids) if self.hash_router is not None else self.router(xf)
        t, k = idx.shape
        uniq = torch.unique(idx)  # ascending, as the reference's idx.unique()
        ids = uniq.tolist()
        keys = [(self.layer_key, e) for e in ids] + ([(self.layer_key, "shared")] if self.has_shared else [])
        slots = self.cache.ensure(keys, self._source)
        n_log = max(len(ids), k)  # logical experts (empty ones never read)
        table = slots[:len(ids)] + [slots[0]] * (n_log - len(ids)) + (slots[-1:] if self.has_shared else [])
        slot_t = torch.tensor(table, dtype=torch.int32).to(xf.device, non_blocking=True)
        idx_local = torch.searchsorted(uniq, idx.reshape(-1)).reshape(t, k).contiguous()
        d = self.cfg.dims(t, self.has_shared)
        d.n_experts, d.top_k, d.n_group, d.topk_group = n_log, k, 1, 1
        ws = self._ws.get(d, xf.device)
        y = torch.empty_like(xf)
        bank = self.cache.c_struct()
        st = C.lib().mosaic_moe_routed_slots(ctypes.byref(d), ops._ptr(xf), ops._ptr(idx_local),
                                             ops._ptr(w.contiguous()), ctypes.byref(bank), ops._ptr(slot_t),
                                             self.cache.capacity, ops._ptr(y), ops._ptr(ws), ws.numel(),
                                             ops._stream())
        C.check(st, "mosaic_moe_routed_slots")
        self.last_weights, self.last_idx = w, idx
        return y.to(x.dtype).view(shape)

    def workspace(self, tokens: int, device):
        """The workspace of the last call's dims (for mosaic_read_error)."""
        return self._ws.buf
