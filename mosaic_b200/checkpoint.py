"""Checkpoint loader: safetensors shards with MXFP4 experts -> resident MoE layers.

Reference contract (paths inside fazin-ahamed/Mosaic):

* tensor names and formats, ``mosaicvm/runtime/streaming_model.py:30-100``
  (``validate_exact_v4_tensors``) and ``:150-205``: per layer ``i`` the routed
  experts ``layers.i.ffn.experts.<e>.w{1,3,2}.weight`` (packed E2M1, uint8 or
  int8 ``[N, K/2]``, low nibble first) with ``.scale`` (E8M0 ``[N, K/32]``),
  w1 = gate ``[I, H]``, w3 = up ``[I, H]``, w2 = down ``[H, I]``; the router
  ``ffn.gate.weight`` ``[E, H]``, ``ffn.gate.bias`` ``[E]`` on routed layers,
  ``ffn.gate.tid2eid`` ``[V, k]`` on the first ``num_hash_layers`` layers
  (which have no bias); the shared expert ``ffn.shared_experts.w{1,3,2}``;
* shard lookup, ``mosaicvm/runtime/loader.py:20-45`` (``ShardIndex``):
  ``model.safetensors.index.json`` (``weight_map``) or one ``model.safetensors``;
* config keys and their aliases, ``mosaicvm/model/config.py:121-128``.

The reference keeps routed experts on the host and dequantises the selected
ones to bf16 every step.  Here every expert of a layer is copied once, in its
packed MXFP4 form, into HBM (a V4 layer's 256 experts are ~3.2 GB, so all 43
layers fit one B200) through a double-buffered pinned staging pipeline, and
re-laid out on the device for the MMA.  The safetensors header is parsed here
(8-byte little-endian length, JSON header, raw little-endian data) and the
data is read through ``numpy.memmap``, so no tensor is materialised twice on
the host.
"""
from __future__ import annotations

import json
import struct
from dataclasses import dataclass, fields
from pathlib import Path

import numpy as np
import torch

from .moe import ExactContractError, ExpertBank, HashMoELayer, MoEConfig, MoELayer, exact_target

# safetensors dtype -> (numpy dtype of the raw container, bytes per element)
_ST_DTYPES = {
    "U8": np.uint8, "I8": np.int8, "F8_E8M0": np.uint8, "F8_E4M3": np.uint8, "F8_E5M2": np.uint8,
    "BF16": np.uint16, "F16": np.float16, "F32": np.float32, "F64": np.float64,
    "I16": np.int16, "I32": np.int32, "I64": np.int64, "U16": np.uint16, "U32": np.uint32, "U64": np.uint64,
    "BOOL": np.bool_,
}


class ShardIndex:
    """Maps tensor name -> (shard file, dtype, shape, byte range) (loader.py:20-45)."""

    def __init__(self, root: str | Path):
        self.root = Path(root)
        index_path = self.root / "model.safetensors.index.json"
        self.shards: dict[str, str] = {}
        if index_path.exists():
            self.shards = dict(json.loads(index_path.read_text())["weight_map"])
        elif (self.root / "model.safetensors").exists():
            self.shards = {k: "model.safetensors" for k in self._header("model.safetensors")}
        else:
            raise FileNotFoundError(f"no safetensors under {self.root}")
        self._headers: dict[str, dict] = {}
        self._maps: dict[str, np.memmap] = {}

    def _header(self, shard: str) -> dict:
        with open(self.root / shard, "rb") as f:
            (n,) = struct.unpack("<Q", f.read(8))
            if n > 100 << 20:
                raise ValueError(f"{shard}: implausible safetensors header of {n} bytes")
            head = json.loads(f.read(n))
        head.pop("__metadata__", None)
        base = 8 + n
        return {k: (v["dtype"], tuple(v["shape"]), base + v["data_offsets"][0], base + v["data_offsets"][1])
                for k, v in head.items()}

    def __contains__(self, name: str) -> bool:
        return name in self.shards

    def keys(self):
        return list(self.shards)

    def meta(self, name: str):
        """(safetensors dtype string, shape) of a tensor."""
        shard = self.shards[name]
        if shard not in self._headers:
            self._headers[shard] = self._header(shard)
        dt, shape, _, _ = self._headers[shard][name]
        return dt, shape

    def array(self, name: str) -> np.ndarray:
        """The tensor's raw container as a read-only numpy view of the file (no copy)."""
        shard = self.shards[name]
        dt, shape = self.meta(name)
        _, _, begin, end = self._headers[shard][name]
        if shard not in self._maps:
            self._maps[shard] = np.memmap(self.root / shard, dtype=np.uint8, mode="r")
        npdt = np.dtype(_ST_DTYPES[dt])
        raw = self._maps[shard][begin:end]
        if raw.size != int(np.prod(shape, dtype=np.int64)) * npdt.itemsize:
            raise ValueError(f"{name}: byte range does not match dtype {dt} and shape {shape}")
        return raw.view(npdt).reshape(shape)

    def tensor(self, name: str) -> torch.Tensor:
        """CPU tensor of a tensor's values: BF16 as bfloat16, F8_E4M3 as float8_e4m3fn,
        F8_E8M0 and packed FP4 as their raw bytes (copied out of the file)."""
        dt, _ = self.meta(name)
        a = np.array(self.array(name))
        t = torch.from_numpy(a)
        if dt == "BF16":
            return t.view(torch.bfloat16)
        if dt == "F8_E4M3":
            return t.view(torch.float8_e4m3fn)
        return t


# config.json keys of the MoE fields, both spellings (config.py:121-128 plus the
# inference config's names for the group limit and sizes)
_CONFIG_KEYS = {
    "hidden_size": ("hidden_size", "dim"),
    "moe_intermediate_size": ("moe_intermediate_size", "moe_inter_dim"),
    "n_routed_experts": ("n_routed_experts",),
    "num_experts_per_tok": ("num_experts_per_tok", "n_activated_experts"),
    "n_group": ("n_group", "n_expert_groups"),
    "topk_group": ("topk_group", "n_limited_groups"),
    "routed_scaling_factor": ("routed_scaling_factor", "route_scale"),
    "scoring_func": ("scoring_func", "score_func"),
    "norm_topk_prob": ("norm_topk_prob",),
    "swiglu_limit": ("swiglu_limit",),
    "n_shared_experts": ("n_shared_experts",),
}


def moe_config_from_checkpoint(root: str | Path, act_mode: str = "bf16"):
    """(MoEConfig, num_hash_layers, raw config dict) from ``config.json``.

    Missing keys take the reference V4Config defaults (config.py:26-55) where
    MoEConfig has none of its own: sqrtsoftplus scores, scale 1.5, no groups.
    """
    raw = json.loads((Path(root) / "config.json").read_text())
    v4_defaults = {"hidden_size": 4096, "moe_intermediate_size": 2048, "n_routed_experts": 256,
                   "num_experts_per_tok": 6, "n_group": 1, "topk_group": 1, "routed_scaling_factor": 1.5,
                   "scoring_func": "sqrtsoftplus", "norm_topk_prob": True, "swiglu_limit": 10.0,
                   "n_shared_experts": 1}
    kw = {}
    for field, names in _CONFIG_KEYS.items():
        val = next((raw[n] for n in names if n in raw), v4_defaults[field])
        kw[field] = val
    kw["n_group"] = kw["n_group"] or 1
    kw["topk_group"] = kw["topk_group"] or kw["n_group"]
    known = {f.name for f in fields(MoEConfig)}
    cfg = MoEConfig(**{k: v for k, v in kw.items() if k in known}, act_mode=act_mode)
    cfg.validate()
    n_hash = int(next((raw[n] for n in ("num_hash_layers", "n_hash_layers") if n in raw), 0))
    return cfg, n_hash, raw


@dataclass(frozen=True)
class TensorRule:
    """One tensor a layer must (or must not) carry on the exact path.

    ``suffix`` is the name after the layer prefix; ``dtypes`` the accepted
    safetensors dtypes (None: any); ``shape`` the required shape (None: any);
    ``forbidden`` marks a tensor whose presence breaks the contract.
    """

    suffix: str
    dtypes: frozenset | None = None
    shape: tuple | None = None
    forbidden: bool = False


_PACKED_E2M1 = frozenset({"U8", "I8"})   # two E2M1 codes per byte, low nibble first
_E8M0 = frozenset({"F8_E8M0"})


def exact_layer_rules(cfg: MoEConfig, hash_layer: bool) -> list[TensorRule]:
    """The tensor table of one MoE layer under the exact MXFP4 contract.

    Every routed expert carries ``w1`` (gate) and ``w3`` (up) as packed E2M1
    ``[I, H/2]`` with E8M0 scales ``[I, H/32]``, and ``w2`` (down) as
    ``[H, I/2]`` with ``[H, I/32]`` scales (mosaicvm/runtime/streaming_model.py:30-100
    states the same formats for expert 0 at the V4 sizes).  A hash-routed
    layer has a ``tid2eid`` table and no score bias; a score-routed layer has
    the bias.
    """
    h, i = cfg.hidden_size, cfg.moe_intermediate_size
    dims = {"w1": (i, h), "w3": (i, h), "w2": (h, i)}
    rules = []
    for e in range(cfg.n_routed_experts):
        for w, (rows, k) in dims.items():
            rules.append(TensorRule(f"ffn.experts.{e}.{w}.weight", _PACKED_E2M1, (rows, k // 2)))
            rules.append(TensorRule(f"ffn.experts.{e}.{w}.scale", _E8M0, (rows, k // 32)))
    if hash_layer:
        rules.append(TensorRule("ffn.gate.tid2eid"))
        rules.append(TensorRule("ffn.gate.bias", forbidden=True))
    else:
        rules.append(TensorRule("ffn.gate.bias"))
    return rules


def check_tensor_rules(index: ShardIndex, prefix: str, rules: list[TensorRule]) -> list[str]:
    """Evaluates ``rules`` against the shard headers; returns one line per broken rule."""
    issues = []
    for r in rules:
        name = prefix + r.suffix
        if r.forbidden:
            if name in index:
                issues.append(f"{name}: present, but a hash-routed layer takes no score bias")
            continue
        if name not in index:
            issues.append(f"{name}: not in the checkpoint")
            continue
        dt, shape = index.meta(name)
        if r.dtypes is not None and dt not in r.dtypes:
            issues.append(f"{name}: dtype {dt}, the exact path needs {' or '.join(sorted(r.dtypes))}")
        if r.shape is not None and tuple(shape) != tuple(r.shape):
            issues.append(f"{name}: shape {tuple(shape)}, the exact path needs {tuple(r.shape)}")
    return issues


def validate_exact_v4_tensors(index: ShardIndex, prefix: str, layer_idx: int, cfg: MoEConfig,
                              num_hash_layers: int) -> None:
    """Checks one layer's tensors against :func:`exact_layer_rules`.

    Stricter than the reference's check (mosaicvm/runtime/streaming_model.py:30-100),
    which inspects expert 0 only: every routed expert of the config is checked,
    at the config's sizes.  Raises ExactContractError listing every broken rule
    (a layer without any routed expert tensor is reported once).
    """
    rules = exact_layer_rules(cfg, hash_layer=layer_idx < num_hash_layers)
    issues = check_tensor_rules(index, prefix, rules)
    expert_rules = [r for r in rules if r.suffix.startswith("ffn.experts.")]
    if expert_rules and all(prefix + r.suffix not in index for r in expert_rules):
        issues = [f"{prefix}ffn.experts.*: no routed expert tensors"] + [
            m for m in issues if not m.startswith(prefix + "ffn.experts.")]
    if issues:
        raise ExactContractError(f"layer {layer_idx} breaks the exact MXFP4 tensor contract: " + "; ".join(issues))


class PinnedStager:
    """Host -> device copies through ``n_buffers`` pinned staging buffers on a copy stream.

    ``copy(dst, src)`` copies a host numpy array (a file mapping, typically) into
    a contiguous device tensor slice: the host fills one pinned buffer while the
    DMA of the previous one runs.  ``finish()`` makes the caller's stream wait
    for every copy issued so far.
    """

    def __init__(self, device, chunk_bytes: int = 64 << 20, n_buffers: int = 2):
        dev = torch.device(device)
        if dev.type == "cuda" and dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        self.device = dev
        self.chunk = int(chunk_bytes)
        self.bufs = [torch.empty(self.chunk, dtype=torch.uint8, pin_memory=True) for _ in range(n_buffers)]
        self.events = [None] * n_buffers
        self.stream = torch.cuda.Stream(device=self.device)
        self.turn = 0
        self.bytes = 0

    def copy(self, dst: torch.Tensor, src: np.ndarray) -> None:
        if not dst.is_contiguous() or dst.device != self.device:
            raise ValueError("PinnedStager.copy needs a contiguous tensor on the stager's device")
        flat_src = np.ascontiguousarray(src).reshape(-1).view(np.uint8)
        flat_dst = dst.view(-1).view(torch.uint8)
        if flat_src.size != flat_dst.numel():
            raise ValueError(f"size mismatch: {flat_src.size} host bytes for {flat_dst.numel()} device bytes")
        off = 0
        while off < flat_src.size:
            n = min(self.chunk, flat_src.size - off)
            i = self.turn
            self.turn = (self.turn + 1) % len(self.bufs)
            if self.events[i] is not None:
                self.events[i].synchronize()  # the DMA that last read this buffer is done
            self.bufs[i][:n].numpy()[:] = flat_src[off:off + n]
            with torch.cuda.stream(self.stream):
                flat_dst[off:off + n].copy_(self.bufs[i][:n], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(self.stream)
            self.events[i] = ev
            off += n
        self.bytes += flat_src.size

    def finish(self) -> None:
        torch.cuda.current_stream(self.device).wait_stream(self.stream)


def _bf16_values(index: ShardIndex, name: str) -> torch.Tensor:
    """fp32 copy of a tensor's values after the reference loader's cast to bf16
    (``StreamingLoader.load_tensor``, loader.py:107-110, casts every non-expert
    tensor to bf16 before it reaches an fp32 parameter)."""
    t = index.tensor(name)
    if index.meta(name)[0] == "F8_E8M0":
        t = t.view(torch.float8_e8m0fnu)
    return t.to(torch.bfloat16).float()


def _router_weight(index: ShardIndex, name: str) -> torch.Tensor:
    """fp32 router weight as the reference loads it (streaming_model.py:103-111
    ``_maybe_dequant``): bf16 values, times the ``.scale`` block grid when one exists
    (rounded to bf16 again)."""
    w = _bf16_values(index, name)
    sname = name.replace(".weight", ".scale")
    if sname in index and sname != name:
        s = _bf16_values(index, sname)
        n, k = w.shape
        if s.dim() == 2 and n % s.shape[0] == 0 and k % s.shape[1] == 0:
            bn, bk = n // s.shape[0], k // s.shape[1]
            w = (w.view(s.shape[0], bn, s.shape[1], bk) * s[:, None, :, None]).reshape(n, k)
        else:
            w = w * s.reshape(-1)[0]
        w = w.to(torch.bfloat16).float()
    return w.contiguous()


def load_moe_layer(root: str | Path | ShardIndex, layer_idx: int, *, cfg: MoEConfig | None = None,
                   num_hash_layers: int | None = None, device="cuda", act_mode: str = "bf16",
                   stager: PinnedStager | None = None, keep_packed: bool = False):
    """One MoE layer of a checkpoint, resident on ``device``.

    Returns a :class:`MoELayer` (routed layers) or :class:`HashMoELayer` (the first
    ``num_hash_layers`` layers, with ``hash_router.tid2eid`` bound).  Under the
    exact target the layer's tensors are checked first
    (:func:`validate_exact_v4_tensors`).  The shared expert must be MXFP4 like
    the routed ones; any other format raises NotImplementedError.
    """
    index = root if isinstance(root, ShardIndex) else ShardIndex(root)
    if cfg is None or num_hash_layers is None:
        c2, nh, _ = moe_config_from_checkpoint(index.root, act_mode)
        cfg = cfg or c2
        num_hash_layers = nh if num_hash_layers is None else num_hash_layers
    prefix = f"layers.{layer_idx}."
    if exact_target():
        validate_exact_v4_tensors(index, prefix, layer_idx, cfg, num_hash_layers)
    h, inter, e = cfg.hidden_size, cfg.moe_intermediate_size, cfg.n_routed_experts
    names = [f"{prefix}ffn.experts.{i}." for i in range(e)]
    missing = [n + "w1.weight" for n in names if n + "w1.weight" not in index]
    if missing:
        raise ValueError(f"layer {layer_idx}: {len(missing)} of {e} experts missing (first: {missing[0]})")
    shared = f"{prefix}ffn.shared_experts."
    has_shared = cfg.n_shared_experts > 0
    if has_shared:
        dt, _ = index.meta(shared + "w1.weight")
        if dt not in _PACKED_E2M1 or shared + "w1.scale" not in index or index.meta(shared + "w1.scale")[0] != "F8_E8M0":
            raise NotImplementedError(f"layer {layer_idx}: shared expert stored as {dt}; the expert GEMM takes "
                                      "MXFP4 (packed E2M1 + E8M0) weights only")
        names.append(shared)
    n = len(names)
    dev = torch.device(device)
    gu_p = torch.empty(n, 2 * inter, h // 2, dtype=torch.uint8, device=dev)
    gu_s = torch.empty(n, 2 * inter, h // 32, dtype=torch.uint8, device=dev)
    dn_p = torch.empty(n, h, inter // 2, dtype=torch.uint8, device=dev)
    dn_s = torch.empty(n, h, inter // 32, dtype=torch.uint8, device=dev)
    st = stager or PinnedStager(dev)
    want = {"w1.weight": (inter, h // 2), "w3.weight": (inter, h // 2), "w2.weight": (h, inter // 2),
            "w1.scale": (inter, h // 32), "w3.scale": (inter, h // 32), "w2.scale": (h, inter // 32)}
    for j, base in enumerate(names):
        for suffix, shape in want.items():
            got = index.meta(base + suffix)[1]
            if tuple(got) != shape:
                raise ValueError(f"{base}{suffix}: expected shape {shape}, got {tuple(got)}")
        st.copy(gu_p[j, :inter], index.array(base + "w1.weight"))
        st.copy(gu_p[j, inter:], index.array(base + "w3.weight"))
        st.copy(gu_s[j, :inter], index.array(base + "w1.scale"))
        st.copy(gu_s[j, inter:], index.array(base + "w3.scale"))
        st.copy(dn_p[j], index.array(base + "w2.weight"))
        st.copy(dn_s[j], index.array(base + "w2.scale"))
    st.finish()
    bank = ExpertBank(gu_p, gu_s, dn_p, dn_s, has_shared=has_shared, keep_packed=keep_packed)
    is_hash = layer_idx < num_hash_layers
    if is_hash:
        layer = HashMoELayer(cfg, layer_idx, bank)
        layer.hash_router.weight.data = _router_weight(index, f"{prefix}ffn.gate.weight").to(dev)
        tid = f"{prefix}ffn.gate.tid2eid"
        if tid in index:
            layer.hash_router.tid2eid = index.tensor(tid).long()
    else:
        layer = MoELayer(cfg, bank)
        layer.router.weight.data = _router_weight(index, f"{prefix}ffn.gate.weight").to(dev)
        bname = f"{prefix}ffn.gate.bias"
        if bname in index:
            layer.router.e_score_correction_bias.data = _bf16_values(index, bname).to(dev)
    return layer


def load_moe_layers(root: str | Path, layers=None, *, device="cuda", act_mode: str = "bf16"):
    """Every MoE layer (or the listed indices) of a checkpoint, sharing one staging pipeline."""
    index = ShardIndex(root)
    cfg, n_hash, raw = moe_config_from_checkpoint(root, act_mode)
    if layers is None:
        n_layers = int(next((raw[k] for k in ("num_hidden_layers", "n_layers") if k in raw), 0))
        layers = range(n_layers)
    st = PinnedStager(device)
    return [load_moe_layer(index, i, cfg=cfg, num_hash_layers=n_hash, device=device, act_mode=act_mode, stager=st)
            for i in layers]
