"""The reference CPU expert path, timed as the CPU baseline (test / baseline infrastructure).

"Reference CPU expert path" = the router (torch fp32 F.linear + sigmoid +
bias + group-limited top-k, ``oracle.router``), ``act_quant_ref``, the FP4
linear of the reference's AVX-VNNI C kernel (``mosaicvm/bench/vnni_source_kernel.c``,
compiled from the reference's own source into ``oracle/_ref/``) for gate/up
and down of every expert, torch SwiGLU, and the ordered combine.  The bf16
decode config therefore runs with FP8-activation semantics on the CPU (the
VNNI kernel consumes E4M3).

The operand layouts the VNNI kernel expects are restated here from
``mosaicvm/bench/vnni_source.py:38-79``: weights as 2*E2M1 int8 tiled
[N/8][K/4][8][4] plus per-32 int32 weight sums; activations as 512*E4M3 + 2^18
split into three unsigned byte planes tiled [3][M][K/4][8][4].  When the
reference library is not available (no AVX-VNNI on the host, or no reference
checkout when it was built) the plain-C restatement ``fp4_linear_port.c`` runs
the same arithmetic (kind "port").
"""
from __future__ import annotations

import ctypes
import os
import time
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

from .formats import act_quant_ref, decode_e2m1, e4m3_to_f32, e8m0_to_fp32, to_bf16
from .router import route

HERE = Path(__file__).resolve().parent
VNNI_LIB = HERE / "_ref" / "libvnni_source.so"
PORT_LIB = HERE / "libfp4_linear_port.so"


def host_has_avx_vnni() -> bool:
    try:
        return "avx_vnni" in Path("/proc/cpuinfo").read_text()
    except OSError:
        return False


class FP4LinearCPU:
    """y fp32 [M, N] = source-exact FP4 linear of E4M3 rows against an MXFP4 matrix."""

    def __init__(self, kind: str | None = None):
        if kind is None:
            kind = "reference" if (VNNI_LIB.exists() and host_has_avx_vnni()) else "port"
        self.kind = kind
        ptr = lambda dt: np.ctypeslib.ndpointer(dt, flags="C_CONTIGUOUS")  # noqa: E731
        self._prep = None
        if PORT_LIB.exists():
            self._prep = ctypes.CDLL(str(PORT_LIB))
            self._prep.vnni_prepare.argtypes = [ptr(np.uint8), ctypes.c_int, ctypes.c_int, ptr(np.int8), ptr(np.int32)]
            self._prep.vnni_prepare.restype = None
        if kind == "reference":
            self.lib = ctypes.CDLL(str(VNNI_LIB))
            self.lib.vnni_source_gemm.argtypes = [ptr(np.uint8), ptr(np.float32), ptr(np.int8), ptr(np.float32),
                                                  ptr(np.int32), ptr(np.float32)] + [ctypes.c_int] * 3
            self.lib.vnni_source_gemm.restype = None
        elif kind == "port":
            if not PORT_LIB.exists():
                raise RuntimeError(f"{PORT_LIB} missing: run `python oracle/build.py`")
            self.lib = ctypes.CDLL(str(PORT_LIB))
            self.lib.fp4_linear_port.argtypes = [ptr(np.uint8), ptr(np.float32), ptr(np.uint8), ptr(np.float32),
                                                 ptr(np.float32)] + [ctypes.c_int] * 3
            self.lib.fp4_linear_port.restype = None
        else:
            raise ValueError(kind)

    def prepare(self, packed: np.ndarray, scale: np.ndarray):
        packed = np.ascontiguousarray(packed, dtype=np.uint8)
        n, half_k = packed.shape
        k = half_k * 2
        sw = np.ascontiguousarray(e8m0_to_fp32(scale), dtype=np.float32)
        if self.kind == "port":
            return ("port", packed, sw, n, k)
        if self._prep is not None:
            tiled = np.empty((n // 8, k // 4, 8, 4), dtype=np.int8)
            sums = np.empty((n, k // 32), dtype=np.int32)
            self._prep.vnni_prepare(packed, n, k, tiled, sums)
            return ("reference", tiled, sw, sums, n, k)
        qw = np.rint(decode_e2m1(packed) * 2.0).astype(np.int8)
        tiled = np.ascontiguousarray(qw.reshape(n // 8, 8, k // 4, 4).transpose(0, 2, 1, 3))
        sums = np.ascontiguousarray(qw.reshape(n, k // 32, 32).sum(-1, dtype=np.int32))
        return ("reference", tiled, sw, sums, n, k)

    def __call__(self, q: np.ndarray, sa: np.ndarray, prepared) -> np.ndarray:
        q = np.ascontiguousarray(q, dtype=np.uint8)
        sa = np.ascontiguousarray(sa, dtype=np.float32)
        m, k = q.shape
        if prepared[0] == "port":
            _, packed, sw, n, kk = prepared
            y = np.empty((m, n), dtype=np.float32)
            self.lib.fp4_linear_port(q, sa, packed, sw, y, m, n, k)
            return y
        _, tiled, sw, sums, n, kk = prepared
        qa = np.rint(e4m3_to_f32(q).astype(np.float64) * 512.0).astype(np.int32)
        u = qa + (1 << 18)
        planes = np.stack([((u >> sh) & 0xFF).astype(np.uint8) for sh in (0, 8, 16)])
        tiled_a = np.ascontiguousarray(np.broadcast_to(planes.reshape(3, m, k // 4, 1, 4), (3, m, k // 4, 8, 4)))
        y = np.empty((m, n), dtype=np.float32)
        self.lib.vnni_source_gemm(tiled_a, sa, tiled, sw, sums, y, m, n, k)
        return y


class F32LinearCPU:
    """y fp32 [M, N] = x fp32 [M, K] against the dequantised MXFP4 matrix
    (``fp4_linear_f32`` of ``oracle/fp4_linear_port.c``: double accumulation,
    one rounding).  The oracle's bf16-path linear at V3 sizes, where numpy's
    dequantise-then-matmul is too slow for tens of experts."""

    def __init__(self):
        if not PORT_LIB.exists():
            raise RuntimeError(f"{PORT_LIB} missing: run `python oracle/build.py`")
        ptr = lambda dt: np.ctypeslib.ndpointer(dt, flags="C_CONTIGUOUS")  # noqa: E731
        self.lib = ctypes.CDLL(str(PORT_LIB))
        self.lib.fp4_linear_f32.argtypes = [ptr(np.float32), ptr(np.uint8), ptr(np.float32), ptr(np.float32)] + \
            [ctypes.c_int] * 3
        self.lib.fp4_linear_f32.restype = None

    def __call__(self, x: np.ndarray, packed: np.ndarray, scale: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        packed = np.ascontiguousarray(packed, dtype=np.uint8)
        sw = np.ascontiguousarray(e8m0_to_fp32(scale), dtype=np.float32)
        m, k = x.shape
        n = packed.shape[0]
        y = np.empty((m, n), dtype=np.float32)
        self.lib.fp4_linear_f32(x, packed, sw, y, m, n, k)
        return y


def _silu(x):
    return F.silu(torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32))).numpy()


def expert_fp8_cpu(lin: FP4LinearCPU, xq, xs, w, prep_gu, prep_dn, inter: int, limit: float) -> np.ndarray:
    gu = to_bf16(lin(xq, xs, prep_gu))
    gate, up = gu[:, :inter], gu[:, inter:]
    if limit > 0:
        gate = np.minimum(gate, np.float32(limit))
        up = np.clip(up, np.float32(-limit), np.float32(limit))
    z = (_silu(gate) * up * w[:, None]).astype(np.float32)
    zq, zs = act_quant_ref(to_bf16(z))
    return to_bf16(lin(zq, zs, prep_dn))


class LayerCPU:
    """The reference CPU expert path over one whole MoE layer.

    Every expert's operands are prepared once (the reference prepares its
    weights once too, ``vnni_source.prepare_weights``); ``step`` then runs the
    path on a batch of tokens: the router on every token, ``act_quant_ref``,
    each touched expert on its own tokens (gate/up, SwiGLU, route weight,
    re-quantise, down), the shared expert on every token, and the combine in
    ascending expert id, all on the host cores.

    bank: oracle layout with every routed expert (``gu_packed [E, 2I, H/2]``
    ...) and the shared expert (``sh_*``).
    """

    def __init__(self, bank: dict, kind: str | None = None):
        self.lin = FP4LinearCPU(kind)
        self.kind = self.lin.kind
        lin = self.lin
        self.inter = bank["gu_packed"].shape[1] // 2
        self.n_experts = bank["gu_packed"].shape[0]
        self.prep = [(lin.prepare(bank["gu_packed"][e], bank["gu_scale"][e]),
                      lin.prepare(bank["dn_packed"][e], bank["dn_scale"][e])) for e in range(self.n_experts)]
        self.shared = (lin.prepare(bank["sh_gu_packed"], bank["sh_gu_scale"]),
                       lin.prepare(bank["sh_dn_packed"], bank["sh_dn_scale"]))

    def step(self, x, router_w, bias, *, top_k, n_group, topk_group, route_scale, limit: float = 0.0):
        """One layer step on x [T, H] (bf16 values).  Returns (y fp32 [T, H]
        holding bf16 values, seconds, routing (w, idx))."""
        t0 = time.perf_counter()
        xt = torch.as_tensor(x)
        w, idx = route(xt, router_w, bias, top_k=top_k, n_group=n_group, topk_group=topk_group,
                       route_scale=route_scale)
        xn = xt.float().numpy()
        t = xn.shape[0]
        idx_np = idx.numpy()
        w_np = w.numpy().astype(np.float32)
        xq, xs = act_quant_ref(xn)
        partials = np.zeros((t, top_k, xn.shape[1]), dtype=np.float32)
        for e in np.unique(idx_np):
            tok, slot = np.nonzero(idx_np == e)
            pg, pd = self.prep[e]
            partials[tok, slot] = expert_fp8_cpu(self.lin, xq[tok], xs[tok], w_np[tok, slot], pg, pd, self.inter,
                                                 limit)
        order = np.argsort(idx_np, axis=1, kind="stable")
        acc = np.zeros((t, xn.shape[1]), dtype=np.float32)
        for s_ in range(top_k):
            acc = acc + partials[np.arange(t), order[:, s_]]
        shared = expert_fp8_cpu(self.lin, xq, xs, np.ones(t, np.float32), self.shared[0], self.shared[1],
                                self.inter, limit)
        y = to_bf16(shared + to_bf16(acc))
        return y, time.perf_counter() - t0, (w, idx)


def _cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return os.uname().machine
