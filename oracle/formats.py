"""MXFP4 / E8M0 / E4M3 number formats, restated on the CPU (test oracle).

Reference behaviour followed (paths inside fazin-ahamed/Mosaic):

* ``mosaicvm/kernels/mxfp4.py:19-23``  locked E2M1 value table.
* ``mosaicvm/kernels/mxfp4.py:32-43``  FLOOR E8M0 block scale
  (``exponent(amax) - 2``, clamped to [-127, 128], NaN -> 255).
* ``mosaicvm/kernels/mxfp4.py:46-82``  fp32 -> E2M1 round-to-nearest-even
  with saturation at 6.0.
* ``mosaicvm/kernels/mxfp4.py:85-88``  low nibble = even K index.
* ``mosaicvm/kernels/fp4_source.py:35-64``  ``pack_mxfp4_nk``: weight [N, K]
  -> packed uint8 [N, K/2] + E8M0 [N, K/32] (scale blocks run along K).
* ``mosaicvm/kernels/fp4_source.py:67-75``  E8M0 byte -> fp32 power of two.
* ``mosaicvm/runtime/fp8.py:19-34``  ``dequant_fp4`` (LUT first, then scale).
* ``mosaicvm/kernels/fp4_source.py:110-129``  ``act_quant_ref``: per 1x128
  block, s = 2^ceil(log2(max(amax, 1e-4) / 448)) computed from the IEEE bits,
  q = e4m3fn(clamp(x / s, +-448)).

The integer paths are numpy; torch (CPU) is used only for the fp32 -> bf16 and
fp32 -> e4m3fn casts, because the reference performs exactly those torch casts.
"""
from __future__ import annotations

import numpy as np
import torch

E2M1_LUT = (
    0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
    -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0,
)
_LUT32 = np.array(E2M1_LUT, dtype=np.float32)
MX_BLOCK = 32
ACT_BLOCK = 128
ACT_FP8_MAX = 448.0


def _as_f32(a) -> np.ndarray:
    if isinstance(a, torch.Tensor):
        a = a.detach().to(torch.float32).cpu().numpy()
    return np.ascontiguousarray(a, dtype=np.float32)


def floor_e8m0(amax: np.ndarray) -> np.ndarray:
    """Biased FLOOR E8M0 exponent of a block maximum (mxfp4.py:32-43)."""
    bits = _as_f32(amax).view(np.int32)
    unbiased = ((bits >> 23) & 0xFF) - 127 - 2
    unbiased = np.clip(unbiased, -127, 128)
    biased = (unbiased + 127).astype(np.int32)
    biased = np.where(np.isnan(_as_f32(amax)), 255, biased)
    return biased.astype(np.uint8)


def f32_to_e2m1(x: np.ndarray) -> np.ndarray:
    """fp32 -> 4-bit E2M1 code, RNE, saturating (mxfp4.py:46-82).

    Magnitudes below 1.0 are rounded to the 0.5 grid by one fp32 addition of
    2^22 (whose ulp is 0.5, so the hardware add performs the RNE step);
    normal magnitudes round the fp32 mantissa to one bit with a tie-to-even
    carry; magnitudes >= 6.0 saturate to code 7.
    """
    x = _as_f32(x)
    bits = x.view(np.uint32)
    sign = (bits >> 28) & 0x8
    mag = np.abs(x)
    sat = mag >= np.float32(6.0)
    den = (~sat) & (mag < np.float32(1.0))
    big = np.float32(2.0 ** 22)
    den_code = ((mag + big).view(np.uint32) - big.view(np.uint32)).astype(np.uint32)
    mbits = mag.view(np.uint32).astype(np.int64)
    odd = (mbits >> 22) & 1
    norm_code = ((mbits + ((1 - 127) << 23) + ((1 << 21) - 1) + odd) >> 22) & 0xF
    code = np.where(sat, 7, np.where(den, den_code, norm_code)).astype(np.uint32)
    return ((code & 0x7) | sign).astype(np.uint8)


def pack_mxfp4_nk(w) -> tuple[np.ndarray, np.ndarray]:
    """w [N, K] (any float) -> (packed uint8 [N, K/2], scale uint8 E8M0 [N, K/32]).

    Follows fp4_source.py:35-64 on the in-tree FLOOR path (the quack packer
    is absent from the reference environment, so this is the path it takes).
    """
    w = _as_f32(w)
    if w.ndim != 2:
        raise ValueError(f"pack_mxfp4_nk expects [N, K], got {w.shape}")
    n, k = w.shape
    if k % MX_BLOCK:
        raise ValueError(f"K={k} must be a multiple of {MX_BLOCK}")
    blk = w.reshape(n, k // MX_BLOCK, MX_BLOCK)
    amax = np.abs(blk).max(axis=-1)
    sb = floor_e8m0(amax)
    sf = (sb.astype(np.uint32) << 23).view(np.float32)
    sf = np.maximum(sf, np.float32(2.0 ** -126))
    codes = f32_to_e2m1((blk / sf[..., None]).astype(np.float32)).reshape(n, k)
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).astype(np.uint8)
    return np.ascontiguousarray(packed), np.ascontiguousarray(sb)


def e8m0_to_fp32(scale) -> np.ndarray:
    """E8M0 bytes -> fp32 powers of two (fp4_source.py:67-75)."""
    s = np.asarray(scale).astype(np.int32)
    e = np.clip(s - 127, -127, 128)
    return ((e + 127).astype(np.uint32) << 23).view(np.float32)


def decode_e2m1(packed) -> np.ndarray:
    """packed [..., K/2] -> fp32 E2M1 values [..., K], unscaled."""
    p = np.asarray(packed, dtype=np.uint8)
    lo = _LUT32[p & 0xF]
    hi = _LUT32[p >> 4]
    return np.stack((lo, hi), axis=-1).reshape(*p.shape[:-1], p.shape[-1] * 2)


def dequant_fp4(packed, scale) -> np.ndarray:
    """packed [N, K/2] + E8M0 [N, K/32] -> fp32 [N, K] (runtime/fp8.py:19-34).

    Every value LUT[code] * 2^(s-127) is exact in fp32 and in bf16, so this
    equals the reference's bf16 ``dequant_fp4`` output widened to fp32.
    """
    vals = decode_e2m1(packed)
    sf = e8m0_to_fp32(scale)
    return vals * np.repeat(sf, MX_BLOCK, axis=-1)


def to_bf16(x) -> np.ndarray:
    """fp32 -> bf16 (RNE, torch cast) -> fp32."""
    t = torch.from_numpy(_as_f32(x))
    return t.to(torch.bfloat16).to(torch.float32).numpy()


def act_quant_ref(x) -> tuple[np.ndarray, np.ndarray]:
    """x [M, K] -> (e4m3fn bytes uint8 [M, K], pow2 scales fp32 [M, K/128]).

    fp4_source.py:110-129: amax per 128 block clamped to >= 1e-4; the scale is
    2^ceil(log2(amax * (1/448))) taken from the IEEE exponent and a non-zero
    mantissa test; q = e4m3fn(clamp(x / s, -448, 448)).
    """
    xf = _as_f32(x)
    m, k = xf.shape
    if k % ACT_BLOCK:
        raise ValueError(f"K={k} must be a multiple of {ACT_BLOCK}")
    blk = xf.reshape(m, k // ACT_BLOCK, ACT_BLOCK)
    a = np.maximum(np.abs(blk).max(axis=-1), np.float32(1e-4))
    v = (a * np.float32(1.0 / ACT_FP8_MAX)).astype(np.float32)
    bits = v.view(np.int32)
    pexp = ((bits >> 23) & 0xFF) - 127 + ((bits & 0x7FFFFF) != 0).astype(np.int32)
    s = ((pexp + 127).astype(np.uint32) << 23).view(np.float32)
    y = np.clip(blk / s[..., None], -ACT_FP8_MAX, ACT_FP8_MAX).astype(np.float32)
    q = torch.from_numpy(y.reshape(m, k)).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    return np.ascontiguousarray(q), np.ascontiguousarray(s)


def e4m3_to_f32(q) -> np.ndarray:
    """e4m3fn bytes -> fp32 (exact)."""
    t = torch.from_numpy(np.ascontiguousarray(q, dtype=np.uint8))
    return t.view(torch.float8_e4m3fn).to(torch.float32).numpy()


def fp4_linear_source(q, sa, packed, scale_w) -> np.ndarray:
    """Source-exact FP4 linear in fp32: [M, K] e4m3 x [N, K] e2m1 -> [M, N].

    Same arithmetic as fp4_source.py:132-156 and bench/vnni_source_kernel.c:
    for each 32-wide K group g in ascending order, the exact dot product of
    the E4M3 and E2M1 values (computed here in int64 on 512*A and 2*W, which
    are integers for every finite code) is rounded once to fp32, scaled by
    1/1024, by the activation scale of its 128-block and by the E8M0 weight
    scale, then added to an fp32 accumulator.
    """
    q = np.asarray(q, dtype=np.uint8)
    m, k = q.shape
    n = packed.shape[0]
    g = k // MX_BLOCK
    qa = np.rint(e4m3_to_f32(q).astype(np.float64) * 512.0).astype(np.int64)
    qw = np.rint(decode_e2m1(packed).astype(np.float64) * 2.0).astype(np.int64)
    qa = qa.reshape(m, g, MX_BLOCK)
    qw = qw.reshape(n, g, MX_BLOCK)
    sw = e8m0_to_fp32(scale_w)  # [N, G]
    sa = np.asarray(sa, dtype=np.float32)
    acc = np.zeros((m, n), dtype=np.float32)
    for gi in range(g):
        dot = qa[:, gi, :] @ qw[:, gi, :].T  # exact int64
        part = dot.astype(np.float32) * np.float32(1.0 / 1024.0)
        part = part * sa[:, gi // 4][:, None]
        part = part * sw[:, gi][None, :]
        acc = acc + part
    return acc
