"""GPU format kernels against the oracle: MXFP4 packer, act_quant, scale re-layout.

Bit-exact bars (integer / byte work): the packer and act_quant must equal the
oracle byte for byte (the oracle itself equals the reference on the golden
vectors, tests/test_oracle_golden.py).
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import formats as fm

pytestmark = pytest.mark.gpu
GOLD = Path(__file__).parent / "golden"


@pytest.fixture(scope="module")
def ops():
    from mosaic_b200 import ops as o

    return o


@pytest.mark.parametrize("shape,std", [((64, 256), 0.02), ((256, 7168), 0.02), ((33, 96), 3.0), ((8, 32), 1e-3)])
def test_pack_mxfp4_bit_exact(ops, shape, std):
    g = torch.Generator().manual_seed(shape[0] * 7 + shape[1])
    w = torch.randn(*shape, generator=g) * std
    p, s = ops.pack_mxfp4_nk(w.cuda())
    pr, sr = fm.pack_mxfp4_nk(w)
    assert np.array_equal(p.cpu().numpy(), pr)
    assert np.array_equal(s.cpu().numpy(), sr)


def test_pack_mxfp4_golden_edges(ops):
    gold = np.load(GOLD / "formats.npz")
    for key in ("pack", "edge"):
        w = torch.from_numpy(gold[key + "_w"]).cuda()
        p, s = ops.pack_mxfp4_nk(w)
        assert np.array_equal(p.cpu().numpy(), gold[key + "_packed"])
        assert np.array_equal(s.cpu().numpy(), gold[key + "_scale"])


def test_pack_all_e2m1_ties(ops):
    # every representable magnitude, midpoints and +-1 ulp around them, both signs, several scales
    grid = np.array([0, .5, 1, 1.5, 2, 3, 4, 6], dtype=np.float32)
    mids = (grid[1:] + grid[:-1]) / 2
    vals = np.concatenate([grid, mids, np.nextafter(mids, 0), np.nextafter(mids, 10), [5.999, 6.0, 7.5]])
    vals = np.concatenate([vals, -vals]).astype(np.float32)
    vals = np.resize(vals, (len(vals) + 31) // 32 * 32)
    rows = [vals * np.float32(2.0 ** e) for e in range(-12, 12)]
    for r in rows:
        r[0] = np.float32(6.0 * 2.0 ** 0)  # pin the block max so the scale is stable
    w = np.stack(rows).astype(np.float32)
    p, s = ops.pack_mxfp4_nk(torch.from_numpy(w).cuda())
    pr, sr = fm.pack_mxfp4_nk(w)
    assert np.array_equal(p.cpu().numpy(), pr) and np.array_equal(s.cpu().numpy(), sr)


def test_act_quant_golden(ops):
    gold = np.load(GOLD / "formats.npz")
    for key in ("act", "actb"):
        x = torch.from_numpy(gold[key + "_x"]).to(torch.bfloat16).cuda()
        q, s = ops.act_quant(x)
        assert np.array_equal(q.view(torch.uint8).cpu().numpy(), gold[key + "_q"])
        assert np.array_equal(s.cpu().numpy().view(np.uint32), gold[key + "_s"].view(np.uint32))


def test_act_quant_every_e4m3_code(ops):
    # all finite E4M3 values, their midpoints and +-1 ulp, scaled so amax hits 448 exactly
    codes = torch.arange(256, dtype=torch.int32).to(torch.uint8).view(torch.float8_e4m3fn).float()
    fin = codes[torch.isfinite(codes)].numpy()
    fin = np.unique(fin)
    mids = (fin[1:] + fin[:-1]) / 2
    vals = np.concatenate([fin, mids, np.nextafter(mids, -1e9), np.nextafter(mids, 1e9)]).astype(np.float32)
    vals = vals[np.abs(vals) <= 448]
    vals = np.resize(vals, (len(vals) + 127) // 128 * 128)
    x = vals.reshape(-1, 128).copy()
    x[:, 0] = 448.0
    xb = torch.from_numpy(x).to(torch.bfloat16)
    q, s = ops.act_quant(xb.cuda())
    qr, sr = fm.act_quant_ref(xb.float().numpy())
    assert np.array_equal(q.view(torch.uint8).cpu().numpy(), qr)
    assert np.array_equal(s.cpu().numpy(), sr)


@pytest.mark.parametrize("m,k", [(1, 128), (37, 7168), (512, 2048)])
def test_act_quant_random(ops, m, k):
    g = torch.Generator().manual_seed(m + k)
    x = (torch.randn(m, k, generator=g) * torch.logspace(-6, 3, m).unsqueeze(1)).to(torch.bfloat16)
    q, s = ops.act_quant(x.cuda())
    qr, sr = fm.act_quant_ref(x.float().numpy())
    assert np.array_equal(q.view(torch.uint8).cpu().numpy(), qr)
    assert np.array_equal(s.cpu().numpy(), sr)


@pytest.mark.parametrize("halves", [1, 2])
def test_prepack_scales_layout(ops, halves):
    g = torch.Generator().manual_seed(3)
    sc = torch.randint(0, 255, (3, 512, 16), generator=g, dtype=torch.uint8)
    out = ops.prepack_scales(sc.cuda(), halves=halves).cpu().numpy()
    nb = 512 // 128 // halves
    ref = np.empty((3, nb, 4, halves, 512), dtype=np.uint8)
    a = sc.numpy()
    for b in range(512):
        r_local = (b >> 4) + 32 * ((b & 15) >> 2)
        kb = b & 3
        for h in range(halves):
            for n in range(nb):
                for kt in range(4):
                    ref[:, n, kt, h, b] = a[:, h * (512 // halves) + n * 128 + r_local, kt * 4 + kb]
    assert np.array_equal(out, ref)


@pytest.mark.parametrize("halves", [1, 2])
def test_repack_weights_layout(ops, halves):
    g = torch.Generator().manual_seed(4)
    p = torch.randint(0, 256, (2, 512, 192), generator=g, dtype=torch.uint8)  # rows 512, K 384
    out = ops.repack_weights(p.cuda(), halves=halves).cpu().numpy()
    a = p.numpy()
    nb = 512 // 128 // halves
    # rows = (half, row block, r); columns = (K-tile, 64 bytes)
    ref = a.reshape(2, halves, nb, 128, 3, 64).transpose(0, 2, 4, 1, 3, 5)
    assert np.array_equal(out, ref)
