"""Expert-parallel path on the GPU.

* world 1 (no process group): ExpertParallelMoELayer == MoELayer bit for bit;
* N ranks emulated in one process: every rank's dispatch, the all-to-all as
  slicing, each owner's per-row expert pass, the return exchange and the
  combine — each rank's output equals MoELayer on that rank's tokens bit for
  bit (the router's split-K depends on the token count, so the reference is
  the single-GPU layer on the same tokens);
* dispatch send rows and counts equal the CPU restatement byte for byte;
* on a box with 2+ GPUs, a real 2-rank NCCL run (torchrun) of the same check.
"""
from __future__ import annotations

import os
import subprocess
import sys

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _small_layer(act_mode, seed=3, t=96):
    from mosaic_b200 import MoEConfig, MoELayer
    from mosaic_b200 import synthetic

    cfg = MoEConfig(hidden_size=512, moe_intermediate_size=256, n_routed_experts=32, num_experts_per_tok=4,
                    n_group=4, topk_group=2, routed_scaling_factor=2.5, act_mode=act_mode)
    bank = synthetic.make_bank(512, 256, 32, seed)
    layer = MoELayer(cfg, bank)
    synthetic.make_router(layer, seed)
    x = synthetic.make_tokens(t, 512, seed)
    return layer, x


@pytest.mark.parametrize("act_mode", ["bf16", "fp8"])
def test_ep_world1_bit_identical_to_layer(act_mode):
    from mosaic_b200.ep import ExpertParallelMoELayer

    layer, x = _small_layer(act_mode)
    ep = ExpertParallelMoELayer.from_layer(layer)
    y_ref = layer(x)
    y = ep(x)
    torch.cuda.synchronize()
    assert torch.equal(ep.last_idx, layer.last_idx)
    assert torch.equal(y, y_ref)


def test_ep_world1_v3_decode_bit_identical():
    from mosaic_b200 import synthetic
    from mosaic_b200.ep import ExpertParallelMoELayer

    layer, x = synthetic.make_layer(tokens=64, seed=21, act_mode="bf16", n_experts=64)
    ep = ExpertParallelMoELayer.from_layer(layer)
    assert torch.equal(ep(x), layer(x))


def _emulate(layer, xs, world):
    """Run the EP layer step of `world` ranks in one process; the exchanges are slicing."""
    from mosaic_b200 import _capi as C
    from mosaic_b200.ep import CudaEPKernels, shard_bank

    cfg, b = layer.cfg, layer.bank
    k, h = cfg.num_experts_per_tok, cfg.hidden_size
    kern = [CudaEPKernels() for _ in range(world)]
    banks = [shard_bank(b.gu_packed, b.gu_scale, b.dn_packed, b.dn_scale, rank=r, world=world,
                        n_experts=cfg.n_routed_experts, has_shared=b.has_shared) for r in range(world)]
    dims, sends, counts, wss = [], [], [], []
    for r in range(world):
        d = cfg.dims(xs[r].shape[0], b.has_shared)
        w, idx = layer.router(xs[r])
        s, c, ws = kern[r].dispatch(d, world, xs[r], idx, w)
        dims.append(d), sends.append(s), counts.append(c.cpu().tolist()), wss.append(ws)
    cnt = np.array(counts)  # [src, dest]
    off = np.concatenate([np.zeros((world, 1), dtype=np.int64), np.cumsum(cnt, axis=1)], axis=1)
    pdt = torch.float32 if cfg.act_mode == "bf16" else torch.bfloat16
    parts = [torch.full((xs[r].shape[0] * (k + 1), h), float("nan"), dtype=pdt, device="cuda")
             for r in range(world)]
    for d in range(world):
        recv = torch.cat([sends[r][off[r, d]:off[r, d + 1]] for r in range(world)])
        dl = cfg.dims(1, b.has_shared)
        dl.n_experts = cfg.n_routed_experts // world
        out = torch.full((recv.shape[0], h), float("nan"), dtype=pdt, device="cuda")
        kern[d].expert_rows(dl, banks[d], recv, out)
        pos = 0
        for r in range(world):
            n = int(cnt[r, d])
            parts[r][off[r, d]:off[r, d] + n] = out[pos:pos + n]
            pos += n
    ys = []
    for r in range(world):
        t = xs[r].shape[0]
        dl = cfg.dims(t, b.has_shared)
        dl.n_experts = cfg.n_routed_experts // world
        kern[r].shared_rows(dl, banks[r], xs[r], parts[r][t * k:])
        y = torch.empty_like(xs[r])
        kern[r].combine(dims[r], parts[r], wss[r], y)
        assert kern[r].read_error(wss[r]) == 0
        ys.append(y)
    return ys, cnt


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("act_mode", ["bf16", "fp8"])
def test_ep_emulated_ranks_bit_identical(world, act_mode):
    layer, x = _small_layer(act_mode, seed=5 + world, t=150)
    bounds = np.linspace(0, x.shape[0], world + 1).astype(int)
    xs = [x[bounds[r]:bounds[r + 1]].contiguous() for r in range(world)]
    ys, cnt = _emulate(layer, xs, world)
    torch.cuda.synchronize()
    assert cnt.sum() == x.shape[0] * layer.cfg.num_experts_per_tok
    for r in range(world):
        assert torch.equal(ys[r], layer(xs[r])), f"rank {r}"


def test_ep_emulated_v3_dims_8_ranks():
    """V3 dimensions, 64 experts over 8 emulated ranks (8 per rank), 32 decode tokens each."""
    from mosaic_b200 import synthetic

    layer, x = synthetic.make_layer(tokens=256, seed=31, act_mode="bf16", n_experts=64)
    xs = [x[32 * r:32 * (r + 1)].contiguous() for r in range(8)]
    ys, _ = _emulate(layer, xs, 8)
    for r in range(8):
        assert torch.equal(ys[r], layer(xs[r])), f"rank {r}"


def test_ep_dispatch_rows_match_cpu_restatement():
    from mosaic_b200.ep import CudaEPKernels
    from tests.ep_cpu_kernels import CpuEPKernels

    layer, x = _small_layer("bf16", seed=9, t=77)
    w, idx = layer.router(x)
    d = layer.cfg.dims(x.shape[0], True)
    send, counts, _ = CudaEPKernels().dispatch(d, 4, x, idx, w)
    cs, cc, _ = CpuEPKernels(None, None, layer.cfg, {}).dispatch(d, 4, x.cpu(), idx.cpu(), w.cpu())
    assert torch.equal(counts.cpu(), cc)
    assert torch.equal(send.cpu(), cs)


class _DevBytes:
    """A uint8 view of device memory the C ABI owns (the exchange region)."""

    def __init__(self, ptr: int, n: int):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "|u1", "data": (ptr, False), "version": 3}


@pytest.mark.parametrize("hidden", [512, 768, 7168])
def test_ep_e4m3_rows_equal_act_quant_of_the_send_rows(hidden):
    """mosaic_ep_dispatch_exchange at world 1: the received E4M3 rows are, byte
    for byte, the CPU restatement's send rows (expert order, same tails) with
    the token values replaced by the oracle's act_quant_ref codes and biased
    exponents (zero padding up to 16 bytes)."""
    import ctypes

    from mosaic_b200 import _capi as C
    from mosaic_b200 import MoEConfig, ops, synthetic
    from mosaic_b200.ep import PeerExchange
    from oracle.formats import act_quant_ref
    from tests.ep_cpu_kernels import CpuEPKernels

    t, k, e = 77, 4, 32
    cfg = MoEConfig(hidden_size=hidden, moe_intermediate_size=256, n_routed_experts=e, num_experts_per_tok=k,
                    n_group=1, topk_group=1, act_mode="fp8")
    x = synthetic.make_tokens(t, hidden, 31) * 3.0
    g = torch.Generator().manual_seed(5)
    idx = torch.stack([torch.randperm(e, generator=g)[:k] for _ in range(t)]).cuda()
    w = torch.rand(t, k, generator=g).cuda()
    d = cfg.dims(t, True)
    px = PeerExchange(max_tokens=t, top_k=k, n_experts=e, hidden=hidden, partial_f32=False, row_e4m3=True)
    try:
        lib = C.lib()
        ws = torch.empty(lib.mosaic_moe_workspace_bytes(ctypes.byref(d)), dtype=torch.uint8, device="cuda")
        C.check(lib.mosaic_ep_dispatch_exchange(ctypes.byref(d), ctypes.byref(px.peers), ops._ptr(x), ops._ptr(idx),
                                                ops._ptr(w), ops._ptr(ws), ws.numel(), ops._stream()),
                "mosaic_ep_dispatch_exchange")
        torch.cuda.synchronize()
        assert px.error() == 0
        rb = C.ep_row_bytes_e4m3(hidden)
        got = torch.as_tensor(_DevBytes(px.recv_rows, t * k * rb), device="cuda").cpu().numpy().reshape(t * k, rb)
    finally:
        px.close()
    send, _, meta = CpuEPKernels(None, None, cfg, {}).dispatch(d, 1, x.cpu(), idx.cpu(), w.cpu())
    send = send.numpy()
    q, sc = act_quant_ref(x.cpu().float().numpy())
    tok = np.repeat(np.arange(t), k)[meta["order"]]
    kt = hidden // 128
    pad = (kt + 15) & ~15
    want = np.zeros((t * k, rb), dtype=np.uint8)
    want[:, :hidden] = q[tok]
    want[:, hidden:hidden + kt] = (np.log2(sc[tok]).astype(np.int32) + 127).astype(np.uint8)
    want[:, hidden + pad:] = send[:, 2 * hidden:]
    assert np.array_equal(got, want)


def test_expert_rows_rejects_bad_ids_on_device():
    from mosaic_b200 import _capi as C
    from mosaic_b200.ep import CudaEPKernels, shard_bank

    layer, x = _small_layer("bf16", seed=4, t=8)
    b = layer.bank
    bank = shard_bank(b.gu_packed, b.gu_scale, b.dn_packed, b.dn_scale, rank=0, world=2, n_experts=32,
                      has_shared=True)
    rows = torch.zeros(8, C.ep_row_bytes(512), dtype=torch.uint8, device="cuda")
    tail = rows[:, 1024:].view(torch.int32)
    tail[:, 0] = torch.arange(8, device="cuda") * 5  # ids 0..35: 17+ are out of range for 16 + shared
    tail[:, 1] = torch.ones(8, device="cuda").view(torch.int32)
    dl = layer.cfg.dims(1, True)
    dl.n_experts = 16
    kern = CudaEPKernels()
    out = torch.empty(8, 512, device="cuda")
    kern.expert_rows(dl, bank, rows, out)
    assert kern.read_error(kern._ws_rows.t) == C.MOSAIC_ERR_RANGE


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_two_gpus_nccl():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=ROOT)
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29533",
           os.path.join(ROOT, "tests", "ep_nccl_check.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, cwd=ROOT)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert r.stdout.count("EP_OK") == 2, r.stdout[-2000:]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_two_gpus_rank_departure_seen_before_the_next_step():
    """One of two GPU ranks leaves between steps (PeerHealth.leave) and exits;
    the other's next step raises PeerFailure before launching anything."""
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=ROOT)
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29534",
           os.path.join(ROOT, "tests", "ep_failure_gpu_check.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, cwd=ROOT)
    out = r.stdout + r.stderr
    assert r.returncode == 0, out[-3000:]
    assert out.count("STEP1_OK") == 2 and "rank 1 LEFT" in out, out[-3000:]
    assert "rank 0 PEER_FAILURE_SEEN" in out, out[-3000:]


@pytest.mark.parametrize("act_mode,unit_rows", [("bf16", False), ("fp8", False), ("fp8", True)])
def test_ep_p2p_world1_bit_identical_and_graph_capturable(act_mode, unit_rows):
    """The device-driven exchange path (own region only at world 1): eager
    steps and CUDA-graph replays equal MoELayer bit for bit, no device error.
    With unit rows every token goes once to the one rank with all k of its
    experts in its slots."""
    from mosaic_b200.ep import ExpertParallelMoELayer

    layer, x = _small_layer(act_mode, seed=13, t=64)
    ep = ExpertParallelMoELayer.from_layer(layer, exchange="p2p", max_tokens=64, unit_rows=unit_rows)
    try:
        y_ref = layer(x)
        for _ in range(3):  # several steps: epochs advance, buffers are reused
            y = ep(x)
            torch.cuda.synchronize()
            assert torch.equal(y, y_ref)
        assert ep.peer_exchange().error() == 0
        xs = x.clone()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            ys = ep(xs)
        x2 = x.flip(0).contiguous()
        xs.copy_(x2)
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        assert torch.equal(ys, layer(x2))
        assert ep.peer_exchange().error() == 0
        del g
    finally:
        ep.close()


@pytest.mark.parametrize("exchange", ["nccl", "p2p"])
def test_ep_world1_hash_routed_bit_identical(exchange):
    """A hash-routed EP layer (table of 3 columns, token ids given) equals the
    single-GPU HashMoELayer bit for bit, on both exchanges."""
    from mosaic_b200 import HashMoELayer, MoEConfig
    from mosaic_b200 import synthetic
    from mosaic_b200.ep import ExpertParallelMoELayer

    cfg = MoEConfig(hidden_size=512, moe_intermediate_size=256, n_routed_experts=32, num_experts_per_tok=4,
                    n_group=1, topk_group=1, routed_scaling_factor=1.5, act_mode="bf16", scoring_func="sqrtsoftplus")
    layer = HashMoELayer(cfg, 5, synthetic.make_bank(512, 256, 32, 7))
    g = torch.Generator().manual_seed(7)
    layer.hash_router.weight.data = (torch.randn(32, 512, generator=g) / 512 ** 0.5).cuda()
    layer.hash_router.tid2eid = torch.randint(0, 32, (1000, 3), generator=g, dtype=torch.int32)
    x = synthetic.make_tokens(48, 512, 7)
    tok = torch.randint(0, 5000, (48,), generator=g).cuda()
    ep = ExpertParallelMoELayer.from_layer(layer, exchange=exchange, max_tokens=48)
    try:
        y_ref = layer(x, tok)
        y = ep(x, tok)
        torch.cuda.synchronize()
        assert torch.equal(ep.last_idx, layer.last_idx) and ep.last_idx.shape == (48, 3)
        assert torch.equal(y, y_ref)
    finally:
        ep.close()
