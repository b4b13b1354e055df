// Grouped block-scaled expert GEMM for the MoE layer (tcgen05, sm_100a).
//
// One persistent kernel serves both expert projections:
//   mode 0 (gate/up): D_gate = W_gate . X^T and D_up = W_up . X^T for a 128-row
//     block of the intermediate dimension, then the epilogue computes
//     z = SiLU(clamp(gate)) * clamp(up) * route_weight, rounds z to bf16 and
//     re-quantises it (FP8 mode: the reference act_quant per 128; bf16 mode:
//     hi + lo E4M3 with per-32 scales) straight into the down GEMM's input;
//   mode 1 (down): D = W_down . Z^T for a 128-row block of the hidden
//     dimension, written as per-assignment partials (fp32 or bf16).
//
// Swap-AB orientation: A = expert weights (E2M1 codes, E8M0 per-32 scales;
// MMA M = 128 weight rows), B = activation rows of the expert's token tile
// (E4M3, per-32 scales; MMA N = token rows, padded to 16, doubled in bf16
// mode for the lo plane).  Both operands arrive by TMA (weights through the
// 16U4_ALIGN16B type, which unpacks FP4 into the padded smem layout that
// kind::mxf8f6f4 reads), scale factors go smem -> TMEM with tcgen05.cp, and
// the fp32 accumulators live in TMEM.
//
// Warp roles (192 threads): warp 0 = TMA producer, warp 1 = TMEM owner and MMA
// issuer, warps 2..5 = epilogue (warp w reads TMEM lanes 32*(w%4)..+31).
// Reference behaviour: mosaicvm/kernels/qpa_mma.py:337-486 (grouped ordered
// gate/up and down kernels), mosaicvm/kernels/mxint.py:1301-1346 (fused
// SwiGLU / route weight / bf16 / act_quant epilogue).
#include "common.cuh"
#include "kernels.h"

namespace mosaic {

namespace {

constexpr int kThreads = 192;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColGate = 0;
constexpr uint32_t kColUp = 128;
constexpr uint32_t kColSfa0 = 256;
constexpr uint32_t kColSfa1 = 260;
constexpr uint32_t kColSfb = 264;
constexpr int kMaxStages = 8;

struct Ctrl {
  uint64_t full[kMaxStages];
  uint64_t empty[kMaxStages];
  uint64_t acc_full;
  uint64_t acc_empty;
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
  float red[4][16];
};

struct Plan {
  int stage_bytes, off_a1, off_b, off_sfa0, off_sfa1, off_sfb, stages;
};

__host__ __device__ inline Plan make_plan(int mode) {
  Plan pl;
  if (mode == 0) {
    pl.off_a1 = 16384;
    pl.off_b = 32768;
    pl.off_sfa0 = 49152;
    pl.off_sfa1 = 49664;
    pl.off_sfb = 50176;
    pl.stage_bytes = 51200;
    pl.stages = 4;
  } else {
    pl.off_a1 = 0;
    pl.off_b = 16384;
    pl.off_sfa0 = 32768;
    pl.off_sfa1 = 32768;
    pl.off_sfb = 33280;
    pl.stage_bytes = 34816;
    pl.stages = 6;
  }
  return pl;
}

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

__global__ void __launch_bounds__(kThreads, 1)
    moe_gemm_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                    const GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const Plan pl = make_plan(p.mode);
  const int S = pl.stages;
  Ctrl* ctrl = reinterpret_cast<Ctrl*>(smem + S * pl.stage_bytes);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const bool gu = (p.mode == 0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&ctrl->full[s], 1);
      mbar_init(&ctrl->empty[s], 1);
    }
    mbar_init(&ctrl->acc_full, 1);
    mbar_init(&ctrl->acc_empty, 128);
    mbar_init(&ctrl->drain, 1);
    ctrl->abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmap_w);
    prefetch_tmap(&tmap_x);
  }
  if (warp == 1) {
    tmem_alloc(&ctrl->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctrl->tmem_base;
  volatile int* abort = &ctrl->abort;

  int n_tiles = *p.n_tiles;
  if (n_tiles > p.max_tiles) n_tiles = p.max_tiles;
  const int n_items = n_tiles * p.n_blocks;
  const int KT = p.K / 128;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    int it = 0;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
      const int tile = item / p.n_blocks;
      const int nb = item - tile * p.n_blocks;
      const int e = p.tiles[3 * tile + 0];
      const int row0 = p.tiles[3 * tile + 1];
      const int rows = p.tiles[3 * tile + 2];
      const int rpad = (rows + 15) & ~15;
      const int n = p.hilo ? 2 * rpad : rpad;
      bool ok = true;
      for (int kt = 0; kt < KT; ++kt, ++it) {
        const int s = it % S;
        const uint32_t ph = static_cast<uint32_t>(it / S) & 1u;
        if (!mbar_wait(&ctrl->empty[s], ph ^ 1u, abort)) {
          ok = false;
          break;
        }
        uint8_t* st = smem + s * pl.stage_bytes;
        uint32_t* sfb = reinterpret_cast<uint32_t*>(st + pl.off_sfb);
        for (int r = lane; r < 128; r += 32) {
          uint32_t w = 0x7F7F7F7Fu;
          if (r < n) {
            const int plane = (p.hilo && r >= rpad) ? 1 : 0;
            const int row = row0 + r - plane * rpad;
            if (row < p.R) w = p.x_sf[static_cast<size_t>(plane) * p.x_sf_plane + static_cast<size_t>(kt) * p.R_pad + row];
          }
          sfb[(r & 31) * 4 + (r >> 5)] = w;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          const uint32_t tx = (gu ? 2u : 1u) * (8192u + 512u) + static_cast<uint32_t>(n) * 128u;
          mbar_arrive_expect_tx(&ctrl->full[s], tx);
          tma_load_3d(st, &tmap_w, &ctrl->full[s], kt * 128, nb * 128, e);
          const uint8_t* wsf = p.w_sf + (static_cast<size_t>(e) * p.w_rowtiles + nb) * KT * 512 +
                               static_cast<size_t>(kt) * 512;
          bulk_load(st + pl.off_sfa0, wsf, 512, &ctrl->full[s]);
          if (gu) {
            tma_load_3d(st + pl.off_a1, &tmap_w, &ctrl->full[s], kt * 128, p.I + nb * 128, e);
            const uint8_t* wsf1 = p.w_sf +
                                  (static_cast<size_t>(e) * p.w_rowtiles + p.I / 128 + nb) * KT * 512 +
                                  static_cast<size_t>(kt) * 512;
            bulk_load(st + pl.off_sfa1, wsf1, 512, &ctrl->full[s]);
          }
          for (int b = 0; b < rpad / 16; ++b) {
            tma_load_2d(st + pl.off_b + b * 2048, &tmap_x, &ctrl->full[s], kt * 128, row0 + 16 * b);
            if (p.hilo)
              tma_load_2d(st + pl.off_b + (rpad / 16 + b) * 2048, &tmap_x, &ctrl->full[s], kt * 128,
                          p.R_pad + row0 + 16 * b);
          }
        }
        __syncwarp();
      }
      if (!ok) {
        if (lane == 0) set_error(p.err, MOSAIC_ERR_TIMEOUT);
        ctrl->abort = 1;
        break;
      }
    }
    // Wait (bounded) for the last armed stage so no TMA write is in flight at exit.
    if (it > 0 && lane == 0) {
      const int s = (it - 1) % S;
      volatile int never = 0;
      mbar_wait(&ctrl->full[s], static_cast<uint32_t>((it - 1) / S) & 1u, &never);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ----------------------------------------------------------------- MMA
    int it = 0;
    uint32_t acc_ph = 0;
    bool issued = false;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
      const int tile = item / p.n_blocks;
      const int rows = p.tiles[3 * tile + 2];
      const int rpad = (rows + 15) & ~15;
      const int n = p.hilo ? 2 * rpad : rpad;
      bool ok = mbar_wait(&ctrl->acc_empty, acc_ph ^ 1u, abort);
      tc_fence_after();
      for (int kt = 0; ok && kt < KT; ++kt, ++it) {
        const int s = it % S;
        const uint32_t ph = static_cast<uint32_t>(it / S) & 1u;
        if (!mbar_wait(&ctrl->full[s], ph, abort)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          uint8_t* st = smem + s * pl.stage_bytes;
          const uint32_t a0 = smem_u32(st);
          const uint32_t a1 = smem_u32(st + pl.off_a1);
          const uint32_t bb = smem_u32(st + pl.off_b);
          tc_cp_32x128b_x4(tmem + kColSfa0, desc_sf(smem_u32(st + pl.off_sfa0)));
          if (gu) tc_cp_32x128b_x4(tmem + kColSfa1, desc_sf(smem_u32(st + pl.off_sfa1)));
          tc_cp_32x128b_x4(tmem + kColSfb, desc_sf(smem_u32(st + pl.off_sfb)));
#pragma unroll
          for (uint32_t kb = 0; kb < 4; ++kb) {
            const uint32_t idesc = idesc_mxf8f6f4(n, kb);
            const uint64_t bdesc = desc_sw128(bb + kb * 32);
            const uint32_t acc = (kt > 0 || kb > 0) ? 1u : 0u;
            const uint32_t sfb = (tmem + kColSfb) | (kb << 30);
            tc_mma_mxf8f6f4(tmem + kColGate, desc_sw128(a0 + kb * 32), bdesc, idesc, acc,
                            (tmem + kColSfa0) | (kb << 30), sfb);
            if (gu)
              tc_mma_mxf8f6f4(tmem + kColUp, desc_sw128(a1 + kb * 32), bdesc, idesc, acc,
                              (tmem + kColSfa1) | (kb << 30), sfb);
          }
          tc_commit(&ctrl->empty[s]);
          issued = true;
        }
        __syncwarp();
      }
      if (!ok) {
        if (lane == 0) set_error(p.err, MOSAIC_ERR_TIMEOUT);
        ctrl->abort = 1;
        break;
      }
      if (lane == 0) tc_commit(&ctrl->acc_full);
      __syncwarp();
      acc_ph ^= 1u;
    }
    // Drain: every MMA / copy this warp issued has completed before TMEM is freed.
    if (lane == 0 && issued) {
      tc_commit(&ctrl->drain);
      volatile int never = 0;
      mbar_wait(&ctrl->drain, 0, &never);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int lrow = q * 32 + lane;
    const uint32_t tq = tmem + (static_cast<uint32_t>(q * 32) << 16);
    uint32_t acc_ph = 0;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
      const int tile = item / p.n_blocks;
      const int nb = item - tile * p.n_blocks;
      const int e = p.tiles[3 * tile + 0];
      const int row0 = p.tiles[3 * tile + 1];
      const int rows = p.tiles[3 * tile + 2];
      const int rpad = (rows + 15) & ~15;
      const bool round_mid = p.fp8 || (e == p.shared_expert);
      if (!mbar_wait(&ctrl->acc_full, acc_ph, abort)) {
        if (lane == 0) set_error(p.err, MOSAIC_ERR_TIMEOUT);
        ctrl->abort = 1;
        break;
      }
      tc_fence_after();
      for (int c0 = 0; c0 < rpad; c0 += 16) {
        if (gu) {
          uint32_t g[16], u[16], g2[16], u2[16];
          tmem_ld16(tq + kColGate + c0, g);
          tmem_ld16(tq + kColUp + c0, u);
          if (p.hilo) {
            tmem_ld16(tq + kColGate + rpad + c0, g2);
            tmem_ld16(tq + kColUp + rpad + c0, u2);
          }
          tmem_ld_wait();
          float zd[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int col = c0 + j;
            float gv = __uint_as_float(g[j]);
            float uv = __uint_as_float(u[j]);
            if (p.hilo) {
              gv += __uint_as_float(g2[j]);
              uv += __uint_as_float(u2[j]);
            }
            if (round_mid) {
              gv = bf16r(gv);
              uv = bf16r(uv);
            }
            if (p.swiglu_limit > 0.f) {
              gv = fminf(gv, p.swiglu_limit);
              uv = fminf(fmaxf(uv, -p.swiglu_limit), p.swiglu_limit);
            }
            const float w = (col < rows) ? p.row_weight[row0 + col] : 0.f;
            float z = gv / (1.0f + expf(-gv)) * uv;
            z = z * w;
            zd[j] = (col < rows) ? bf16r(z) : 0.f;
          }
          const int ncol = p.I;  // width of the quantised output rows
          const int n = nb * 128 + lrow;
          if (p.fp8) {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const float m = warp_max(fabsf(zd[j]));
              if (lane == 0) ctrl->red[q][j] = m;
            }
            epi_bar();
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int col = c0 + j;
              const float amax = fmaxf(fmaxf(ctrl->red[0][j], ctrl->red[1][j]), fmaxf(ctrl->red[2][j], ctrl->red[3][j]));
              const int ex = pow2_scale_exp(amax, 1e-4f);
              const float y = fminf(fmaxf(zd[j] * exp2i(-ex), -448.f), 448.f);
              if (col < rows) {
                const int r = row0 + col;
                p.zq[static_cast<size_t>(r) * ncol + n] = f32_to_e4m3(y);
                if (lrow == 0) {
                  const uint32_t b = static_cast<uint32_t>(ex + 127) & 0xFFu;
                  p.zsf[static_cast<size_t>(nb) * p.R_pad + r] = b * 0x01010101u;
                }
              }
            }
            epi_bar();
          } else {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int col = c0 + j;
              const float m = warp_max(fabsf(zd[j]));
              int eh = pow2_scale_exp(m, 1e-30f);
              eh = max(-126, min(127, eh));
              const uint8_t hb = f32_to_e4m3(zd[j] * exp2i(-eh));
              const float res = zd[j] - e4m3_to_f32(hb) * exp2i(eh);
              const float m2 = warp_max(fabsf(res));
              int el = pow2_scale_exp(m2, fmaxf(m * 1e-7f, 1e-30f));
              el = max(-126, min(127, el));
              const uint8_t lb = f32_to_e4m3(res * exp2i(-el));
              if (col < rows) {
                const int r = row0 + col;
                p.zq[static_cast<size_t>(r) * ncol + n] = hb;
                p.zq[(static_cast<size_t>(p.R_pad) + r) * ncol + n] = lb;
                if (lane == 0) {
                  uint8_t* w0 = reinterpret_cast<uint8_t*>(p.zsf + static_cast<size_t>(nb) * p.R_pad + r);
                  uint8_t* w1 = reinterpret_cast<uint8_t*>(p.zsf + p.z_sf_plane + static_cast<size_t>(nb) * p.R_pad + r);
                  w0[q] = static_cast<uint8_t>(eh + 127);
                  w1[q] = static_cast<uint8_t>(el + 127);
                }
              }
            }
          }
        } else {
          uint32_t d[16], d2[16];
          tmem_ld16(tq + kColGate + c0, d);
          if (p.hilo) tmem_ld16(tq + kColGate + rpad + c0, d2);
          tmem_ld_wait();
          const int n = nb * 128 + lrow;
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int col = c0 + j;
            if (col < rows) {
              float v = __uint_as_float(d[j]);
              if (p.hilo) v += __uint_as_float(d2[j]);
              if (round_mid) v = bf16r(v);
              const size_t o = static_cast<size_t>(row0 + col) * p.H + n;
              if (p.out_f32)
                reinterpret_cast<float*>(p.out)[o] = v;
              else
                reinterpret_cast<__nv_bfloat16*>(p.out)[o] = __float2bfloat16_rn(v);
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&ctrl->acc_empty);
      acc_ph ^= 1u;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

}  // namespace

size_t gemm_smem_bytes(int mode) {
  const Plan pl = make_plan(mode);
  return static_cast<size_t>(pl.stages) * pl.stage_bytes + sizeof(Ctrl) + 1024;
}

cudaError_t launch_moe_gemm(const CUtensorMap& tmap_w, const CUtensorMap& tmap_x, const GemmParams& p, int grid,
                            cudaStream_t stream) {
  const size_t smem = gemm_smem_bytes(p.mode);
  cudaError_t err = cudaFuncSetAttribute(moe_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
  if (err != cudaSuccess) return err;
  moe_gemm_kernel<<<grid, kThreads, smem, stream>>>(tmap_w, tmap_x, p);
  return cudaGetLastError();
}

}  // namespace mosaic
