// Grouped block-scaled expert GEMM for the MoE layer (tcgen05, sm_100a).
//
// One persistent kernel serves both expert projections:
//   mode 0 (gate/up): D_gate = W_gate . X^T and D_up = W_up . X^T for a 128-row
//     block of the intermediate dimension, then the epilogue computes
//     z = SiLU(clamp(gate)) * clamp(up) * route_weight, rounds z to bf16 and
//     re-quantises it (FP8 mode: the reference act_quant per 128; bf16 mode:
//     hi + lo E4M3 with per-32 scales) straight into the down GEMM's input
//     rows and scale-factor chunks;
//   mode 1 (down): D = W_down . Z^T for a 128-row block of the hidden
//     dimension, written as per-assignment partials (fp32 or bf16).
//
// Swap-AB orientation: A = expert weights (E2M1 codes, E8M0 per-32 scales;
// MMA M = 128 weight rows), B = the activation rows of one token tile of one
// expert (E4M3, per-32 scales; MMA N = token rows padded to 16, doubled in
// bf16 mode for the lo plane).  Weights arrive by TMA through the
// 16U4_ALIGN16B type (packed FP4 in HBM, unpacked into the 16-byte-per-16-
// values smem layout kind::mxf8f6f4 reads), activation rows by TMA, and both
// operands' scale factors by bulk copies of pre-laid-out 512-byte chunks
// (weights: mosaic_prepack_scales; activations: written per token tile by the
// quantiser and by this kernel's gate/up epilogue), then smem -> TMEM with
// tcgen05.cp.  Accumulators live in TMEM, double-buffered when N <= 64 so the
// epilogue of one tile overlaps the main loop of the next.
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
constexpr int kMaxStages = 10;
constexpr int kSmemBudget = 225 * 1024;

struct Ctrl {
  uint64_t full[kMaxStages];
  uint64_t empty[kMaxStages];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
  float red[4][16];
};

struct Plan {
  int stage_bytes, off_a1, off_b, off_sfa0, off_sfa1, off_sfb, stages;
};

__host__ __device__ inline Plan make_plan(int mode, int max_n) {
  Plan pl;
  const int na = (mode == 0) ? 2 : 1;
  const int b_bytes = ((max_n * 128 + 1023) / 1024) * 1024;
  pl.off_a1 = 16384;
  pl.off_b = 16384 * na;
  pl.off_sfa0 = pl.off_b + b_bytes;
  pl.off_sfa1 = pl.off_sfa0 + 512;
  pl.off_sfb = pl.off_sfa0 + 512 * na;
  pl.stage_bytes = ((pl.off_sfb + 512 + 1023) / 1024) * 1024;
  int s = (kSmemBudget - static_cast<int>(sizeof(Ctrl)) - 1024) / pl.stage_bytes;
  pl.stages = s > kMaxStages ? kMaxStages : s;
  return pl;
}

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Sum over the C accumulation chains (chain stride acc_w columns) of 16 columns,
// adding the lo-plane columns (lo_off > 0: columns lo_off.. of the same chain).
// Chains and planes are added in a fixed order, so the result is deterministic.
__device__ __forceinline__ void tmem_sum16(uint32_t taddr, int C, uint32_t acc_w, int lo_off, float (&out)[16]) {
#pragma unroll
  for (int j = 0; j < 16; ++j) out[j] = 0.f;
  for (int c = 0; c < C; ++c) {
    uint32_t r[16], r2[16];
    tmem_ld16(taddr + c * acc_w, r);
    if (lo_off) tmem_ld16(taddr + c * acc_w + lo_off, r2);
    tmem_ld_wait();
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      float v = __uint_as_float(r[j]);
      if (lo_off) v += __uint_as_float(r2[j]);
      out[j] += v;
    }
  }
}

// Word index, inside a 512-byte scale chunk, of token row n (< 128).
__device__ __forceinline__ int sf_word(int n) { return (n & 31) * 4 + (n >> 5); }

__global__ void __launch_bounds__(kThreads, 1)
    moe_gemm_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                    const GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const Plan pl = make_plan(p.mode, p.max_n);
  const int S = pl.stages;
  Ctrl* ctrl = reinterpret_cast<Ctrl*>(smem + S * pl.stage_bytes);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const bool gu = (p.mode == 0);
  const int nbuf = p.nbuf;
  const int C = p.chains;
  // TMEM: accumulator of (buffer b, chain c) at column (b*C + c) * acc_w, the up
  // half at +max_n; chain c's scale factors at sf_base + 16c (SFA gate / down,
  // SFA up, SFB at +0, +4, +8).  K-tile kt accumulates into chain kt % C, so
  // consecutive k-tiles are independent MMA chains; the epilogue sums them.
  const uint32_t acc_w = static_cast<uint32_t>((gu ? 2 : 1) * p.max_n);
  const uint32_t up_off = static_cast<uint32_t>(p.max_n);
  const uint32_t sf_base = kTmemCols - 16u * static_cast<uint32_t>(C);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&ctrl->full[s], 1);
      mbar_init(&ctrl->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&ctrl->acc_full[b], 1);
      mbar_init(&ctrl->acc_empty[b], 128);
    }
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
    bool ok = true;
    for (int item = blockIdx.x; ok && item < n_items; item += gridDim.x) {
      const int tile = item / p.n_blocks;
      const int nb = item - tile * p.n_blocks;
      const int e = p.tiles[3 * tile + 0];
      const int row0 = p.tiles[3 * tile + 1];
      const int rows = p.tiles[3 * tile + 2];
      const int rpad = (rows + 15) & ~15;
      const int n = p.hilo ? 2 * rpad : rpad;
      const uint32_t tx = (gu ? 2u : 1u) * (8192u + 512u) + 512u + static_cast<uint32_t>(n) * 128u;
      const uint8_t* wsf0 = p.w_sf + (static_cast<size_t>(e) * p.w_rowtiles + nb) * KT * 512;
      const uint8_t* wsf1 = p.w_sf + (static_cast<size_t>(e) * p.w_rowtiles + p.I / 128 + nb) * KT * 512;
      const uint8_t* xsf = p.x_sft + static_cast<size_t>(tile) * KT * 512;
      const int wt0 = (e * p.w_rowtiles + nb) * KT;               // first weight tile of this row block
      const int wt1 = (e * p.w_rowtiles + p.I / 128 + nb) * KT;   // up rows (gate/up mode)
      for (int kt = 0; kt < KT; ++kt, ++it) {
        const int s = it % S;
        const uint32_t ph = static_cast<uint32_t>(it / S) & 1u;
        if (!mbar_wait(&ctrl->empty[s], ph ^ 1u, abort)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          uint8_t* st = smem + s * pl.stage_bytes;
          uint64_t* fb = &ctrl->full[s];
          mbar_arrive_expect_tx(fb, tx);
          tma_load_3d(st, &tmap_w, fb, 0, 0, wt0 + kt);
          bulk_load(st + pl.off_sfa0, wsf0 + static_cast<size_t>(kt) * 512, 512, fb);
          if (gu) {
            tma_load_3d(st + pl.off_a1, &tmap_w, fb, 0, 0, wt1 + kt);
            bulk_load(st + pl.off_sfa1, wsf1 + static_cast<size_t>(kt) * 512, 512, fb);
          }
          for (int b = 0; b < rpad / 16; ++b) {
            tma_load_2d(st + pl.off_b + b * 2048, &tmap_x, fb, kt * 128, row0 + 16 * b);
            if (p.hilo)
              tma_load_2d(st + pl.off_b + (rpad / 16 + b) * 2048, &tmap_x, fb, kt * 128, p.R_pad + row0 + 16 * b);
          }
          bulk_load(st + pl.off_sfb, xsf + static_cast<size_t>(kt) * 512, 512, fb);
        }
        __syncwarp();
      }
    }
    if (!ok) {
      if (lane == 0) set_error(p.err, MOSAIC_ERR_TIMEOUT);
      ctrl->abort = 1;
    }
    // Wait (bounded) for the last armed stage so no copy is in flight at exit.
    if (it > 0 && lane == 0) {
      const int s = (it - 1) % S;
      volatile int never = 0;
      mbar_wait(&ctrl->full[s], static_cast<uint32_t>((it - 1) / S) & 1u, &never);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ----------------------------------------------------------------- MMA
    int it = 0, li = 0;
    bool issued = false, ok = true;
    for (int item = blockIdx.x; ok && item < n_items; item += gridDim.x, ++li) {
      const int tile = item / p.n_blocks;
      const int rows = p.tiles[3 * tile + 2];
      const int rpad = (rows + 15) & ~15;
      const int n = p.hilo ? 2 * rpad : rpad;
      const int b = li % nbuf;
      const uint32_t aph = static_cast<uint32_t>(li / nbuf) & 1u;
      if (!mbar_wait(&ctrl->acc_empty[b], aph ^ 1u, abort)) {
        ok = false;
        break;
      }
      tc_fence_after();
      for (int kt = 0; kt < KT; ++kt, ++it) {
        const int c = kt % C;
        const uint32_t d_gate = tmem + static_cast<uint32_t>(b * C + c) * acc_w;
        const uint32_t d_up = d_gate + up_off;
        const uint32_t col_sfa0 = tmem + sf_base + 16u * c;
        const uint32_t col_sfa1 = col_sfa0 + 4u;
        const uint32_t col_sfb = col_sfa0 + 8u;
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
          tc_cp_32x128b_x4(col_sfa0, desc_sf(smem_u32(st + pl.off_sfa0)));
          if (gu) tc_cp_32x128b_x4(col_sfa1, desc_sf(smem_u32(st + pl.off_sfa1)));
          tc_cp_32x128b_x4(col_sfb, desc_sf(smem_u32(st + pl.off_sfb)));
#pragma unroll
          for (uint32_t kb = 0; kb < 4; ++kb) {
            const uint32_t idesc = idesc_mxf8f6f4(n, kb);
            const uint64_t bdesc = desc_sw128(bb + kb * 32);
            const uint32_t acc = (kt >= C || kb > 0) ? 1u : 0u;
            const uint32_t sfb = col_sfb | (kb << 30);
            tc_mma_mxf8f6f4(d_gate, desc_sw128(a0 + kb * 32), bdesc, idesc, acc, col_sfa0 | (kb << 30), sfb);
            if (gu) tc_mma_mxf8f6f4(d_up, desc_sw128(a1 + kb * 32), bdesc, idesc, acc, col_sfa1 | (kb << 30), sfb);
          }
          tc_commit(&ctrl->empty[s]);
          issued = true;
        }
        __syncwarp();
      }
      if (!ok) break;
      if (lane == 0) tc_commit(&ctrl->acc_full[b]);
      __syncwarp();
    }
    if (!ok) {
      if (lane == 0) set_error(p.err, MOSAIC_ERR_TIMEOUT);
      ctrl->abort = 1;
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
    int li = 0;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x, ++li) {
      const int tile = item / p.n_blocks;
      const int nb = item - tile * p.n_blocks;
      const int e = p.tiles[3 * tile + 0];
      const int row0 = p.tiles[3 * tile + 1];
      const int rows = p.tiles[3 * tile + 2];
      const int rpad = (rows + 15) & ~15;
      const bool round_mid = p.fp8 || (e == p.shared_expert);
      const int b = li % nbuf;
      const uint32_t aph = static_cast<uint32_t>(li / nbuf) & 1u;
      if (!mbar_wait(&ctrl->acc_full[b], aph, abort)) {
        if (lane == 0) set_error(p.err, MOSAIC_ERR_TIMEOUT);
        ctrl->abort = 1;
        break;
      }
      tc_fence_after();
      const uint32_t c_buf = static_cast<uint32_t>(b * C) * acc_w;
      for (int c0 = 0; c0 < rpad; c0 += 16) {
        if (gu) {
          float gs[16], us[16];
          tmem_sum16(tq + c_buf + c0, C, acc_w, p.hilo ? rpad : 0, gs);
          tmem_sum16(tq + c_buf + up_off + c0, C, acc_w, p.hilo ? rpad : 0, us);
          float zd[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int col = c0 + j;
            float gv = gs[j];
            float uv = us[j];
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
          const int ncol = p.I;
          const int nn = nb * 128 + lrow;
          uint32_t* zsf = p.z_sft + (static_cast<size_t>(tile) * (p.I / 128) + nb) * 128;
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
              const float amax =
                  fmaxf(fmaxf(ctrl->red[0][j], ctrl->red[1][j]), fmaxf(ctrl->red[2][j], ctrl->red[3][j]));
              const int ex = pow2_scale_exp(amax, 1e-4f);
              const float y = fminf(fmaxf(zd[j] * exp2i(-ex), -448.f), 448.f);
              if (col < rows) {
                p.zq[static_cast<size_t>(row0 + col) * ncol + nn] = f32_to_e4m3(y);
                if (lrow == 0) zsf[sf_word(col)] = (static_cast<uint32_t>(ex + 127) & 0xFFu) * 0x01010101u;
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
                p.zq[static_cast<size_t>(r) * ncol + nn] = hb;
                p.zq[(static_cast<size_t>(p.R_pad) + r) * ncol + nn] = lb;
                if (lane == 0) {
                  reinterpret_cast<uint8_t*>(zsf + sf_word(col))[q] = static_cast<uint8_t>(eh + 127);
                  reinterpret_cast<uint8_t*>(zsf + sf_word(rpad + col))[q] = static_cast<uint8_t>(el + 127);
                }
              }
            }
          }
        } else {
          float ds[16];
          tmem_sum16(tq + c_buf + c0, C, acc_w, p.hilo ? rpad : 0, ds);
          const int nn = nb * 128 + lrow;
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int col = c0 + j;
            if (col < rows) {
              float v = ds[j];
              if (round_mid) v = bf16r(v);
              const size_t o = static_cast<size_t>(row0 + col) * p.H + nn;
              if (p.out_f32)
                reinterpret_cast<float*>(p.out)[o] = v;
              else
                reinterpret_cast<__nv_bfloat16*>(p.out)[o] = __float2bfloat16_rn(v);
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&ctrl->acc_empty[b]);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

}  // namespace

size_t gemm_smem_bytes(int mode, int max_n) {
  const Plan pl = make_plan(mode, max_n);
  return static_cast<size_t>(pl.stages) * pl.stage_bytes + sizeof(Ctrl) + 1024;
}

cudaError_t launch_moe_gemm(const CUtensorMap& tmap_w, const CUtensorMap& tmap_x, const GemmParams& p, int grid,
                            cudaStream_t stream) {
  if (p.max_n < 16 || p.max_n > 128 || p.nbuf < 1 || p.nbuf > 2 || p.chains < 1 || p.chains > 4)
    return cudaErrorInvalidValue;
  const int acc_w = (p.mode == 0 ? 2 : 1) * p.max_n;
  if (p.nbuf * p.chains * acc_w > static_cast<int>(kTmemCols) - 16 * p.chains) return cudaErrorInvalidValue;
  if (p.K / 128 < p.chains) return cudaErrorInvalidValue;
  const size_t smem = gemm_smem_bytes(p.mode, p.max_n);
  cudaError_t err = cudaFuncSetAttribute(moe_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
  if (err != cudaSuccess) return err;
  moe_gemm_kernel<<<grid, kThreads, smem, stream>>>(tmap_w, tmap_x, p);
  return cudaGetLastError();
}

}  // namespace mosaic
