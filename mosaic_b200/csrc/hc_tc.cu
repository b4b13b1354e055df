// Hyper-connection mixing dot products on the tensor cores (tcgen05 kind::f16).
//
// Reference behaviour: HyperConnections.pre, mosaicvm/model/layers.py:258-267:
// mixes = F.linear(x_flat.float(), fn) scaled by rsqrt(mean(x_flat^2) + eps),
// x_flat = x.flatten(2) [T, hc*D], fn [(2+hc)*hc, hc*D] fp32.  This kernel makes
// the split-K partials of x_flat . fn^T and of sum(x_flat^2) that
// hc_pre_norm_kernel (hc.cu) adds, scales and turns into pre / post / comb.
//
// The same operand scheme as the router logits (router_tc.cu): x is bf16,
// exact as an MMA operand; fn is split into three bf16 parts (hi + mid + lo,
// 3 x 8 significand bits) by hc_split_fn_kernel into [3][32][hc*D] (rows past
// the (2+hc)*hc mixes zero).
//
// Tokens are M (128 per CTA); the three parts side by side are N = 96, so one
// MMA per 16-wide K step gives each token all three parts' dot products in
// TMEM columns [0, 32), [32, 64), [64, 96).  The K slices (64 wide, one ring
// stage each) form groups of four; a group is one accumulation chain of 16
// MMAs (the tensor core's fp32 accumulation error grows with the chain
// length), and the two issuer warps (6, 7) take the groups in turn, each with
// two 96-column TMEM buffers.  Warp 0 loads the slices with TMA (x box 64 x 128
// tokens, the parts box 64 x 96 rows, 128-byte swizzle); warps 2-5 hold one
// token each per lane: they add the token's squares from the staged x tile
// (every slice) and, in group order, each group's 24 mixes as (hi + mid) + lo
// from TMEM, then write the token's partials.
#include "common.cuh"
#include "kernels.h"

namespace mosaic {

namespace {

constexpr int kHtThreads = 256;  // warp 0 TMA, 1 TMEM, 2-5 sums, 6-7 MMA issuers
constexpr int kHtTok = 128;
constexpr int kHtK = 64;
constexpr int kHtN = 32;                         // mixes padded to 32 per part
constexpr int kHtNB = 3 * kHtN;                  // MMA N: the three parts
constexpr int kHtXBytes = kHtTok * 128;          // 16 KB
constexpr int kHtPartBytes = kHtNB * 128;        // 12 KB
constexpr int kHtStageBytes = kHtXBytes + kHtPartBytes;  // 28 KB
constexpr int kHtIssuers = 2;
constexpr int kHtGroup = 4;  // slices per accumulation chain
// Slice j sits in ring stage j % 8 and group j / 4, issuer (j / 4) % 2: stage s
// always feeds issuer s / 4, which thereby waits on every phase of its stages'
// full barriers in order (an issuer that skipped phases could match a parity
// two fills back).
constexpr int kHtStages = kHtGroup * kHtIssuers;
static_assert(kHtStages == 8, "ring of 8 slices: stage s feeds issuer s / 4");
constexpr uint32_t kHtTmemCols = 512;  // 2 issuers x 2 buffers x 96 columns, rounded up
constexpr int kHtRed = 25;  // per token: 24 mixes + the sum of squares (hc.cu's layout)
constexpr int kHtSsq = 24;

struct HtCtrl {
  uint64_t full[kHtStages];
  uint64_t empty[kHtStages];
  uint64_t acc_full[kHtIssuers][2];
  uint64_t acc_empty[kHtIssuers][2];
  uint64_t drain[kHtIssuers];
  uint32_t tmem_base;
  int abort;
};

__device__ __forceinline__ void ht_mma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// kind::f16 instruction descriptor: fp32 D, bf16 A and B (K-major), M = 128, N = 96.
__host__ __device__ __forceinline__ uint32_t ht_idesc() {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(kHtNB >> 3) << 17) |
         (static_cast<uint32_t>(128 >> 4) << 24);
}

__global__ void __launch_bounds__(kHtThreads, 1)
    hc_mix_tc_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_f, int T,
                     int KD, int nmix, float* __restrict__ partial, int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  HtCtrl* ctrl = reinterpret_cast<HtCtrl*>(smem + kHtStages * kHtStageBytes);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t0 = blockIdx.x * kHtTok;
  const int KT = KD / kHtK;
  const int it0 = static_cast<int>(static_cast<long long>(blockIdx.y) * KT / gridDim.y);
  const int it1 = static_cast<int>(static_cast<long long>(blockIdx.y + 1) * KT / gridDim.y);
  const int nit = it1 - it0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kHtStages; ++s) {
      mbar_init(&ctrl->full[s], 1);
      mbar_init(&ctrl->empty[s], 1 + 128);  // the MMA commit + every summing thread
    }
    for (int i = 0; i < kHtIssuers; ++i) {
      for (int b = 0; b < 2; ++b) {
        mbar_init(&ctrl->acc_full[i][b], 1);
        mbar_init(&ctrl->acc_empty[i][b], 128);
      }
      mbar_init(&ctrl->drain[i], 1);
    }
    ctrl->abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmap_x);
    prefetch_tmap(&tmap_f);
  }
  if (warp == 1) {
    tmem_alloc(&ctrl->tmem_base, kHtTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctrl->tmem_base;
  volatile int* abort = &ctrl->abort;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    bool ok = true;
    for (int j = 0; j < nit; ++j) {
      const int s = j % kHtStages;
      const uint32_t ph = static_cast<uint32_t>(j / kHtStages) & 1u;
      if (!mbar_wait(&ctrl->empty[s], ph ^ 1u, abort)) {
        ok = false;
        break;
      }
      if (lane == 0) {
        const int k0 = (it0 + j) * kHtK;
        uint8_t* st = smem + s * kHtStageBytes;
        uint64_t* fb = &ctrl->full[s];
        mbar_arrive_expect_tx(fb, static_cast<uint32_t>(kHtStageBytes));  // whole boxes (rows past T read as 0)
        tma_load_2d(st, &tmap_x, fb, k0, t0);
        tma_load_2d(st + kHtXBytes, &tmap_f, fb, k0, 0);
      }
      __syncwarp();
    }
    if (!ok) {
      if (lane == 0) set_error(err, MOSAIC_ERR_TIMEOUT);
      ctrl->abort = 1;
    }
    if (nit > 0 && lane == 0) {  // no copy in flight at exit
      volatile int never = 0;
      mbar_wait(&ctrl->full[(nit - 1) % kHtStages], static_cast<uint32_t>((nit - 1) / kHtStages) & 1u, &never);
    }
    __syncwarp();
  } else if (warp >= 6) {
    // ------------------------------------------------- MMA issuer i = warp - 6
    const int i = warp - 6;
    bool ok = true, issued = false;
    const uint32_t idesc = ht_idesc();
    for (int g = i, n = 0; ok && g * kHtGroup < nit; g += kHtIssuers, ++n) {
      const int b = n & 1;
      const uint32_t bph = static_cast<uint32_t>(n >> 1) & 1u;
      if (!mbar_wait(&ctrl->acc_empty[i][b], bph ^ 1u, abort)) {
        ok = false;
        break;
      }
      const uint32_t d = tmem + static_cast<uint32_t>((2 * i + b) * kHtNB);
      const int j1 = min((g + 1) * kHtGroup, nit);
      for (int j = g * kHtGroup; j < j1; ++j) {
        const int s = j % kHtStages;
        if (!mbar_wait(&ctrl->full[s], static_cast<uint32_t>(j / kHtStages) & 1u, abort)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t sa = smem_u32(smem + s * kHtStageBytes);
          const uint32_t sb = sa + kHtXBytes;
          const uint32_t first = (j == g * kHtGroup) ? 1u : 0u;
#pragma unroll
          for (uint32_t kb = 0; kb < 4; ++kb)
            ht_mma_bf16(d, desc_sw128(sa + kb * 32), desc_sw128(sb + kb * 32), idesc, (first && kb == 0) ? 0u : 1u);
          tc_commit(&ctrl->empty[s]);
          if (j == j1 - 1) tc_commit(&ctrl->acc_full[i][b]);
          issued = true;
        }
        __syncwarp();
      }
    }
    if (!ok) {
      if (lane == 0) set_error(err, MOSAIC_ERR_TIMEOUT);
      ctrl->abort = 1;
    }
    if (lane == 0 && issued) {  // every MMA done before TMEM is freed
      tc_commit(&ctrl->drain[i]);
      volatile int never = 0;
      mbar_wait(&ctrl->drain[i], 0, &never);
    }
    __syncwarp();
  } else if (warp >= 2) {
    // ------------------------------------- warps 2-5: one token per lane
    const int q = warp & 3;  // TMEM lanes 32q .. 32q+31
    const int row = q * 32 + lane;
    const int t = t0 + row;
    const uint32_t trow = tmem + (static_cast<uint32_t>(q * 32) << 16);
    float acc[kHtSsq];
#pragma unroll
    for (int m = 0; m < kHtSsq; ++m) acc[m] = 0.f;
    float ssq = 0.f;
    bool ok = true;
    for (int j = 0; j < nit; ++j) {
      const int s = j % kHtStages;
      // squares of this token's 64 staged values, in k order (the row's 16-byte
      // chunk c sits at chunk c ^ (row % 8) of the swizzled tile)
      if (!mbar_wait(&ctrl->full[s], static_cast<uint32_t>(j / kHtStages) & 1u, abort)) {
        ok = false;
        break;
      }
      const uint8_t* xr = smem + s * kHtStageBytes + row * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint4 raw = *reinterpret_cast<const uint4*>(xr + ((c ^ (row & 7)) << 4));
        const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          const float2 f = __bfloat1622float2(h2[h]);
          ssq = fmaf(f.x, f.x, ssq);
          ssq = fmaf(f.y, f.y, ssq);
        }
      }
      // the next fill of this stage is a TMA (async proxy) write: order this
      // thread's generic reads of the tile before it
      fence_proxy_async_smem();
      mbar_arrive(&ctrl->empty[s]);
      if (j % kHtGroup != kHtGroup - 1 && j != nit - 1) continue;
      // the group's mixes: issuer (j / 4) % 2, its buffer n & 1 for the issuer's n-th group
      const int g = j / kHtGroup, i = g % kHtIssuers, n = g / kHtIssuers, b = n & 1;
      if (!mbar_wait(&ctrl->acc_full[i][b], static_cast<uint32_t>(n >> 1) & 1u, abort)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t col = trow + static_cast<uint32_t>((2 * i + b) * kHtNB);
      uint32_t r[6][16];
#pragma unroll
      for (int c = 0; c < 6; ++c) tmem_ld16(col + 16u * c, r[c]);
      tmem_ld_wait();
#pragma unroll
      for (int m = 0; m < kHtSsq; ++m) {
        const float hi = __uint_as_float(r[m >> 4][m & 15]);
        const float mid = __uint_as_float(r[2 + (m >> 4)][m & 15]);
        const float lo = __uint_as_float(r[4 + (m >> 4)][m & 15]);
        acc[m] += (hi + mid) + lo;
      }
      tc_fence_before();
      mbar_arrive(&ctrl->acc_empty[i][b]);
    }
    if (!ok) {
      if (lane == 0) set_error(err, MOSAIC_ERR_TIMEOUT);
      ctrl->abort = 1;
    } else if (t < T) {
      float* out = partial + (static_cast<size_t>(blockIdx.y) * T + t) * kHtRed;
#pragma unroll
      for (int m = 0; m < kHtSsq; ++m)
        if (m < nmix) out[m] = acc[m];
      out[kHtSsq] = ssq;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kHtTmemCols);
}

// fn fp32 [nmix][KD] -> parts bf16 [3][32][KD]: hi, mid, lo with hi + mid + lo =
// fn; rows nmix..31 zero.
__global__ void hc_split_fn_kernel(const float* __restrict__ fn, int nmix, int KD, __nv_bfloat16* __restrict__ parts) {
  const size_t n = static_cast<size_t>(kHtN) * KD;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int m = static_cast<int>(i / KD);
    const float v = m < nmix ? fn[i] : 0.f;  // row m of fn starts at m * KD, as row m of a part
    const __nv_bfloat16 hi = __float2bfloat16_rn(v);
    const float r1 = v - __bfloat162float(hi);
    const __nv_bfloat16 mid = __float2bfloat16_rn(r1);
    parts[i] = hi;
    parts[n + i] = mid;
    parts[2 * n + i] = __float2bfloat16_rn(r1 - __bfloat162float(mid));
  }
}

}  // namespace

int hc_mix_tc_splits(int T, int KD, int num_sms) {
  const int tiles = (T + kHtTok - 1) / kHtTok;
  int s = num_sms / tiles;  // one wave of CTAs
  // at most one split per lane of the Sinkhorn kernel's warp: every lane then
  // loads its split's partials in one round
  if (s > 32) s = 32;
  const int kt = KD / kHtK;
  if (s > kt) s = kt;
  return s < 1 ? 1 : s;
}

size_t hc_fn_parts_bytes(int KD) { return 3 * static_cast<size_t>(kHtN) * KD * 2; }

cudaError_t launch_hc_split_fn(const float* fn, int nmix, int KD, void* parts, int num_sms, cudaStream_t stream) {
  const size_t n = static_cast<size_t>(kHtN) * KD;
  size_t blocks = (n + 255) / 256;
  const size_t cap = static_cast<size_t>(num_sms) * 8;
  if (blocks > cap) blocks = cap;
  hc_split_fn_kernel<<<static_cast<int>(blocks), 256, 0, stream>>>(fn, nmix, KD,
                                                                   static_cast<__nv_bfloat16*>(parts));
  return cudaGetLastError();
}

cudaError_t launch_hc_mix_tc(const CUtensorMap& tmap_x, const CUtensorMap& tmap_f, int T, int KD, int nmix,
                             int splits, float* partial, int* err, cudaStream_t stream) {
  if (KD % kHtK || nmix < 1 || nmix > kHtSsq || splits < 1 || splits > KD / kHtK) return cudaErrorInvalidValue;
  const size_t smem = kHtStages * kHtStageBytes + sizeof(HtCtrl) + 1024;
  cudaError_t e =
      cudaFuncSetAttribute(hc_mix_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  dim3 grid((T + kHtTok - 1) / kHtTok, splits);
  hc_mix_tc_kernel<<<grid, kHtThreads, smem, stream>>>(tmap_x, tmap_f, T, KD, nmix, partial, err);
  return cudaGetLastError();
}

}  // namespace mosaic
