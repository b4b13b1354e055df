// Router logits on the tensor cores for large batches (tcgen05 kind::f16).
//
// Reference behaviour: the fp32 logits F.linear(x.float(), W.float()) of
// mosaicvm/model/layers.py:129 (Router.forward) / the vendored Gate's
// linear(x.float(), self.weight.float()), .mosaicvm/source/inference_model.py:570.
//
// x is bf16, so it is exact as an MMA operand.  W is fp32; it is split into
// three bf16 parts, W = hi + mid + lo (hi = bf16(W), mid = bf16(W - hi),
// lo = bf16(W - hi - mid): 3 x 8 significand bits cover fp32's 24), and the
// logits are accumulated in fp32 TMEM as x.hi + x.mid + x.lo.  Every product
// of a bf16 pair is exact in fp32, so the result differs from an fp32 FMA
// chain only in summation order and rounding, like any split-K order.
//
// A CTA takes 128 tokens x 128 experts (one TMEM accumulator of 128 columns)
// over all of K: warp 0 loads 64-wide K slices of x and of the three parts
// with TMA (128-byte swizzle), warp 1 issues 4 x 3 MMAs (K = 16 each) per slice
// into the one accumulator, warps 2-5 read it back and write the logits.
#include "common.cuh"
#include "kernels.h"

namespace mosaic {

namespace {

constexpr int kRtThreads = 192;
constexpr int kRtTok = 128;
constexpr int kRtExp = 128;
constexpr int kRtK = 64;  // bf16 per 128-byte swizzled row
constexpr int kRtStages = 3;
constexpr int kRtTileBytes = 128 * 128;                       // 128 rows x 128 B
constexpr int kRtStageBytes = kRtTileBytes * 4;               // x tile + three W-part tiles
constexpr uint32_t kRtTmemCols = 128;

struct RtCtrl {
  uint64_t full[kRtStages];
  uint64_t empty[kRtStages];
  uint64_t acc_full;
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

__device__ __forceinline__ void tc_mma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Instruction descriptor of kind::f16: fp32 accumulator, bf16 A and B (both
// K-major), M = 128, N = n.
__host__ __device__ __forceinline__ uint32_t idesc_bf16(int n) {
  uint32_t d = 0;
  d |= 1u << 4;                                 // D format: F32
  d |= 1u << 7;                                 // A format: BF16
  d |= 1u << 10;                                // B format: BF16
  d |= static_cast<uint32_t>(n >> 3) << 17;     // N / 8
  d |= static_cast<uint32_t>(128 >> 4) << 24;   // M / 16
  return d;
}

__global__ void __launch_bounds__(kRtThreads, 1)
    router_logits_tc_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                            int T, int H, int E, float* __restrict__ logits, int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  RtCtrl* ctrl = reinterpret_cast<RtCtrl*>(smem + kRtStages * kRtStageBytes);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t0 = blockIdx.x * kRtTok;
  const int e0 = blockIdx.y * kRtExp;
  const int n = min(kRtExp, E - e0);  // MMA N: a multiple of 16 (E is)
  const int KT = H / kRtK;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kRtStages; ++s) {
      mbar_init(&ctrl->full[s], 1);
      mbar_init(&ctrl->empty[s], 1);
    }
    mbar_init(&ctrl->acc_full, 1);
    mbar_init(&ctrl->drain, 1);
    ctrl->abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmap_x);
    prefetch_tmap(&tmap_w);
  }
  if (warp == 1) {
    tmem_alloc(&ctrl->tmem_base, kRtTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctrl->tmem_base;
  volatile int* abort = &ctrl->abort;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    const uint32_t tx = static_cast<uint32_t>(4 * kRtTileBytes);  // whole boxes (rows past the tensor read as 0)
    bool ok = true;
    for (int it = 0; it < KT; ++it) {
      const int s = it % kRtStages;
      const uint32_t ph = static_cast<uint32_t>(it / kRtStages) & 1u;
      if (!mbar_wait(&ctrl->empty[s], ph ^ 1u, abort)) {
        ok = false;
        break;
      }
      if (lane == 0) {
        uint8_t* st = smem + s * kRtStageBytes;
        uint64_t* fb = &ctrl->full[s];
        mbar_arrive_expect_tx(fb, tx);
        tma_load_2d(st, &tmap_x, fb, it * kRtK, t0);
        for (int p = 0; p < 3; ++p) tma_load_2d(st + (1 + p) * kRtTileBytes, &tmap_w, fb, it * kRtK, p * E + e0);
      }
      __syncwarp();
    }
    if (!ok) {
      if (lane == 0) set_error(err, MOSAIC_ERR_TIMEOUT);
      ctrl->abort = 1;
    }
    if (KT > 0 && lane == 0) {  // no copy in flight at exit
      volatile int never = 0;
      mbar_wait(&ctrl->full[(KT - 1) % kRtStages], static_cast<uint32_t>((KT - 1) / kRtStages) & 1u, &never);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ----------------------------------------------------------------- MMA
    bool ok = true, issued = false;
    const uint32_t idesc = idesc_bf16(n);
    for (int it = 0; it < KT; ++it) {
      const int s = it % kRtStages;
      const uint32_t ph = static_cast<uint32_t>(it / kRtStages) & 1u;
      if (!mbar_wait(&ctrl->full[s], ph, abort)) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (lane == 0) {
        const uint32_t sa = smem_u32(smem + s * kRtStageBytes);
#pragma unroll
        for (uint32_t kb = 0; kb < 4; ++kb) {
#pragma unroll
          for (uint32_t p = 0; p < 3; ++p) {
            const uint32_t sb = sa + (1 + p) * kRtTileBytes;
            tc_mma_bf16(tmem, desc_sw128(sa + kb * 32), desc_sw128(sb + kb * 32), idesc,
                        (it == 0 && kb == 0 && p == 0) ? 0u : 1u);
          }
        }
        tc_commit(&ctrl->empty[s]);
        issued = true;
      }
      __syncwarp();
    }
    if (!ok) {
      if (lane == 0) set_error(err, MOSAIC_ERR_TIMEOUT);
      ctrl->abort = 1;
    }
    if (lane == 0) {
      if (ok) tc_commit(&ctrl->acc_full);
      if (issued) {  // every MMA done before TMEM is freed
        tc_commit(&ctrl->drain);
        volatile int never = 0;
        mbar_wait(&ctrl->drain, 0, &never);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lanes 32q .. 32q+31 = tokens t0 + 32q + lane
    if (mbar_wait(&ctrl->acc_full, 0, abort)) {
      tc_fence_after();
      const int t = t0 + q * 32 + lane;
      for (int c0 = 0; c0 < n; c0 += 16) {
        uint32_t r[16];
        tmem_ld16(tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(c0), r);
        tmem_ld_wait();
        if (t < T) {
          float* row = logits + static_cast<size_t>(t) * E + e0 + c0;
#pragma unroll
          for (int j = 0; j < 16; j += 4)
            *reinterpret_cast<float4*>(row + j) = make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]),
                                                              __uint_as_float(r[j + 2]), __uint_as_float(r[j + 3]));
        }
      }
    } else if (lane == 0) {
      set_error(err, MOSAIC_ERR_TIMEOUT);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kRtTmemCols);
}

// W fp32 [E][H] -> parts bf16 [3][E][H]: hi, mid, lo with hi + mid + lo = W.
__global__ void router_split_w_kernel(const float* __restrict__ w, size_t n, __nv_bfloat16* __restrict__ parts) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const float v = w[i];
    const __nv_bfloat16 hi = __float2bfloat16_rn(v);
    const float r1 = v - __bfloat162float(hi);
    const __nv_bfloat16 mid = __float2bfloat16_rn(r1);
    const float r2 = r1 - __bfloat162float(mid);
    parts[i] = hi;
    parts[n + i] = mid;
    parts[2 * n + i] = __float2bfloat16_rn(r2);
  }
}

}  // namespace

size_t router_tc_smem_bytes() { return kRtStages * kRtStageBytes + sizeof(RtCtrl) + 1024; }

cudaError_t launch_router_split_w(const float* w, int E, int H, void* parts, int num_sms, cudaStream_t stream) {
  const size_t n = static_cast<size_t>(E) * H;
  size_t blocks = (n + 255) / 256;
  const size_t cap = static_cast<size_t>(num_sms) * 8;
  if (blocks > cap) blocks = cap;
  router_split_w_kernel<<<static_cast<int>(blocks), 256, 0, stream>>>(w, n, static_cast<__nv_bfloat16*>(parts));
  return cudaGetLastError();
}

cudaError_t launch_router_logits_tc(const CUtensorMap& tmap_x, const CUtensorMap& tmap_w, int T, int H, int E,
                                    float* logits, int* err, cudaStream_t stream) {
  if (H % kRtK || E % 16 || E < 16) return cudaErrorInvalidValue;
  const size_t smem = router_tc_smem_bytes();
  cudaError_t e = cudaFuncSetAttribute(router_logits_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  dim3 grid((T + kRtTok - 1) / kRtTok, (E + kRtExp - 1) / kRtExp);
  router_logits_tc_kernel<<<grid, kRtThreads, smem, stream>>>(tmap_x, tmap_w, T, H, E, logits, err);
  return cudaGetLastError();
}

}  // namespace mosaic
