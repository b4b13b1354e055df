// Router logits on the tensor cores (tcgen05 kind::f16), every batch size.
//
// Reference behaviour: the fp32 logits F.linear(x.float(), W.float()) of
// mosaicvm/model/layers.py:129 (Router.forward) / the vendored Gate's
// linear(x.float(), self.weight.float()), .mosaicvm/source/inference_model.py:570.
//
// x is bf16, so it is exact as an MMA operand.  W is fp32; it is split into
// three bf16 parts, W = hi + mid + lo (hi = bf16(W), mid = bf16(W - hi),
// lo = bf16(W - hi - mid): 3 x 8 significand bits cover fp32's 24), and the
// logits are x.hi + x.mid + x.lo.  Every product of a bf16 pair is exact in
// fp32, but the tensor core's fp32 accumulation is not rounded like an fp32
// add: measured against fp64 (logit error over ||x o w||, V3 router), chains
// of ~21 MMAs stay near 8e-7 on average, 336 give 1.2e-5 and 1344 give
// 4.7e-5, growing with the chain length, while the FMA kernels give 4-10e-7.
// So every 64-wide K slice starts a fresh chain of 12 MMAs (4 K-steps x 3
// parts) in one of two TMEM buffers, and warps 2-5 add the slices' results in
// fp32 registers in slice order: a split-K order like any other.
//
// A CTA takes 128 tokens x 128 experts over a range of K (grid.z splits K;
// split z writes out[z][T][E], and the top-k pass adds the splits): warp 0
// loads 64-wide K slices with TMA, warp 1 issues each slice's 12 MMAs into
// TMEM buffer (slice & 1), warps 2-5 add each buffer into their token row's
// 128 register accumulators and write the row at the end.  Two ways to get
// the three parts:
//
// - kConvert = false (large batches): a separate kernel splits W once per call
//   into bf16 [3][E][H], and the producer loads the three part tiles with
//   128-byte-swizzled TMA boxes;
// - kConvert = true (small batches, where that pass would cost as much as the
//   logits): the producer loads the fp32 W tile [128 experts][64] unswizzled,
//   and warps 2-5 split it into the three part tiles, writing the 128-byte
//   swizzle that TMA would have written (16-byte chunk c of row r at chunk
//   c ^ (r % 8)), then fence the writes to the async proxy and arrive on the
//   stage's `conv` barrier, which the MMA issuer waits on.
#include "common.cuh"
#include "kernels.h"

namespace mosaic {

namespace {

constexpr int kRtThreads = 192;
constexpr int kRtTok = 128;
constexpr int kRtExp = 128;
constexpr int kRtK = 64;                       // bf16 per 128-byte swizzled row
constexpr int kRtTileBytes = 128 * 128;        // 128 rows x 128 B
constexpr int kRtRawBytes = 128 * kRtK * 4;    // fp32 W tile [128][64], unswizzled
constexpr uint32_t kRtTmemCols = 256;        // two 128-column slice accumulators
constexpr int kRtMaxStages = 3;

template <bool kConvert>
struct RtShape {
  // x tile + three part tiles (+ the raw fp32 tile)
  static constexpr int kStageBytes = 4 * kRtTileBytes + (kConvert ? kRtRawBytes : 0);
  static constexpr int kStages = kConvert ? 2 : 3;
};

struct RtCtrl {
  uint64_t full[kRtMaxStages];
  uint64_t empty[kRtMaxStages];
  uint64_t conv[kRtMaxStages];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
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

// hi + mid + lo split of two fp32 values, packed as bf16 pairs (first value low).
__device__ __forceinline__ void split3(float a, float b, uint32_t& hi, uint32_t& mid, uint32_t& lo) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  const float ra = a - __low2float(h), rb = b - __high2float(h);
  const __nv_bfloat162 m = __floats2bfloat162_rn(ra, rb);
  const __nv_bfloat162 l = __floats2bfloat162_rn(ra - __low2float(m), rb - __high2float(m));
  hi = *reinterpret_cast<const uint32_t*>(&h);
  mid = *reinterpret_cast<const uint32_t*>(&m);
  lo = *reinterpret_cast<const uint32_t*>(&l);
}

template <bool kConvert>
__global__ void __launch_bounds__(kRtThreads, 1)
    router_logits_tc_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                            int T, int H, int E, float* __restrict__ out, int* err) {
  using Shape = RtShape<kConvert>;
  constexpr int kStages = Shape::kStages;
  constexpr int kStageBytes = Shape::kStageBytes;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  RtCtrl* ctrl = reinterpret_cast<RtCtrl*>(smem + kStages * kStageBytes);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t0 = blockIdx.x * kRtTok;
  const int e0 = blockIdx.y * kRtExp;
  const int n = min(kRtExp, E - e0);  // MMA N: a multiple of 16 (E is)
  const int KT = H / kRtK;
  // this split's K slices [it0, it1); the launcher keeps gridDim.z <= KT
  const int it0 = static_cast<int>(static_cast<long long>(blockIdx.z) * KT / gridDim.z);
  const int it1 = static_cast<int>(static_cast<long long>(blockIdx.z + 1) * KT / gridDim.z);
  const int nit = it1 - it0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&ctrl->full[s], 1);
      mbar_init(&ctrl->empty[s], 1);
      mbar_init(&ctrl->conv[s], 128);  // every converter thread arrives
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&ctrl->acc_full[b], 1);
      mbar_init(&ctrl->acc_empty[b], 128);  // every epilogue thread arrives
    }
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
    // whole boxes count (rows past the tensor read as 0)
    const uint32_t tx = static_cast<uint32_t>(kConvert ? kRtTileBytes + kRtRawBytes : 4 * kRtTileBytes);
    bool ok = true;
    for (int j = 0; j < nit; ++j) {
      const int s = j % kStages;
      const uint32_t ph = static_cast<uint32_t>(j / kStages) & 1u;
      if (!mbar_wait(&ctrl->empty[s], ph ^ 1u, abort)) {
        ok = false;
        break;
      }
      if (lane == 0) {
        const int k0 = (it0 + j) * kRtK;
        uint8_t* st = smem + s * kStageBytes;
        uint64_t* fb = &ctrl->full[s];
        mbar_arrive_expect_tx(fb, tx);
        tma_load_2d(st, &tmap_x, fb, k0, t0);
        if (kConvert) {
          tma_load_2d(st + 4 * kRtTileBytes, &tmap_w, fb, k0, e0);
        } else {
          for (int p = 0; p < 3; ++p) tma_load_2d(st + (1 + p) * kRtTileBytes, &tmap_w, fb, k0, p * E + e0);
        }
      }
      __syncwarp();
    }
    if (!ok) {
      if (lane == 0) set_error(err, MOSAIC_ERR_TIMEOUT);
      ctrl->abort = 1;
    }
    if (nit > 0 && lane == 0) {  // no copy in flight at exit
      volatile int never = 0;
      mbar_wait(&ctrl->full[(nit - 1) % kStages], static_cast<uint32_t>((nit - 1) / kStages) & 1u, &never);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ----------------------------------------------------------------- MMA
    bool ok = true, issued = false;
    const uint32_t idesc = idesc_bf16(n);
    for (int j = 0; j < nit; ++j) {
      const int s = j % kStages;
      const uint32_t ph = static_cast<uint32_t>(j / kStages) & 1u;
      const int b = j & 1;
      const uint32_t bph = static_cast<uint32_t>(j >> 1) & 1u;
      if (!mbar_wait(&ctrl->full[s], ph, abort) || (kConvert && !mbar_wait(&ctrl->conv[s], ph, abort)) ||
          !mbar_wait(&ctrl->acc_empty[b], bph ^ 1u, abort)) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (lane == 0) {
        const uint32_t sa = smem_u32(smem + s * kStageBytes);
        const uint32_t d = tmem + static_cast<uint32_t>(b) * kRtExp;
#pragma unroll
        for (uint32_t kb = 0; kb < 4; ++kb) {
#pragma unroll
          for (uint32_t p = 0; p < 3; ++p) {
            const uint32_t sb = sa + (1 + p) * kRtTileBytes;
            tc_mma_bf16(d, desc_sw128(sa + kb * 32), desc_sw128(sb + kb * 32), idesc, (kb | p) ? 1u : 0u);
          }
        }
        tc_commit(&ctrl->empty[s]);
        tc_commit(&ctrl->acc_full[b]);
        issued = true;
      }
      __syncwarp();
    }
    if (!ok) {
      if (lane == 0) set_error(err, MOSAIC_ERR_TIMEOUT);
      ctrl->abort = 1;
    }
    if (lane == 0 && issued) {  // every MMA done before TMEM is freed
      tc_commit(&ctrl->drain);
      volatile int never = 0;
      mbar_wait(&ctrl->drain, 0, &never);
    }
    __syncwarp();
  } else {
    // --------------------------------- warps 2-5: [W split], slice sums, output
    const int q = warp & 3;  // TMEM lanes 32q .. 32q+31 = tokens t0 + 32q + lane
    const int t = t0 + q * 32 + lane;
    const uint32_t trow = tmem + (static_cast<uint32_t>(q * 32) << 16);
    float acc[kRtExp];
#pragma unroll
    for (int i = 0; i < kRtExp; ++i) acc[i] = 0.f;
    // adds slice j's accumulator (buffer j & 1) to acc, then frees the buffer
    auto add_slice = [&](int j) -> bool {
      const int b = j & 1;
      if (!mbar_wait(&ctrl->acc_full[b], static_cast<uint32_t>(j >> 1) & 1u, abort)) return false;
      tc_fence_after();
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t r[4][16];
#pragma unroll
        for (int c = 0; c < 4; ++c)
          if ((h * 4 + c) * 16 < n)
            tmem_ld16(trow + static_cast<uint32_t>(b * kRtExp + (h * 4 + c) * 16), r[c]);
        tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < 4; ++c)
          if ((h * 4 + c) * 16 < n)
#pragma unroll
            for (int i = 0; i < 16; ++i) acc[(h * 4 + c) * 16 + i] += __uint_as_float(r[c][i]);
      }
      tc_fence_before();
      mbar_arrive(&ctrl->acc_empty[b]);
      return true;
    };
    bool ok = true;
    for (int j = 0; j < nit && ok; ++j) {
      if (kConvert) {
        // W split: a warp takes two rows per pass (rows 2(c + 4i) and the next,
        // c = warp - 2), lane l four values of row (l / 16) at 4 (l % 16): a
        // 512-byte read and a 256-byte write per part per pass, both at the
        // minimum wavefront count.  Rows past E were zero-filled by the copy.
        const int s = j % kStages;
        if (!mbar_wait(&ctrl->full[s], static_cast<uint32_t>(j / kStages) & 1u, abort)) {
          ok = false;
          break;
        }
        uint8_t* st = smem + s * kStageBytes;
        const uint8_t* raw = st + 4 * kRtTileBytes;
        const uint32_t col = static_cast<uint32_t>(lane & 15) * 8u;  // byte in the 128-byte bf16 row
#pragma unroll 4
        for (int i = 0; i < 16; ++i) {
          const int r = 2 * ((warp - 2) + 4 * i) + (lane >> 4);
          const float4 v = *reinterpret_cast<const float4*>(raw + r * (kRtK * 4) + (lane & 15) * 16);
          uint2 hi, mid, lo;
          split3(v.x, v.y, hi.x, mid.x, lo.x);
          split3(v.z, v.w, hi.y, mid.y, lo.y);
          const uint32_t off = static_cast<uint32_t>(r) * 128u + ((((col >> 4) ^ static_cast<uint32_t>(r & 7)) << 4) |
                                                                 (col & 15u));
          *reinterpret_cast<uint2*>(st + 1 * kRtTileBytes + off) = hi;
          *reinterpret_cast<uint2*>(st + 2 * kRtTileBytes + off) = mid;
          *reinterpret_cast<uint2*>(st + 3 * kRtTileBytes + off) = lo;
        }
        fence_proxy_async_smem();  // the MMA reads the parts through the async proxy
        mbar_arrive(&ctrl->conv[s]);
      }
      if (j > 0) ok = add_slice(j - 1);  // overlaps the MMAs of slice j
    }
    if (ok && nit > 0) ok = add_slice(nit - 1);
    if (!ok) {
      if (lane == 0) set_error(err, MOSAIC_ERR_TIMEOUT);
      ctrl->abort = 1;
    } else if (t < T) {
      float* orow = out + (static_cast<size_t>(blockIdx.z) * T + t) * E + e0;
#pragma unroll
      for (int c0 = 0; c0 < kRtExp; c0 += 4)
        if (c0 < n) *reinterpret_cast<float4*>(orow + c0) = make_float4(acc[c0], acc[c0 + 1], acc[c0 + 2], acc[c0 + 3]);
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

template <bool kConvert>
size_t rt_smem_bytes() {
  return RtShape<kConvert>::kStages * RtShape<kConvert>::kStageBytes + sizeof(RtCtrl) + 1024;
}

}  // namespace

bool router_tc_applies(int H, int E) { return H % kRtK == 0 && E % 16 == 0 && E >= 16 && E <= 256; }

// In-kernel W split when every CTA takes at most two K slices; otherwise the
// split pass pays for itself (four converter warps cost ~3 us per slice, the
// MMAs ~1 us).
bool router_tc_convert(int T, int H, int E, int num_sms) {
  if (!router_tc_applies(H, E)) return false;
  const int kt = H / kRtK;
  const int s = router_tc_splits(T, H, E, num_sms);
  return (kt + s - 1) / s <= 2;
}

int router_tc_splits(int T, int H, int E, int num_sms) {
  const int tiles = ((T + kRtTok - 1) / kRtTok) * ((E + kRtExp - 1) / kRtExp);
  int s = num_sms / tiles;  // one wave of CTAs
  const int kt = H / kRtK;
  if (s > 64) s = 64;      // bounds the partials the top-k pass adds
  if (s > kt) s = kt;
  return s < 1 ? 1 : s;
}

cudaError_t launch_router_split_w(const float* w, int E, int H, void* parts, int num_sms, cudaStream_t stream) {
  const size_t n = static_cast<size_t>(E) * H;
  size_t blocks = (n + 255) / 256;
  const size_t cap = static_cast<size_t>(num_sms) * 8;
  if (blocks > cap) blocks = cap;
  router_split_w_kernel<<<static_cast<int>(blocks), 256, 0, stream>>>(w, n, static_cast<__nv_bfloat16*>(parts));
  return cudaGetLastError();
}

cudaError_t launch_router_logits_tc(const CUtensorMap& tmap_x, const CUtensorMap& tmap_w, bool convert, int T, int H,
                                    int E, int splits, float* out, int* err, cudaStream_t stream) {
  if (!router_tc_applies(H, E) || splits < 1 || splits > H / kRtK) return cudaErrorInvalidValue;
  dim3 grid((T + kRtTok - 1) / kRtTok, (E + kRtExp - 1) / kRtExp, splits);
  if (convert) {
    const size_t smem = rt_smem_bytes<true>();
    cudaError_t e = cudaFuncSetAttribute(router_logits_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    router_logits_tc_kernel<true><<<grid, kRtThreads, smem, stream>>>(tmap_x, tmap_w, T, H, E, out, err);
  } else {
    const size_t smem = rt_smem_bytes<false>();
    cudaError_t e = cudaFuncSetAttribute(router_logits_tc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    router_logits_tc_kernel<false><<<grid, kRtThreads, smem, stream>>>(tmap_x, tmap_w, T, H, E, out, err);
  }
  return cudaGetLastError();
}

}  // namespace mosaic
