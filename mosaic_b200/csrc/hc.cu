// Hyper-connection pre-mix + RMSNorm (+ act_quant) in front of the MoE, and
// the hyper-connection post-mix behind it (fp32 CUDA cores, HBM-bound).
//
// Reference behaviour:
//   HyperConnections.pre    mosaicvm/model/layers.py:258-267, with the Sinkhorn
//                           split of hc_split_sinkhorn :222-234
//   RMSNorm.forward         mosaicvm/model/layers.py:19-29
//   act_quant_ref           mosaicvm/kernels/fp4_source.py:110-129
//   HyperConnections.post   mosaicvm/model/layers.py:269-271
//
// Two launches.  hc_mix_kernel is a split-K fp32 GEMM of the residual copies
// x_flat [T, hc*D] (bf16) against fn [(2+hc)*hc, hc*D]: a CTA takes 128 tokens
// x one K range, stages 32-wide K slices of x (transposed) and fn in shared
// memory, and each thread accumulates a 4-token x 4-mix tile (plus the tokens'
// sums of squares), so fn is read once per 128 tokens instead of once per
// token.  Each split writes its own partials; hc_pre_norm_kernel (TT tokens
// per CTA) adds them in split order (deterministic), runs the Sinkhorn
// normalisation of the 4x4 combination (one warp per token), forms the
// pre-mix y = sum_m pre_m x_m (bf16) in shared memory, then applies the
// RMSNorm (skipped without a norm weight) and writes the MoE input (and its
// E4M3 act_quant).
#include "common.cuh"
#include "kernels.h"

namespace mosaic {

namespace {

constexpr int kHcThreads = 256;
constexpr int kHcWarps = kHcThreads / 32;
constexpr int kHcChunk = kHcThreads * 8;  // x_flat columns per step: 8 per thread
constexpr int kMaxMix = 24;               // (2 + hc) * hc at hc = 4
constexpr int kRed = kMaxMix + 1;         // mixes + sum of squares per token

__device__ __forceinline__ float sigmoidf(float v) { return 1.0f / (1.0f + expf(-v)); }

constexpr int kMixTok = 128;     // tokens per hc_mix CTA
constexpr int kMixK = 32;        // K slice staged per step
constexpr int kMixThreads = 192; // 32 token groups of 4 x 6 mix groups of 4

__global__ void __launch_bounds__(kMixThreads) hc_mix_kernel(const __nv_bfloat16* __restrict__ x,
                                                            const float* __restrict__ fn, int T, int KD, int nmix,
                                                            int kchunk, float* __restrict__ partial) {
  __shared__ __align__(16) float xs[kMixK][kMixTok];  // x slice, transposed: [k][token]
  __shared__ __align__(16) float fs[kMixK][kMaxMix];  // fn slice, transposed: [k][mix]
  const int tid = threadIdx.x;
  const int t0 = blockIdx.x * kMixTok;
  const int ks = blockIdx.y;
  const int k_begin = ks * kchunk;
  const int k_end = min(KD, k_begin + kchunk);
  const int tg = tid / 6, mg = tid % 6;  // tokens 4tg..4tg+3, mixes 4mg..4mg+3
  float acc[4][4], ssq[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    ssq[i] = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  }
  // The next slice is loaded into registers while the current one is used, so
  // the HBM latency of x overlaps the FMAs.  x: 128 tokens x 32 k = 512 vectors
  // of 8 bf16 (threads < 128 take three, the others two); fn: 24 x 32 = 192 float4.
  uint4 xr[3];
  float4 fr;
  const int fmix = tid >> 3, fseg = tid & 7;
  auto load_slice = [&](int k0) {
#pragma unroll
    for (int u = 0; u < 3; ++u) {
      const int i = tid + u * kMixThreads;
      xr[u] = make_uint4(0u, 0u, 0u, 0u);
      if (i < kMixTok * (kMixK / 8)) {
        const int t = t0 + (i >> 2), k = k0 + (i & 3) * 8;
        if (t < T && k < k_end) xr[u] = __ldg(reinterpret_cast<const uint4*>(x + static_cast<size_t>(t) * KD + k));
      }
    }
    const int k = k0 + fseg * 4;
    fr = make_float4(0.f, 0.f, 0.f, 0.f);
    if (fmix < nmix && k < k_end) fr = __ldg(reinterpret_cast<const float4*>(fn + static_cast<size_t>(fmix) * KD + k));
  };
  if (k_begin < k_end) load_slice(k_begin);
  for (int k0 = k_begin; k0 < k_end; k0 += kMixK) {
#pragma unroll
    for (int u = 0; u < 3; ++u) {
      const int i = tid + u * kMixThreads;
      if (i < kMixTok * (kMixK / 8)) {
        const int row = i >> 2, seg = i & 3;
        const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&xr[u]);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __bfloat1622float2(h2[j]);
          xs[seg * 8 + 2 * j][row] = f.x;
          xs[seg * 8 + 2 * j + 1][row] = f.y;
        }
      }
    }
    fs[fseg * 4 + 0][fmix] = fr.x;
    fs[fseg * 4 + 1][fmix] = fr.y;
    fs[fseg * 4 + 2][fmix] = fr.z;
    fs[fseg * 4 + 3][fmix] = fr.w;
    __syncthreads();
    if (k0 + kMixK < k_end) load_slice(k0 + kMixK);
#pragma unroll 8
    for (int kk = 0; kk < kMixK; ++kk) {
      const float4 xv = *reinterpret_cast<const float4*>(&xs[kk][4 * tg]);
      const float4 fv = *reinterpret_cast<const float4*>(&fs[kk][4 * mg]);
      const float xa[4] = {xv.x, xv.y, xv.z, xv.w};
      const float fa[4] = {fv.x, fv.y, fv.z, fv.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(xa[i], fa[j], acc[i][j]);
        ssq[i] = fmaf(xa[i], xa[i], ssq[i]);
      }
    }
    __syncthreads();
  }
  float* out = partial + static_cast<size_t>(ks) * T * kRed;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int t = t0 + 4 * tg + i;
    if (t >= T) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int mix = 4 * mg + j;
      if (mix < nmix) out[static_cast<size_t>(t) * kRed + mix] = acc[i][j];
    }
    if (mg == 0) out[static_cast<size_t>(t) * kRed + kMaxMix] = ssq[i];
  }
}

template <int TT>
__global__ void __launch_bounds__(kHcThreads) hc_pre_norm_kernel(HcParams p) {
  extern __shared__ __align__(16) uint8_t smem[];
  __nv_bfloat16* ybuf = reinterpret_cast<__nv_bfloat16*>(smem);                   // [TT][D]
  float* red = reinterpret_cast<float*>(smem + static_cast<size_t>(TT) * p.D * 2);  // [warps][TT]
  float* tot = red + kHcWarps * TT * kRed;                                          // [TT][kRed]
  float* pre_s = tot + TT * kRed;                                                   // [TT][4]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int hc = p.hc, D = p.D, KD = hc * D, nmix = (2 + hc) * hc;
  const __nv_bfloat16* x = static_cast<const __nv_bfloat16*>(p.x);
  __nv_bfloat16* yout = static_cast<__nv_bfloat16*>(p.y);
  for (int t0 = blockIdx.x * TT; t0 < p.T; t0 += gridDim.x * TT) {
    // ---- mixing dot products and sums of squares: the splits' partials.  Warp w
    // reduces values w, w+8, ...; lane l adds splits l, l+32, ... in order and
    // a butterfly adds the lanes, so the order is fixed (deterministic).
    for (int i = warp; i < TT * kRed; i += kHcWarps) {
      const int t = t0 + i / kRed, r = i % kRed;
      float s = 0.f;
      if (t < p.T && (r < nmix || r == kMaxMix))
        for (int sp = lane; sp < p.splits; sp += 32) s += p.partial[(static_cast<size_t>(sp) * p.T + t) * kRed + r];
      s = warp_sum(s);
      if (lane == 0) tot[i] = s;
    }
    __syncthreads();
    // ---- Sinkhorn split: warp tt takes token tt; lane 4i+j (< 16) holds comb[i][j],
    // rows are 4-lane groups (xor 1, 2), columns stride 4 (xor 4, 8)
    if (warp < TT && t0 + warp < p.T) {
      const int t = t0 + warp;
      const float* mt = tot + warp * kRed;
      const float rs = 1.0f / sqrtf(mt[kMaxMix] / static_cast<float>(KD) + p.norm_eps);
      if (lane < hc) {
        pre_s[warp * 4 + lane] = sigmoidf(mt[lane] * rs * p.scale[0] + p.base[lane]) + p.hc_eps;
        p.post[static_cast<size_t>(t) * hc + lane] = 2.0f * sigmoidf(mt[hc + lane] * rs * p.scale[1] + p.base[hc + lane]);
      }
      const int ci = (lane >> 2) & 3, cj = lane & 3;
      const bool on = lane < 16 && ci < hc && cj < hc;
      const int r = 2 * hc + ci * hc + cj;
      const float v = on ? mt[r] * rs * p.scale[2] + p.base[r] : -INFINITY;
      float mx = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 2));
      float c = on ? expf(v - mx) : 0.f;
      float sum = c + __shfl_xor_sync(0xFFFFFFFFu, c, 1);
      sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 2);
      c = on ? c / sum + p.hc_eps : 0.f;
      // row / column normalisations: products with the reciprocal of each sum
      for (int it = 1; it < p.iters; ++it) {
        float rsum = c + __shfl_xor_sync(0xFFFFFFFFu, c, 1);
        rsum += __shfl_xor_sync(0xFFFFFFFFu, rsum, 2);
        c *= 1.0f / (rsum + p.hc_eps);
        float csum = c + __shfl_xor_sync(0xFFFFFFFFu, c, 4);
        csum += __shfl_xor_sync(0xFFFFFFFFu, csum, 8);
        c *= 1.0f / (csum + p.hc_eps);
      }
      if (on) p.comb[(static_cast<size_t>(t) * hc + ci) * hc + cj] = c;
    }
    __syncthreads();
    // ---- pass B: y = sum_m pre_m x_m (products rounded, summed in m order), bf16
    float ss2[TT];
#pragma unroll
    for (int t = 0; t < TT; ++t) {
      ss2[t] = 0.f;
      if (t0 + t >= p.T) continue;
      const __nv_bfloat16* xt = x + static_cast<size_t>(t0 + t) * KD;
      for (int d = tid * 8; d < D; d += kHcChunk) {
        float y[8], xv[8];
        load8_bf16(xt + d, xv);
        const float p0 = pre_s[t * 4];
#pragma unroll
        for (int i = 0; i < 8; ++i) y[i] = __fmul_rn(p0, xv[i]);
        for (int m = 1; m < hc; ++m) {
          load8_bf16(xt + static_cast<size_t>(m) * D + d, xv);
          const float pm = pre_s[t * 4 + m];
#pragma unroll
          for (int i = 0; i < 8; ++i) y[i] = __fadd_rn(y[i], __fmul_rn(pm, xv[i]));
        }
        __align__(16) __nv_bfloat16 yb[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          yb[i] = __float2bfloat16_rn(y[i]);
          const float f = __bfloat162float(yb[i]);
          ss2[t] = fmaf(f, f, ss2[t]);
        }
        *reinterpret_cast<uint4*>(ybuf + static_cast<size_t>(t) * D + d) = *reinterpret_cast<const uint4*>(yb);
      }
    }
#pragma unroll
    for (int t = 0; t < TT; ++t) {
      const float v = warp_sum(ss2[t]);
      if (lane == 0) red[warp * TT + t] = v;
    }
    __syncthreads();
    if (tid < TT) {
      float s = 0.f;
      for (int w = 0; w < kHcWarps; ++w) s += red[w * TT + tid];
      tot[tid] = 1.0f / sqrtf(s / static_cast<float>(D) + p.norm_eps);
    }
    __syncthreads();
    // ---- pass C: RMSNorm (x * rsqrt, then * weight), bf16, optional act_quant.
    // Every lane runs the same iterations: quant_block128 shuffles across 16 lanes.
    const int steps = (D + kHcChunk - 1) / kHcChunk;
#pragma unroll
    for (int t = 0; t < TT; ++t) {
      if (t0 + t >= p.T) continue;
      const float r = tot[t];
      for (int s = 0; s < steps; ++s) {
        const int d = s * kHcChunk + tid * 8;
        const bool valid = d < D;
        float v[8];
        if (valid) {
          float yv[8];
          load8_bf16(ybuf + static_cast<size_t>(t) * D + d, yv);
          __align__(16) __nv_bfloat16 ob[8];
          if (p.norm_w) {
            const float4 w0 = __ldg(reinterpret_cast<const float4*>(p.norm_w + d));
            const float4 w1 = __ldg(reinterpret_cast<const float4*>(p.norm_w + d + 4));
            const float w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
            for (int i = 0; i < 8; ++i) ob[i] = __float2bfloat16_rn(__fmul_rn(__fmul_rn(yv[i], r), w[i]));
          } else {  // the pre-mix alone (HyperConnections.pre)
#pragma unroll
            for (int i = 0; i < 8; ++i) ob[i] = __float2bfloat16_rn(yv[i]);
          }
#pragma unroll
          for (int i = 0; i < 8; ++i) v[i] = __bfloat162float(ob[i]);
          *reinterpret_cast<uint4*>(yout + static_cast<size_t>(t0 + t) * D + d) =
              *reinterpret_cast<const uint4*>(ob);
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i) v[i] = 0.f;
        }
        if (p.q) {
          uint8_t b[8];
          const int e = quant_block128(v, b);
          if (valid) {
            *reinterpret_cast<uint2*>(p.q + static_cast<size_t>(t0 + t) * D + d) = pack8(b);
            if ((lane & 15) == 0) p.q_scale[static_cast<size_t>(t0 + t) * (D / 128) + d / 128] = exp2i(e);
          }
        }
      }
    }
    __syncthreads();  // ybuf / red / tot are reused by the next token group
  }
}

// out[t, m] = post[t, m] * y[t] + sum_n comb[t, m, n] * residual[t, n]; 8 values per thread.
__global__ void __launch_bounds__(256) hc_post_kernel(const __nv_bfloat16* __restrict__ y,
                                                      const __nv_bfloat16* __restrict__ res,
                                                      const float* __restrict__ post, const float* __restrict__ comb,
                                                      int T, int D, int hc, __nv_bfloat16* __restrict__ out) {
  const int per_token = D / 8;
  const long long units = static_cast<long long>(T) * per_token;
  for (long long u = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; u < units;
       u += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int t = static_cast<int>(u / per_token);
    const int d = static_cast<int>(u % per_token) * 8;
    float yv[8], rv[4][8];
    load8_bf16(y + static_cast<size_t>(t) * D + d, yv);
#pragma unroll
    for (int n = 0; n < 4; ++n) {
      if (n < hc) {
        load8_bf16(res + (static_cast<size_t>(t) * hc + n) * D + d, rv[n]);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) rv[n][i] = 0.f;
      }
    }
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      if (m >= hc) break;
      const float pm = post[static_cast<size_t>(t) * hc + m];
      const float* cm = comb + (static_cast<size_t>(t) * hc + m) * hc;
      float cv[4];
#pragma unroll
      for (int n = 0; n < 4; ++n) cv[n] = n < hc ? cm[n] : 0.f;
      __align__(16) __nv_bfloat16 ob[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float e = 0.f;
#pragma unroll
        for (int n = 0; n < 4; ++n)
          if (n < hc) e = fmaf(cv[n], rv[n][i], e);
        ob[i] = __float2bfloat16_rn(__fadd_rn(__fmul_rn(pm, yv[i]), e));
      }
      *reinterpret_cast<uint4*>(out + (static_cast<size_t>(t) * hc + m) * D + d) = *reinterpret_cast<const uint4*>(ob);
    }
  }
}

}  // namespace

size_t hc_pre_norm_smem_bytes(int tt, int D) {
  return static_cast<size_t>(tt) * D * 2 + sizeof(float) * (kHcWarps * tt * kRed + tt * kRed + tt * 4);
}

// One token per CTA: the per-token kernel reads nothing that tokens could share,
// and small CTAs keep many loads in flight on every SM.
int hc_tokens_per_cta(int T, int num_sms) {
  (void)T;
  (void)num_sms;
  return 1;
}

// K split of hc_mix_kernel: K ranges of whole 32-wide slices.
void hc_mix_split(int T, int KD, int num_sms, int* splits, int* kchunk) {
  const int tiles = (T + kMixTok - 1) / kMixTok;
  int s = (8 * num_sms + tiles - 1) / tiles;  // about eight CTAs per SM
  const int smax = KD / (8 * kMixK);  // at least eight slices per split
  if (s > smax) s = smax;
  if (s < 1) s = 1;
  int kc = (KD + s - 1) / s;
  kc = (kc + kMixK - 1) / kMixK * kMixK;
  *kchunk = kc;
  *splits = (KD + kc - 1) / kc;
}

size_t hc_pre_norm_workspace_bytes(int T, int D, int hc, int num_sms) {
  int splits = 0, kchunk = 0;
  hc_mix_split(T, hc * D, num_sms, &splits, &kchunk);
  return sizeof(float) * static_cast<size_t>(splits) * T * kRed;
}

cudaError_t launch_hc_pre_norm(const HcParams& p_in, int num_sms, cudaStream_t stream) {
  HcParams p = p_in;
  const int KD = p.hc * p.D;
  int kchunk = 0;
  hc_mix_split(p.T, KD, num_sms, &p.splits, &kchunk);
  dim3 gm((p.T + kMixTok - 1) / kMixTok, p.splits);
  hc_mix_kernel<<<gm, kMixThreads, 0, stream>>>(static_cast<const __nv_bfloat16*>(p.x), p.fn, p.T, KD,
                                                (2 + p.hc) * p.hc, kchunk, p.partial);
  const int tt = hc_tokens_per_cta(p.T, num_sms);
  const int groups = (p.T + tt - 1) / tt;
  const int grid = groups < 16 * num_sms ? groups : 16 * num_sms;
  const size_t smem = hc_pre_norm_smem_bytes(tt, p.D);
#define MOSAIC_HC(TT)                                                                                     \
  do {                                                                                                    \
    cudaError_t e = cudaFuncSetAttribute(hc_pre_norm_kernel<TT>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                         static_cast<int>(smem));                                         \
    if (e != cudaSuccess) return e;                                                                       \
    hc_pre_norm_kernel<TT><<<grid, kHcThreads, smem, stream>>>(p);                                        \
  } while (0)
  if (tt == 4)
    MOSAIC_HC(4);
  else if (tt == 2)
    MOSAIC_HC(2);
  else
    MOSAIC_HC(1);
#undef MOSAIC_HC
  return cudaGetLastError();
}

cudaError_t launch_hc_post(const void* y, const void* residual, const float* post, const float* comb, int T, int D,
                           int hc, void* out, int num_sms, cudaStream_t stream) {
  const long long units = static_cast<long long>(T) * (D / 8);
  long long blocks = (units + 255) / 256;
  const long long cap = static_cast<long long>(num_sms) * 8;
  if (blocks > cap) blocks = cap;
  hc_post_kernel<<<static_cast<int>(blocks), 256, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(y), static_cast<const __nv_bfloat16*>(residual), post, comb, T, D, hc,
      static_cast<__nv_bfloat16*>(out));
  return cudaGetLastError();
}

}  // namespace mosaic
