// Hyper-connection pre-mix + RMSNorm (+ act_quant) in front of the MoE, and
// the hyper-connection post-mix behind it.
//
// Reference behaviour:
//   HyperConnections.pre    mosaicvm/model/layers.py:258-267, with the Sinkhorn
//                           split of hc_split_sinkhorn :222-234
//   RMSNorm.forward         mosaicvm/model/layers.py:19-29
//   act_quant_ref           mosaicvm/kernels/fp4_source.py:110-129
//   HyperConnections.post   mosaicvm/model/layers.py:269-271
//
// Three launches.  hc_split_fn_kernel and hc_mix_tc_kernel (hc_tc.cu) make the
// split-K partials of the mixing dot products x_flat . fn^T (x_flat [T, hc*D]
// bf16, fn [(2+hc)*hc, hc*D]) and of the tokens' sums of squares on the tensor
// cores.  hc_pre_norm_kernel (TT tokens per CTA) adds the partials in a fixed
// order (deterministic), runs the Sinkhorn normalisation of the 4x4
// combination (one warp per token), forms the pre-mix y = sum_m pre_m x_m
// (bf16) in shared memory, then applies the RMSNorm (skipped without a norm
// weight) and writes the MoE input (and its E4M3 act_quant).
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


// Standalone RMSNorm: y = bf16(x * (1 / sqrt(mean(x^2) + eps)) * w) for one row
// per CTA, the row staged in shared memory between the sum-of-squares pass and
// the scaling pass (x is read from HBM once).  Optional act_quant_ref of y.
// Reference: mosaicvm/model/layers.py:19-29 (RMSNorm.forward).
constexpr int kNormThreads = 128;
__global__ void __launch_bounds__(kNormThreads) rms_norm_kernel(const __nv_bfloat16* __restrict__ x,
                                                                const float* __restrict__ w, int D, float eps,
                                                                __nv_bfloat16* __restrict__ y, uint8_t* __restrict__ q,
                                                                float* __restrict__ q_scale) {
  extern __shared__ __align__(16) uint8_t norm_smem[];
  __shared__ float red[kNormThreads / 32];
  uint4* row = reinterpret_cast<uint4*>(norm_smem);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const size_t base = static_cast<size_t>(blockIdx.x) * D;
  const int nvec = D / 8;
  const uint4* src = reinterpret_cast<const uint4*>(x + base);
  float ss = 0.f;
  for (int v = tid; v < nvec; v += kNormThreads) {
    const uint4 raw = __ldg(src + v);
    row[v] = raw;
    const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(h2[i]);
      ss = fmaf(f.x, f.x, ss);
      ss = fmaf(f.y, f.y, ss);
    }
  }
  ss = warp_sum(ss);
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < kNormThreads / 32; ++i) tot += red[i];
  const float r = 1.0f / sqrtf(tot / static_cast<float>(D) + eps);
  // Every lane runs the same iterations (quant_block128 shuffles across 16 lanes).
  const int steps = (nvec + kNormThreads - 1) / kNormThreads;
  for (int s = 0; s < steps; ++s) {
    const int v = s * kNormThreads + tid;
    const bool valid = v < nvec;
    float o[8];
    if (valid) {
      const uint4 raw = row[v];
      const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
      const float4 w0 = __ldg(reinterpret_cast<const float4*>(w) + 2 * v);
      const float4 w1 = __ldg(reinterpret_cast<const float4*>(w) + 2 * v + 1);
      const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
      __align__(16) __nv_bfloat16 ob[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(h2[i]);
        ob[2 * i] = __float2bfloat16_rn(__fmul_rn(__fmul_rn(f.x, r), wv[2 * i]));
        ob[2 * i + 1] = __float2bfloat16_rn(__fmul_rn(__fmul_rn(f.y, r), wv[2 * i + 1]));
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = __bfloat162float(ob[i]);
      reinterpret_cast<uint4*>(y + base)[v] = *reinterpret_cast<const uint4*>(ob);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = 0.f;
    }
    if (q) {
      uint8_t b[8];
      const int e = quant_block128(o, b);
      if (valid) {
        reinterpret_cast<uint2*>(q + base)[v] = pack8(b);
        if ((lane & 15) == 0) q_scale[static_cast<size_t>(blockIdx.x) * (D / 128) + v / 16] = exp2i(e);
      }
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

size_t hc_partials_bytes(int T, int splits) { return sizeof(float) * static_cast<size_t>(splits) * T * kRed; }

cudaError_t launch_hc_pre_norm(const HcParams& p_in, int num_sms, cudaStream_t stream) {
  const HcParams& p = p_in;
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

cudaError_t launch_rms_norm(const void* x, const float* w, int T, int D, float eps, void* y, uint8_t* q,
                            float* q_scale, cudaStream_t stream) {
  const size_t smem = static_cast<size_t>(D) * 2;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(rms_norm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  rms_norm_kernel<<<T, kNormThreads, smem, stream>>>(static_cast<const __nv_bfloat16*>(x), w, D, eps,
                                                     static_cast<__nv_bfloat16*>(y), q, q_scale);
  return cudaGetLastError();
}

}  // namespace mosaic
