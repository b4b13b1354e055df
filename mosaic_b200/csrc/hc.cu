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
// Four launches.  hc_split_fn_kernel and hc_mix_tc_kernel (hc_tc.cu) make the
// split-K partials of the mixing dot products x_flat . fn^T (x_flat [T, hc*D]
// bf16, fn [(2+hc)*hc, hc*D]) and of the tokens' sums of squares on the tensor
// cores.  hc_sinkhorn_kernel (one warp per token) adds the partials in a fixed
// order (deterministic) and runs the Sinkhorn normalisation of the 4x4
// combination; hc_premix_norm_kernel (one token per CTA at a time) forms the
// pre-mix y = sum_m pre_m x_m (bf16) in registers, then applies the RMSNorm
// (skipped without a norm weight) and writes the MoE input (and its E4M3
// act_quant).
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

// ---- partial sums + Sinkhorn split: one warp per token.  Lane r ends up with
// value r of the token (24 mixes, then the sum of squares at kMaxMix): for each
// value, lane l adds splits l, l+32, ... in order and a butterfly adds the
// lanes, so the order is fixed (deterministic).  Writes pre [T][4] (for the
// pre-mix kernel), post and comb.
constexpr int kSkWarps = 8;

__global__ void __launch_bounds__(kSkWarps * 32) hc_sinkhorn_kernel(HcParams p) {
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * kSkWarps + (threadIdx.x >> 5);
  if (t >= p.T) return;  // the whole warp
  const int hc = p.hc, KD = hc * p.D, nmix = (2 + hc) * hc;
  // every value's partials of this lane's splits first (all loads in flight), then
  // the 25 independent butterflies
  float part[kRed];
#pragma unroll
  for (int r = 0; r < kRed; ++r) part[r] = 0.f;
  for (int sp = lane; sp < p.splits; sp += 32) {
    const float* src = p.partial + (static_cast<size_t>(sp) * p.T + t) * kRed;
#pragma unroll
    for (int r = 0; r < kRed; ++r)
      if (r < nmix || r == kMaxMix) part[r] += src[r];
  }
  float mine = 0.f;
#pragma unroll
  for (int r = 0; r < kRed; ++r) {
    const float s = warp_sum(part[r]);
    if (lane == r) mine = s;
  }
  const float rs = 1.0f / sqrtf(__shfl_sync(0xFFFFFFFFu, mine, kMaxMix) / static_cast<float>(KD) + p.norm_eps);
  const float m_post = __shfl_sync(0xFFFFFFFFu, mine, (hc + lane) & 31);
  if (lane < hc) {
    p.pre[static_cast<size_t>(t) * 4 + lane] = sigmoidf(mine * rs * p.scale[0] + p.base[lane]) + p.hc_eps;
    p.post[static_cast<size_t>(t) * hc + lane] = 2.0f * sigmoidf(m_post * rs * p.scale[1] + p.base[hc + lane]);
  }
  // Sinkhorn: lane 4i+j (< 16) holds comb[i][j], rows are 4-lane groups (xor 1,
  // 2), columns stride 4 (xor 4, 8)
  const int ci = (lane >> 2) & 3, cj = lane & 3;
  const bool on = lane < 16 && ci < hc && cj < hc;
  const int r = 2 * hc + ci * hc + cj;
  const float m_comb = __shfl_sync(0xFFFFFFFFu, mine, on ? r : 0);
  const float v = on ? m_comb * rs * p.scale[2] + p.base[r] : -INFINITY;
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

// ---- pre-mix + RMSNorm (+ act_quant): one token per CTA at a time
// (grid-stride).  Each thread loads its PER 8-value chunks of all hc residual
// rows up front (16-byte loads, all in flight together), forms y = sum_m
// pre_m x_m (products rounded, summed in m order, bf16) in registers, and the
// block adds the squares of y in a fixed order for the RMSNorm.
template <int PER>
__global__ void __launch_bounds__(kHcThreads, PER <= 4 ? 2 : 1) hc_premix_norm_kernel(HcParams p) {
  __shared__ float red[kHcWarps];
  __shared__ float rs_s;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int hc = p.hc, D = p.D, KD = hc * D;
  const __nv_bfloat16* x = static_cast<const __nv_bfloat16*>(p.x);
  __nv_bfloat16* yout = static_cast<__nv_bfloat16*>(p.y);
  for (int t = blockIdx.x; t < p.T; t += gridDim.x) {
    const __nv_bfloat16* xt = x + static_cast<size_t>(t) * KD;
    uint4 raw[PER][4];
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      const int d = k * kHcChunk + tid * 8;
#pragma unroll
      for (int m = 0; m < 4; ++m)
        if (d < D && m < hc) raw[k][m] = *reinterpret_cast<const uint4*>(xt + static_cast<size_t>(m) * D + d);
    }
    const float4 pre4 = *reinterpret_cast<const float4*>(p.pre + static_cast<size_t>(t) * 4);
    const float pm[4] = {pre4.x, pre4.y, pre4.z, pre4.w};
    float yv[PER][8];
    float ss2 = 0.f;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      const int d = k * kHcChunk + tid * 8;
      if (d < D) {
        float y[8];
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          if (m >= hc) break;
          const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw[k][m]);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 f = __bfloat1622float2(h2[i]);
            if (m == 0) {
              y[2 * i] = __fmul_rn(pm[0], f.x);
              y[2 * i + 1] = __fmul_rn(pm[0], f.y);
            } else {
              y[2 * i] = __fadd_rn(y[2 * i], __fmul_rn(pm[m], f.x));
              y[2 * i + 1] = __fadd_rn(y[2 * i + 1], __fmul_rn(pm[m], f.y));
            }
          }
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          yv[k][i] = __bfloat162float(__float2bfloat16_rn(y[i]));
          ss2 = fmaf(yv[k][i], yv[k][i], ss2);
        }
      }
    }
    ss2 = warp_sum(ss2);
    if (lane == 0) red[warp] = ss2;
    __syncthreads();
    if (tid == 0) {
      float s = 0.f;
      for (int w = 0; w < kHcWarps; ++w) s += red[w];
      rs_s = 1.0f / sqrtf(s / static_cast<float>(D) + p.norm_eps);
    }
    __syncthreads();
    // ---- RMSNorm (y * rsqrt, then * weight), bf16, optional act_quant.  Every
    // lane runs the same iterations: quant_block128 shuffles across 16 lanes.
    const float r = rs_s;
    const int steps = (D + kHcChunk - 1) / kHcChunk;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      if (k >= steps) break;
      const int d = k * kHcChunk + tid * 8;
      const bool valid = d < D;
      float v[8];
      if (valid) {
        __align__(16) __nv_bfloat16 ob[8];
        if (p.norm_w) {
          const float4 w0 = __ldg(reinterpret_cast<const float4*>(p.norm_w + d));
          const float4 w1 = __ldg(reinterpret_cast<const float4*>(p.norm_w + d + 4));
          const float w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
          for (int i = 0; i < 8; ++i) ob[i] = __float2bfloat16_rn(__fmul_rn(__fmul_rn(yv[k][i], r), w[i]));
        } else {  // the pre-mix alone (HyperConnections.pre)
#pragma unroll
          for (int i = 0; i < 8; ++i) ob[i] = __float2bfloat16_rn(yv[k][i]);
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = __bfloat162float(ob[i]);
        *reinterpret_cast<uint4*>(yout + static_cast<size_t>(t) * D + d) = *reinterpret_cast<const uint4*>(ob);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = 0.f;
      }
      if (p.q) {
        uint8_t b[8];
        const int e = quant_block128(v, b);
        if (valid) {
          *reinterpret_cast<uint2*>(p.q + static_cast<size_t>(t) * D + d) = pack8(b);
          if ((lane & 15) == 0) p.q_scale[static_cast<size_t>(t) * (D / 128) + d / 128] = exp2i(e);
        }
      }
    }
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

int hc_max_d() { return kHcChunk * 8; }

size_t hc_partials_bytes(int T, int splits) { return sizeof(float) * static_cast<size_t>(splits) * T * kRed; }

cudaError_t launch_hc_pre_norm(const HcParams& p, int num_sms, cudaStream_t stream) {
  if (p.D > hc_max_d() || p.D % 8 || p.hc < 1 || p.hc > 4) return cudaErrorInvalidValue;
  hc_sinkhorn_kernel<<<(p.T + kSkWarps - 1) / kSkWarps, kSkWarps * 32, 0, stream>>>(p);
  // two CTAs of 256 threads per SM (the registers of the rows in flight; one above D = 8192)
  const int per_sm = p.D <= 4 * kHcChunk ? 2 : 1;
  const int grid = p.T < per_sm * num_sms ? p.T : per_sm * num_sms;
  if (p.D <= 2 * kHcChunk)
    hc_premix_norm_kernel<2><<<grid, kHcThreads, 0, stream>>>(p);
  else if (p.D <= 4 * kHcChunk)
    hc_premix_norm_kernel<4><<<grid, kHcThreads, 0, stream>>>(p);
  else
    hc_premix_norm_kernel<8><<<grid, kHcThreads, 0, stream>>>(p);
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
