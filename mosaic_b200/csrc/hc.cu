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
// combination; hc_premix_ring_kernel (D <= 8192: token rows streamed into a
// shared-memory ring by bulk copies, two 256-thread groups each on one token
// at a time) or hc_premix_norm_kernel (larger D: one token per CTA, loaded
// into registers) forms the pre-mix y = sum_m pre_m x_m (bf16), then applies
// the RMSNorm (skipped without a norm weight) and writes the MoE input (and
// its E4M3 act_quant).
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

// Packed fp32 pairs (f32x2, sm_100): one instruction for both lanes, each
// lane rounded to nearest like the scalar mul.rn / add.rn / fma.rn.
__device__ __forceinline__ float2 fmul2_rn(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float2 fadd2_rn(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float2 ffma2_rn(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}

// 16-byte load from shared memory (ld.shared: the short-latency path, not a
// generic load that resolves to shared memory at run time)
__device__ __forceinline__ uint4 lds128(const void* p) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(smem_u32(p))
               : "memory");
  return v;
}
__device__ __forceinline__ void named_bar(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
// named barrier that also ORs a predicate over its threads
__device__ __forceinline__ bool named_bar_any(int id, int threads, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.or.pred q, %2, %3, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(v)), "r"(id), "r"(threads)
      : "memory");
  return r != 0;
}
__device__ __forceinline__ float4 pre_of(const HcParams& p, int t) {
  return *reinterpret_cast<const float4*>(p.pre + static_cast<size_t>(t) * 4);
}

// ---- pre-mix + RMSNorm (+ act_quant) of token t by the whole CTA.  Each
// thread takes its PER 8-value chunks of all hc residual rows of the token at
// xt (global or shared memory; 16-byte loads, all issued together), forms
// y = sum_m pre_m x_m (products rounded, summed in m order, bf16) in
// registers, and the block adds the squares of y in a fixed order for the
// RMSNorm.  The THREADS threads (tid 0 .. THREADS - 1) meet once, on named
// barrier bar, after writing their warps' sums of squares to red; every thread
// then adds the THREADS / 32 sums itself.  So that no thread overwrites a sum
// another still reads, callers alternate between two red buffers from one
// token to the next.  pre4: the token's pre-mix weights (p.pre[t]).
// released() runs on every thread after the barrier, when all of them have
// read xt.
template <int THREADS, int PER, bool SMEM, class Hook>
__device__ __forceinline__ void premix_token(const HcParams& p, int t, const __nv_bfloat16* __restrict__ xt,
                                             const float4 pre4, float* red, int tid, int bar, Hook released) {
  constexpr int kChunk = THREADS * 8;  // x_flat columns per step: 8 per thread
  constexpr int kWarps = THREADS / 32;
  const int lane = tid & 31, warp = tid >> 5;
  const int hc = p.hc, D = p.D;
  __nv_bfloat16* yout = static_cast<__nv_bfloat16*>(p.y);
  uint4 raw[PER][4];
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    const int d = k * kChunk + tid * 8;
#pragma unroll
    for (int m = 0; m < 4; ++m)
      if (d < D && m < hc) {
        if (SMEM)
          raw[k][m] = lds128(xt + static_cast<size_t>(m) * D + d);
        else
          raw[k][m] = *reinterpret_cast<const uint4*>(xt + static_cast<size_t>(m) * D + d);
      }
  }
  // the arithmetic on pairs of values (packed f32x2 instructions, each lane
  // rounded as the scalar operation would be)
  const float2 pm[4] = {make_float2(pre4.x, pre4.x), make_float2(pre4.y, pre4.y), make_float2(pre4.z, pre4.z),
                        make_float2(pre4.w, pre4.w)};
  float2 yv[PER][4];
  float2 ss = make_float2(0.f, 0.f);
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    const int d = k * kChunk + tid * 8;
    if (d < D) {
      float2 y[4];
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        if (m >= hc) break;
        const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw[k][m]);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __bfloat1622float2(h2[i]);
          y[i] = m == 0 ? fmul2_rn(pm[0], f) : fadd2_rn(y[i], fmul2_rn(pm[m], f));
        }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        yv[k][i] = __bfloat1622float2(__floats2bfloat162_rn(y[i].x, y[i].y));
        ss = ffma2_rn(yv[k][i], yv[k][i], ss);
      }
    }
  }
  float ss2 = warp_sum(ss.x + ss.y);
  if (lane == 0) red[warp] = ss2;
  // a shared-memory row's next fill is an async-proxy write: order this
  // thread's generic reads of the row before it
  if (SMEM) fence_proxy_async_smem();
  named_bar(bar, THREADS);
  released();
  float sum = 0.f;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) sum += red[w];
  const float rs = 1.0f / sqrtf(sum / static_cast<float>(D) + p.norm_eps);
  // ---- RMSNorm (y * rsqrt, then * weight), bf16, optional act_quant.  Every
  // lane runs the same iterations: quant_block128 shuffles across 16 lanes.
  const float r = rs;
  const int steps = (D + kChunk - 1) / kChunk;
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    if (k >= steps) break;
    const int d = k * kChunk + tid * 8;
    const bool valid = d < D;
    float v[8];
    if (valid) {
      __align__(16) __nv_bfloat162 ob[4];
      if (p.norm_w) {
        const float4 w0 = __ldg(reinterpret_cast<const float4*>(p.norm_w + d));
        const float4 w1 = __ldg(reinterpret_cast<const float4*>(p.norm_w + d + 4));
        const float2 w[4] = {make_float2(w0.x, w0.y), make_float2(w0.z, w0.w), make_float2(w1.x, w1.y),
                             make_float2(w1.z, w1.w)};
        const float2 r2 = make_float2(r, r);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 o = fmul2_rn(fmul2_rn(yv[k][i], r2), w[i]);
          ob[i] = __floats2bfloat162_rn(o.x, o.y);
        }
      } else {  // the pre-mix alone (HyperConnections.pre)
#pragma unroll
        for (int i = 0; i < 4; ++i) ob[i] = __floats2bfloat162_rn(yv[k][i].x, yv[k][i].y);
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 o = __bfloat1622float2(ob[i]);
        v[2 * i] = o.x;
        v[2 * i + 1] = o.y;
      }
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

// Register variant, for D above the ring's 8192: one token per CTA at a time
// (grid-stride), the row loaded straight into registers.
template <int PER>
__global__ void __launch_bounds__(kHcThreads, 1) hc_premix_norm_kernel(HcParams p) {
  __shared__ float red[2][kHcWarps];
  const __nv_bfloat16* x = static_cast<const __nv_bfloat16*>(p.x);
  const size_t KD = static_cast<size_t>(p.hc) * p.D;
  int j = 0;
  for (int t = blockIdx.x; t < p.T; t += gridDim.x, ++j)
    premix_token<kHcThreads, PER, false>(p, t, x + static_cast<size_t>(t) * KD, pre_of(p, t), red[j & 1],
                                         static_cast<int>(threadIdx.x), 0, [] {});
}

// Ring variant, for token rows (hc x D bf16) that fit kHcRing times in shared
// memory: one CTA per SM, two groups of 256 threads, group g taking the CTA's
// tokens g, g + 2, ... (grid-stride over T).  Token i's row arrives in slot
// i % kHcRing by a bulk copy (cp.async.bulk, one per row); once the group that
// consumes token i has read it (the group's one barrier per token) it refills
// the slot with token i + kHcRing, so rows stay in flight while both groups do
// their arithmetic.  Token i completes a phase
// of barrier full[i % (2 * kHcRing)]: each barrier's phases belong to one group
// and are consumed in order, so a parity wait cannot match a stale phase.
// Waits are bounded: a group that gives up records MOSAIC_ERR_TIMEOUT and
// stops; at exit the CTA waits (bounded) for every copy still in flight.
constexpr int kHcRing = 3;
constexpr int kHcBars = 2 * kHcRing;
constexpr int kHcGroupThreads = 256;
constexpr int kHcRingThreads = 2 * kHcGroupThreads;
constexpr int kHcRingChunk = kHcGroupThreads * 8;
constexpr int kHcRingSmem = 225 * 1024;
static_assert(kHcRing * 4 * 4 * kHcRingChunk * 2 <= kHcRingSmem, "three rows of hc 4 x D 8192 bf16");

template <int PER>
__global__ void __launch_bounds__(kHcRingThreads, 1) hc_premix_ring_kernel(HcParams p) {
  extern __shared__ __align__(128) uint8_t ring[];
  __shared__ uint64_t full[kHcBars];
  __shared__ int filled[kHcBars], consumed[kHcBars];
  __shared__ float red[2][2][kHcGroupThreads / 32];  // [group][token parity][warp]
  __shared__ int failed;
  const int g = static_cast<int>(threadIdx.x) / kHcGroupThreads, gt = static_cast<int>(threadIdx.x) % kHcGroupThreads;
  const int bar = 1 + g;  // named barrier of the group (0 is __syncthreads)
  const size_t KD = static_cast<size_t>(p.hc) * p.D;
  const uint32_t row_bytes = static_cast<uint32_t>(KD * 2);
  const __nv_bfloat16* x = static_cast<const __nv_bfloat16*>(p.x);
  const int n = static_cast<int>(blockIdx.x) < p.T ? (p.T - 1 - static_cast<int>(blockIdx.x)) / gridDim.x + 1 : 0;
  auto token = [&](int i) { return static_cast<int>(blockIdx.x + static_cast<size_t>(i) * gridDim.x); };
  auto fill = [&](int i) {  // token i of this CTA into slot i % kHcRing (one thread)
    const int b = i % kHcBars;
    ++filled[b];
    mbar_arrive_expect_tx(&full[b], row_bytes);
    bulk_load(ring + static_cast<size_t>(i % kHcRing) * row_bytes, x + static_cast<size_t>(token(i)) * KD, row_bytes,
              &full[b]);
  };
  if (threadIdx.x == 0) {
    for (int b = 0; b < kHcBars; ++b) {
      mbar_init(&full[b], 1);
      filled[b] = consumed[b] = 0;
    }
    failed = 0;
    fence_mbar_init();
    for (int i = 0; i < kHcRing && i < n; ++i) fill(i);
  }
  __syncthreads();
  volatile int never = 0;
  // the pre-mix weights (an L2 read) one token ahead, off the token's critical path
  float4 pre_next = g < n ? pre_of(p, token(g)) : make_float4(0.f, 0.f, 0.f, 0.f);
  for (int i = g; i < n; i += 2) {
    const int b = i % kHcBars;
    const float4 pre4 = pre_next;
    if (i + 2 < n) pre_next = pre_of(p, token(i + 2));
    const bool ok = mbar_wait(&full[b], static_cast<uint32_t>(i / kHcBars) & 1u, &never);
    if (named_bar_any(bar, kHcGroupThreads, !ok)) {  // the same decision on the group's threads
      if (gt == 0) {
        set_error(p.err, MOSAIC_ERR_TIMEOUT);
        failed = 1;
      }
      break;
    }
    premix_token<kHcGroupThreads, PER, true>(
        p, token(i), reinterpret_cast<const __nv_bfloat16*>(ring + static_cast<size_t>(i % kHcRing) * row_bytes), pre4,
        red[g][(i >> 1) & 1], gt, bar, [&] {
          if (gt == 0) {
            ++consumed[b];
            if (i + kHcRing < n) fill(i + kHcRing);
          }
        });
  }
  __syncthreads();
  if (threadIdx.x == 0 && failed) {  // no copy may land in the CTA's shared memory after it exits
    for (int b = 0; b < kHcBars; ++b)
      if (filled[b] > consumed[b]) mbar_wait(&full[b], static_cast<uint32_t>(filled[b] - 1) & 1u, &never);
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
  if (p.D <= 4 * kHcRingChunk) {  // D <= 8192: the ring (three rows of up to 4 x 8192 bf16 fit)
    const size_t ring_bytes = static_cast<size_t>(kHcRing) * p.hc * p.D * 2;
    const int grid = p.T < num_sms ? p.T : num_sms;
    const bool two = p.D <= 2 * kHcRingChunk;
    const void* fn = two ? reinterpret_cast<const void*>(hc_premix_ring_kernel<2>)
                         : reinterpret_cast<const void*>(hc_premix_ring_kernel<4>);
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(ring_bytes));
    if (e != cudaSuccess) return e;
    if (two)
      hc_premix_ring_kernel<2><<<grid, kHcRingThreads, ring_bytes, stream>>>(p);
    else
      hc_premix_ring_kernel<4><<<grid, kHcRingThreads, ring_bytes, stream>>>(p);
    return cudaGetLastError();
  }
  // D in (8192, 16384]: the register kernel, one CTA of 256 threads per SM
  const int grid = p.T < num_sms ? p.T : num_sms;
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
