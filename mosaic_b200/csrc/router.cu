// Sigmoid group-limited top-k router (fp32 CUDA cores).
//
// Reference behaviour: mosaicvm/model/layers.py:127-150 (Router.forward) with
// the sigmoid score of .mosaicvm/source/inference_model.py:573-574 (Gate);
// the group limit follows the published DeepSeek-V3 rule (group score = sum
// of the two largest biased scores, keep topk_group groups, mask the rest).
//
// Kernel 1 computes fp32 logits x . W^T with a deterministic split-K: every
// split sums its K range sequentially with FMAs and writes its own partial;
// kernel 2 (one warp per token) adds the partials in split order, so a
// logit never depends on scheduling.  Kernel 2 then applies sigmoid + bias,
// the group limit and the top-k, and normalises the unbiased weights.
#include "common.cuh"
#include "kernels.h"

namespace mosaic {

namespace {

constexpr int kTileT = 64;
constexpr int kTileE = 64;
constexpr int kTileK = 32;

__global__ void __launch_bounds__(256) router_logits_kernel(const __nv_bfloat16* __restrict__ x,
                                                            const float* __restrict__ w, int T, int H, int E,
                                                            int kchunk, float* __restrict__ partial) {
  __shared__ float xs[kTileK][kTileT + 4];
  __shared__ float ws[kTileK][kTileE + 4];
  const int t0 = blockIdx.x * kTileT;
  const int e0 = blockIdx.y * kTileE;
  const int split = blockIdx.z;
  const int kbeg = split * kchunk;
  const int kend = min(H, kbeg + kchunk);
  const int tid = threadIdx.x;
  const int tx = tid & 15;
  const int ty = tid >> 4;
  const int lrow = tid >> 2;        // row of the tile this thread loads
  const int lk = (tid & 3) * 8;     // its 8 consecutive k
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;

  for (int k0 = kbeg; k0 < kend; k0 += kTileK) {
    {
      const int t = t0 + lrow;
      float v[8];
      if (t < T) {
        const uint4 raw = *reinterpret_cast<const uint4*>(x + static_cast<size_t>(t) * H + k0 + lk);
        const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __bfloat1622float2(h2[i]);
          v[2 * i] = f.x;
          v[2 * i + 1] = f.y;
        }
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = 0.f;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) xs[lk + i][lrow] = v[i];
    }
    {
      const int e = e0 + lrow;
      float v[8];
      if (e < E) {
        const float4 a = *reinterpret_cast<const float4*>(w + static_cast<size_t>(e) * H + k0 + lk);
        const float4 b = *reinterpret_cast<const float4*>(w + static_cast<size_t>(e) * H + k0 + lk + 4);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
        v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = 0.f;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) ws[lk + i][lrow] = v[i];
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < kTileK; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = xs[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = ws[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int t = t0 + ty * 4 + i;
    if (t >= T) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int e = e0 + tx * 4 + j;
      if (e < E) partial[(static_cast<size_t>(split) * T + t) * E + e] = acc[i][j];
    }
  }
}

// Better candidate: larger value, ties to the lower expert id.
__device__ __forceinline__ bool better(float v, int e, float v2, int e2) {
  return v > v2 || (v == v2 && e < e2);
}

template <int PER>
__global__ void __launch_bounds__(256) router_topk_kernel(const float* __restrict__ partial, int splits,
                                                          const float* __restrict__ bias, int T, int E, int top_k,
                                                          int n_group, int topk_group, float route_scale,
                                                          int norm, float* __restrict__ w_out,
                                                          int64_t* __restrict__ idx_out, int* err) {
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (t >= T) return;
  float s[PER], sel[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int e = lane * PER + i;
    if (e < E) {
      float logit = 0.f;
      for (int sp = 0; sp < splits; ++sp) logit += partial[(static_cast<size_t>(sp) * T + t) * E + e];
      s[i] = 1.0f / (1.0f + expf(-logit));
      sel[i] = s[i] + (bias ? bias[e] : 0.f);
    } else {
      s[i] = 0.f;
      sel[i] = -INFINITY;
    }
  }
  if (n_group > 1 && topk_group < n_group) {
    const int gsz = E / n_group;
    float my_gscore = -INFINITY;
    for (int g = 0; g < n_group; ++g) {
      float m1 = -INFINITY, m2 = -INFINITY;
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        const int e = lane * PER + i;
        if (e < E && e / gsz == g) {
          const float v = sel[i];
          if (v > m1) {
            m2 = m1;
            m1 = v;
          } else if (v > m2) {
            m2 = v;
          }
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float o1 = __shfl_xor_sync(0xFFFFFFFFu, m1, o);
        const float o2 = __shfl_xor_sync(0xFFFFFFFFu, m2, o);
        const float n1 = fmaxf(m1, o1);
        const float n2 = fmaxf(fminf(m1, o1), fmaxf(m2, o2));
        m1 = n1;
        m2 = n2;
      }
      if (lane == g) my_gscore = m1 + m2;
    }
    // rank of each group (lane g holds group g), ties to the lower group id
    int rank = 0;
    for (int h = 0; h < n_group; ++h) {
      const float o = __shfl_sync(0xFFFFFFFFu, my_gscore, h);
      if (lane < n_group && better(o, h, my_gscore, lane)) ++rank;
    }
    const unsigned keep = __ballot_sync(0xFFFFFFFFu, lane < n_group && rank < topk_group);
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int e = lane * PER + i;
      if (e < E && !((keep >> (e / gsz)) & 1u)) sel[i] = -INFINITY;
    }
  }
  float wv[8];
  int iv[8];
  float sum = 0.f;
  for (int j = 0; j < top_k; ++j) {
    float bv = -INFINITY;
    int be = 0x7FFFFFFF;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int e = lane * PER + i;
      if (e < E && better(sel[i], e, bv, be)) {
        bv = sel[i];
        be = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xFFFFFFFFu, bv, o);
      const int oe = __shfl_xor_sync(0xFFFFFFFFu, be, o);
      if (better(ov, oe, bv, be)) {
        bv = ov;
        be = oe;
      }
    }
    if (be >= E || bv == -INFINITY) {
      if (lane == 0) set_error(err, MOSAIC_ERR_RANGE);
      be = 0;
    }
    const int owner = be / PER;
    float my_s = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      if (lane == owner && lane * PER + i == be) {
        my_s = s[i];
        sel[i] = -INFINITY;
      }
    }
    const float sv = __shfl_sync(0xFFFFFFFFu, my_s, owner);
#pragma unroll
    for (int jj = 0; jj < 8; ++jj)
      if (jj == j) {
        wv[jj] = sv;
        iv[jj] = be;
      }
    sum += sv;
  }
  if (lane == 0) {
    const float denom = norm ? fmaxf(sum, 1e-9f) : 1.0f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (j < top_k) {
        float v = wv[j];
        if (norm) v = v / denom;
        w_out[static_cast<size_t>(t) * top_k + j] = v * route_scale;
        idx_out[static_cast<size_t>(t) * top_k + j] = iv[j];
      }
    }
  }
}

}  // namespace

int router_splits(int T, int H, int E, int num_sms) {
  const int tiles = ((T + kTileT - 1) / kTileT) * ((E + kTileE - 1) / kTileE);
  int s = (2 * num_sms + tiles - 1) / tiles;
  const int smax = H / 256 > 0 ? H / 256 : 1;
  if (s > smax) s = smax;
  if (s < 1) s = 1;
  return s;
}

cudaError_t launch_router(const void* x, const float* w, const float* bias, int T, int H, int E, int top_k,
                          int n_group, int topk_group, float route_scale, int norm, float* weights_out,
                          int64_t* idx_out, float* partial, int splits, int* err, cudaStream_t stream) {
  int kchunk = (H + splits - 1) / splits;
  kchunk = (kchunk + kTileK - 1) / kTileK * kTileK;
  const int used = (H + kchunk - 1) / kchunk;
  dim3 g1((T + kTileT - 1) / kTileT, (E + kTileE - 1) / kTileE, used);
  router_logits_kernel<<<g1, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(x), w, T, H, E, kchunk, partial);
  dim3 g2((T + 7) / 8);
  const int per = (E + 31) / 32;
#define MOSAIC_TOPK(P)                                                                                      \
  router_topk_kernel<P><<<g2, 256, 0, stream>>>(partial, used, bias, T, E, top_k, n_group, topk_group,     \
                                                route_scale, norm, weights_out, idx_out, err)
  if (per <= 1)
    MOSAIC_TOPK(1);
  else if (per <= 2)
    MOSAIC_TOPK(2);
  else if (per <= 4)
    MOSAIC_TOPK(4);
  else
    MOSAIC_TOPK(8);
#undef MOSAIC_TOPK
  return cudaGetLastError();
}

}  // namespace mosaic
