// Group-limited top-k router and hash router: the top-k pass, and fp32 FMA
// logits for shapes the tensor-core kernel does not take.
//
// Reference behaviour: mosaicvm/model/layers.py:127-150 (Router.forward) and
// the vendored Gate, .mosaicvm/source/inference_model.py:569-589, whose three
// score functions are kept: sigmoid (:573-574), softmax (:571-572) and
// sqrt(softplus) (:575-576, = layers.py:110-115 _router_scores).  The group
// limit follows the published DeepSeek-V3 rule (group score = sum of the two
// largest biased scores, keep topk_group groups, mask the rest).  Hash routing
// (layers.py:171-197 HashRouter.forward, Gate's tid2eid branch :581-582) takes
// the ids from a token-id table instead of the top-k, and without a table uses
// the salted multiplicative hash of layers.py:180-184.
//
// For T <= 8 (H % 64 == 0) router_small_kernel computes the logits with fp32
// FMAs and runs the top-k in the same launch.  Otherwise the logits x . W^T
// come from the tensor cores (router_tc.cu) wherever H % 64 == 0 and
// E % 16 == 0, else from the FMA kernels here; both write deterministic
// split-K partials [splits][T][E] (every split sums its K range in a fixed
// order).  router_topk_kernel (one warp per token, or 8 per
// token when there are many splits) adds the partials in a fixed order, so a
// logit never depends on scheduling, then applies the score function + bias,
// the group limit and the top-k (or the table lookup), and normalises the
// unbiased weights.
#include "common.cuh"
#include "kernels.h"

namespace mosaic {

namespace {

constexpr int kTileT = 64;
constexpr int kTileE = 64;
constexpr int kTileK = 32;

// Loads this thread's share of one K-slice: 8 consecutive k of one token row
// and of one expert row (zeros past T / E).
__device__ __forceinline__ void load_slice(const __nv_bfloat16* __restrict__ x, const float* __restrict__ w, int T,
                                           int H, int E, int t, int e, int k, float (&xv)[8], float (&wv)[8]) {
  if (t < T) {
    const uint4 raw = *reinterpret_cast<const uint4*>(x + static_cast<size_t>(t) * H + k);
    const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(h2[i]);
      xv[2 * i] = f.x;
      xv[2 * i + 1] = f.y;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) xv[i] = 0.f;
  }
  if (e < E) {
    const float4 a = *reinterpret_cast<const float4*>(w + static_cast<size_t>(e) * H + k);
    const float4 b = *reinterpret_cast<const float4*>(w + static_cast<size_t>(e) * H + k + 4);
    wv[0] = a.x; wv[1] = a.y; wv[2] = a.z; wv[3] = a.w;
    wv[4] = b.x; wv[5] = b.y; wv[6] = b.z; wv[7] = b.w;
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) wv[i] = 0.f;
  }
}

// 64 tokens x 64 experts x one K range per CTA, 4 x 4 outputs per thread.  The
// next K-slice is loaded into registers while the current one is multiplied
// out of a double-buffered shared tile, so global latency overlaps the FMAs.
// Each output sums its K range in ascending k with FMAs (deterministic).
__global__ void __launch_bounds__(256) router_logits_kernel(const __nv_bfloat16* __restrict__ x,
                                                            const float* __restrict__ w, int T, int H, int E,
                                                            int kchunk, float* __restrict__ partial) {
  __shared__ float xs[2][kTileK][kTileT + 4];
  __shared__ float ws[2][kTileK][kTileE + 4];
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

  float xv[8], wv[8];
  load_slice(x, w, T, H, E, t0 + lrow, e0 + lrow, kbeg + lk, xv, wv);
  int buf = 0;
  for (int k0 = kbeg; k0 < kend; k0 += kTileK) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      xs[buf][lk + i][lrow] = xv[i];
      ws[buf][lk + i][lrow] = wv[i];
    }
    __syncthreads();
    if (k0 + kTileK < kend) load_slice(x, w, T, H, E, t0 + lrow, e0 + lrow, k0 + kTileK + lk, xv, wv);
#pragma unroll 8
    for (int kk = 0; kk < kTileK; ++kk) {
      const float4 a = *reinterpret_cast<const float4*>(&xs[buf][kk][ty * 4]);
      const float4 b = *reinterpret_cast<const float4*>(&ws[buf][kk][tx * 4]);
      const float av[4] = {a.x, a.y, a.z, a.w};
      const float bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    buf ^= 1;  // the next slice goes to the other buffer: one barrier per slice suffices
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

// Large batches: 128 tokens x 128 experts per CTA over all of K, 8 x 8 outputs
// per thread (FMA-bound; every output still sums K in ascending order).
constexpr int kBigT = 128;
constexpr int kBigE = 128;
constexpr int kBigK = 16;

bool use_big_tiles(int T, int E, int num_sms) {
  // one wave of 128 x 128 tiles on at least half the SMs beats split-K partials
  return E % kBigE == 0 && 2 * ((T + kBigT - 1) / kBigT) * (E / kBigE) >= num_sms;
}

__global__ void __launch_bounds__(256) router_logits_big_kernel(const __nv_bfloat16* __restrict__ x,
                                                                const float* __restrict__ w, int T, int H, int E,
                                                                float* __restrict__ logits) {
  __shared__ __align__(16) float xs[2][kBigK][kBigT];
  __shared__ __align__(16) float ws[2][kBigK][kBigE];
  const int t0 = blockIdx.x * kBigT;
  const int e0 = blockIdx.y * kBigE;
  const int tid = threadIdx.x;
  const int tx = tid & 15;   // expert group: experts e0 + tx*4 + {0..3} and + 64
  const int ty = tid >> 4;   // token group: tokens t0 + ty*4 + {0..3} and + 64
  // loaders: 128 rows x 16 k per operand; thread loads row (tid >> 1), k half (tid & 1) * 8
  const int lrow = tid >> 1;
  const int lk = (tid & 1) * 8;
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
  float xv[8], wv[8];
  load_slice(x, w, T, H, E, t0 + lrow, e0 + lrow, lk, xv, wv);
  int buf = 0;
  for (int k0 = 0; k0 < H; k0 += kBigK) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      xs[buf][lk + i][lrow] = xv[i];
      ws[buf][lk + i][lrow] = wv[i];
    }
    __syncthreads();
    if (k0 + kBigK < H) load_slice(x, w, T, H, E, t0 + lrow, e0 + lrow, k0 + kBigK + lk, xv, wv);
#pragma unroll
    for (int kk = 0; kk < kBigK; ++kk) {
      const float4 a0 = *reinterpret_cast<const float4*>(&xs[buf][kk][ty * 4]);
      const float4 a1 = *reinterpret_cast<const float4*>(&xs[buf][kk][64 + ty * 4]);
      const float4 b0 = *reinterpret_cast<const float4*>(&ws[buf][kk][tx * 4]);
      const float4 b1 = *reinterpret_cast<const float4*>(&ws[buf][kk][64 + tx * 4]);
      const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    buf ^= 1;
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int t = t0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + i - 4);
    if (t >= T) continue;
    float* row = logits + static_cast<size_t>(t) * E + e0;
    *reinterpret_cast<float4*>(row + tx * 4) = make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
    *reinterpret_cast<float4*>(row + 64 + tx * 4) = make_float4(acc[i][4], acc[i][5], acc[i][6], acc[i][7]);
  }
}

// Better candidate: larger value, ties to the lower expert id.
__device__ __forceinline__ bool better(float v, int e, float v2, int e2) {
  return v > v2 || (v == v2 && e < e2);
}

// sqrt(softplus(l)) with torch's softplus (beta 1, threshold 20: l itself above 20).
// Order-preserving unsigned key of a score (larger score, larger key); NaN
// maps to 0, below every number, so it is never selected.
__device__ __forceinline__ unsigned sel_key(float v) {
  const unsigned u = __float_as_uint(v);
  return isnan(v) ? 0u : ((u & 0x80000000u) ? ~u : (u | 0x80000000u));
}

__device__ __forceinline__ float sqrt_softplus(float l) { return sqrtf(l > 20.f ? l : log1pf(expf(l))); }

// Adds splits sp0, sp0 + step, ... of this lane's PER logits in ascending order.
template <int PER>
__device__ __forceinline__ void add_splits(const float* __restrict__ pp, size_t stride, int splits, int sp0, int step,
                                           bool full, int lane, int E, float (&logit)[PER]) {
  if (full) {
    int sp = sp0;
    for (; sp + 7 * step < splits; sp += 8 * step) {
      float4 v[8][PER / 4 > 0 ? PER / 4 : 1];
#pragma unroll
      for (int u = 0; u < 8; ++u)
#pragma unroll
        for (int q = 0; q < PER / 4; ++q)
          v[u][q] = *reinterpret_cast<const float4*>(pp + static_cast<size_t>(sp + u * step) * stride + 4 * q);
#pragma unroll
      for (int u = 0; u < 8; ++u)
#pragma unroll
        for (int q = 0; q < PER / 4; ++q) {
          logit[4 * q + 0] += v[u][q].x;
          logit[4 * q + 1] += v[u][q].y;
          logit[4 * q + 2] += v[u][q].z;
          logit[4 * q + 3] += v[u][q].w;
        }
    }
    for (; sp < splits; sp += step)
#pragma unroll
      for (int q = 0; q < PER / 4; ++q) {
        const float4 v = *reinterpret_cast<const float4*>(pp + static_cast<size_t>(sp) * stride + 4 * q);
        logit[4 * q + 0] += v.x;
        logit[4 * q + 1] += v.y;
        logit[4 * q + 2] += v.z;
        logit[4 * q + 3] += v.w;
      }
  } else {
#pragma unroll
    for (int i = 0; i < PER; ++i)
      if (lane * PER + i < E)
        for (int sp = sp0; sp < splits; sp += step) logit[i] += pp[static_cast<size_t>(sp) * stride + i];
  }
}

constexpr int kTopkWays = 8;  // warps adding one token's splits when there are many

// One warp per token selects; with ways = kTopkWays a block of that many warps
// serves one token, warp w adding splits w, w + ways, ... and warp 0 adding
// the warps' sums in order w = 0, 1, ... (a fixed order: deterministic).
// Score function + bias, group limit, top-k (or the table lookup) and the
// weight normalisation of token t from this lane's PER logits (experts
// lane * PER + i); lane 0 writes the token's ids and weights.
template <int PER>
__device__ __forceinline__ void topk_select(const float (&logit)[PER], int t, int lane, const float* __restrict__ bias,
                                            int E, int top_k, int n_group, int topk_group, float route_scale,
                                            int norm, float* __restrict__ w_out, int64_t* __restrict__ idx_out,
                                            int* err, const RouteVariant& rv) {
  float s[PER], sel[PER];
  if (rv.score_func == MOSAIC_SCORE_SOFTMAX) {
    // max-shifted exponentials times the reciprocal of their sum
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < PER; ++i)
      if (lane * PER + i < E) m = fmaxf(m, logit[i]);
    m = warp_max(m);
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      s[i] = lane * PER + i < E ? expf(logit[i] - m) : 0.f;
      sum += s[i];
    }
    const float inv = 1.0f / warp_sum(sum);
#pragma unroll
    for (int i = 0; i < PER; ++i) s[i] *= inv;
  } else if (rv.score_func == MOSAIC_SCORE_SQRTSOFTPLUS) {  // a warp-uniform branch around each loop
#pragma unroll
    for (int i = 0; i < PER; ++i) s[i] = sqrt_softplus(logit[i]);
  } else {
#pragma unroll
    for (int i = 0; i < PER; ++i) s[i] = 1.0f / (1.0f + expf(-logit[i]));
  }
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int e = lane * PER + i;
    if (e < E) {
      sel[i] = s[i] + (bias ? bias[e] : 0.f);
    } else {
      s[i] = 0.f;
      sel[i] = -INFINITY;
    }
  }
  // hash routing: the ids come from the token's table row, in table order
  const int32_t* trow = nullptr;
  if (rv.tid2eid) {
    const long long tk = rv.token_ids ? static_cast<long long>(rv.token_ids[t]) : static_cast<long long>(t);
    long long r = tk % rv.table_rows;
    if (r < 0) r += rv.table_rows;  // floor modulo, as torch's % on int64
    trow = rv.tid2eid + r * top_k;
  }
  if (!trow && n_group > 1 && topk_group < n_group) {
    const int gsz = E / n_group;
    float my_gscore = -INFINITY;
    const int lpg = gsz / PER;  // lanes per group when a lane's experts lie in one group
    if (gsz % PER == 0 && lpg >= 1 && lpg <= 32 && (lpg & (lpg - 1)) == 0) {
      // top-2 of this lane's experts, then a butterfly over the group's lanes
      float m1 = -INFINITY, m2 = -INFINITY;
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        const float v = sel[i];
        if (v > m1) {
          m2 = m1;
          m1 = v;
        } else if (v > m2) {
          m2 = v;
        }
      }
      for (int o = 1; o < lpg; o <<= 1) {
        const float o1 = __shfl_xor_sync(0xFFFFFFFFu, m1, o);
        const float o2 = __shfl_xor_sync(0xFFFFFFFFu, m2, o);
        const float n1 = fmaxf(m1, o1);
        const float n2 = fmaxf(fminf(m1, o1), fmaxf(m2, o2));
        m1 = n1;
        m2 = n2;
      }
      // lane g takes group g's score from the group's first lane
      const float gs = __shfl_sync(0xFFFFFFFFu, m1 + m2, (lane * lpg) & 31);
      if (lane < n_group) my_gscore = gs;
    } else
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
    int be;
    if (trow) {
      be = trow[j];  // warp-uniform
      if (be < 0 || be >= E) {
        if (lane == 0) set_error(err, MOSAIC_ERR_RANGE);
        be = 0;
      }
    } else {
      // the largest biased score (an order-preserving key; NaN never wins), then
      // the lowest expert id holding it: two warp reductions
      unsigned bk = 0u;
      int bi = -1;
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        if (lane * PER + i < E && sel_key(sel[i]) > bk) {  // strict: the lane's lowest id among equals
          bk = sel_key(sel[i]);
          bi = i;
        }
      }
      const unsigned mk = __reduce_max_sync(0xFFFFFFFFu, bk);
      be = __reduce_min_sync(0xFFFFFFFFu, (bi >= 0 && bk == mk) ? lane * PER + bi : 0x7FFFFFFF);
      if (be >= E || mk <= sel_key(-INFINITY)) {
        if (lane == 0) set_error(err, MOSAIC_ERR_RANGE);
        be = 0;
      }
    }
    const int owner = be / PER;
    float my_s = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      if (lane == owner && lane * PER + i == be) {
        my_s = s[i];
        if (!trow) sel[i] = -INFINITY;  // a table may name an expert twice
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

template <int PER>
__global__ void __launch_bounds__(256) router_topk_kernel(const float* __restrict__ partial, int splits, int ways,
                                                          const float* __restrict__ bias, int T, int E, int top_k,
                                                          int n_group, int topk_group, float route_scale,
                                                          int norm, float* __restrict__ w_out,
                                                          int64_t* __restrict__ idx_out, int* err, RouteVariant rv) {
  griddep_wait();  // the logits kernel's partials are visible
  griddep_launch();
  __shared__ float red[kTopkWays][32 * 8];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int t = ways > 1 ? blockIdx.x : blockIdx.x * (blockDim.x >> 5) + warp;  // one token per warp / block
  if (t >= T) return;
  float logit[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) logit[i] = 0.f;
  // vector path: this lane's experts in range and every row start 16-byte aligned
  const bool full = (lane + 1) * PER <= E && (PER % 4 == 0) && (E % 4 == 0);
  const float* pp = partial + static_cast<size_t>(t) * E + lane * PER;
  const size_t stride = static_cast<size_t>(T) * E;
  if (ways > 1) {
    add_splits<PER>(pp, stride, splits, warp, ways, full, lane, E, logit);
#pragma unroll
    for (int i = 0; i < PER; ++i) red[warp][lane * PER + i] = logit[i];
    __syncthreads();
    if (warp != 0) return;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      float v = 0.f;
      for (int w = 0; w < ways; ++w) v += red[w][lane * PER + i];
      logit[i] = v;
    }
  } else {
    add_splits<PER>(pp, stride, splits, 0, 1, full, lane, E, logit);
  }
  topk_select<PER>(logit, t, lane, bias, E, top_k, n_group, topk_group, route_scale, norm, w_out, idx_out, err, rv);
}

// Small batches (T <= kSmallT): the logits and the top-k in one launch.  CTA c
// takes experts 2c and 2c + 1; warp w takes expert 2c + (w & 1) over the H
// quarter w / 2: fp32 FMAs over 4 consecutive k per lane (lane-strided by
// 128), a butterfly over the lanes, then the quarters added in order (a fixed
// order).  The logits go to logits[T][E]; the CTA that arrives last (an
// arrival count the caller zeroes) runs the top-k of every token, a warp per
// token.  The tensor-core path for these sizes is two launches of ~128 CTAs
// with a split-K top-k.
constexpr int kSmallT = 8;

template <int PER>
__global__ void __launch_bounds__(256, 1) router_small_kernel(const __nv_bfloat16* __restrict__ x,
                                                           const float* __restrict__ w, const float* __restrict__ bias,
                                                           int T, int H, int E, int top_k, int n_group,
                                                           int topk_group, float route_scale, int norm,
                                                           float* __restrict__ logits, int* __restrict__ arrivals,
                                                           float* __restrict__ w_out, int64_t* __restrict__ idx_out,
                                                           int* err, RouteVariant rv) {
  griddep_wait();
  griddep_launch();
  __shared__ float part[8][kSmallT];
  __shared__ int last;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int e = 2 * blockIdx.x + (warp & 1);
  const int hq = H / 4, k0 = (warp >> 1) * hq;
  float acc[kSmallT];
#pragma unroll
  for (int t = 0; t < kSmallT; ++t) acc[t] = 0.f;
  if (e < E) {
    // kSmallU K steps of 128 per trip, every load of the trip issued before its FMAs
    constexpr int kSmallU = 7;
    const float* wr = w + static_cast<size_t>(e) * H + k0;
    for (int kb = lane * 4; kb < hq; kb += 128 * kSmallU) {
      float4 wv[kSmallU];
#pragma unroll
      for (int u = 0; u < kSmallU; ++u)
        wv[u] = kb + 128 * u < hq ? *reinterpret_cast<const float4*>(wr + kb + 128 * u) : make_float4(0.f, 0.f, 0.f, 0.f);
      // every token's loads of the trip in flight together (rows past T read row 0, unused)
      uint2 raw[kSmallT][kSmallU];
#pragma unroll
      for (int t = 0; t < kSmallT; ++t) {
        const __nv_bfloat16* xt = x + static_cast<size_t>(t < T ? t : 0) * H + k0 + kb;
#pragma unroll
        for (int u = 0; u < kSmallU; ++u)
          raw[t][u] = kb + 128 * u < hq ? *reinterpret_cast<const uint2*>(xt + 128 * u) : make_uint2(0u, 0u);
      }
#pragma unroll
      for (int t = 0; t < kSmallT; ++t) {
#pragma unroll
        for (int u = 0; u < kSmallU; ++u) {
          const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw[t][u]);
          const float2 a = __bfloat1622float2(h2[0]), b = __bfloat1622float2(h2[1]);
          acc[t] = fmaf(a.x, wv[u].x, acc[t]);
          acc[t] = fmaf(a.y, wv[u].y, acc[t]);
          acc[t] = fmaf(b.x, wv[u].z, acc[t]);
          acc[t] = fmaf(b.y, wv[u].w, acc[t]);
        }
      }
    }
  }
#pragma unroll
  for (int t = 0; t < kSmallT; ++t) {
    const float v = warp_sum(acc[t]);
    if (lane == 0) part[warp][t] = v;
  }
  __syncthreads();
  if (threadIdx.x < 2 * T) {
    const int h = threadIdx.x & 1, t = threadIdx.x >> 1;
    const int ee = 2 * blockIdx.x + h;
    if (ee < E) logits[static_cast<size_t>(t) * E + ee] = ((part[h][t] + part[2 + h][t]) + part[4 + h][t]) + part[6 + h][t];
  }
  __threadfence();  // this CTA's logits before its arrival
  __syncthreads();
  if (threadIdx.x == 0) last = atomicAdd(arrivals, 1) == static_cast<int>(gridDim.x) - 1;
  __syncthreads();
  if (!last) return;
  __threadfence();
  if (warp < T) {
    float logit[PER];
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int e2 = lane * PER + i;
      logit[i] = e2 < E ? __ldcg(logits + static_cast<size_t>(warp) * E + e2) : 0.f;
    }
    topk_select<PER>(logit, warp, lane, bias, E, top_k, n_group, topk_group, route_scale, norm, w_out, idx_out, err,
                     rv);
  }
}

// Table-less hash routing (layers.py:180-184): one expert per token,
//   salt   = layer_idx * 2654435761 mod 2^31          (Python integers)
//   hashed = ((int32(token) + salt) * 2654435761) mod 2^31
//   id     = hashed mod E,  weight = route_scale
// evaluated as torch evaluates it on int32 tensors: the sum and the product
// wrap modulo 2^32, the literal 2^31 wraps to -2^31, and % is the floor
// modulo, so the first remainder lies in (-2^31, 0] and the second in [0, E).
__global__ void router_hash_salted_kernel(const int64_t* __restrict__ token_ids, int T, int E, int32_t salt,
                                          float route_scale, float* __restrict__ w_out,
                                          int64_t* __restrict__ idx_out) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T) return;
  const uint32_t tok = static_cast<uint32_t>(token_ids ? token_ids[t] : static_cast<int64_t>(t));
  const uint32_t h = (tok + static_cast<uint32_t>(salt)) * 2654435761u;
  const int32_t hs = static_cast<int32_t>(h);
  // floor(hs / -2^31) is -1 for hs > 0 and 0 otherwise (hs > -2^31 or == -2^31 -> 0 remainder)
  int64_t r = hs > 0 ? static_cast<int64_t>(hs) - 2147483648LL : (hs == INT32_MIN ? 0 : static_cast<int64_t>(hs));
  int64_t id = r % E;
  if (id < 0) id += E;
  w_out[t] = route_scale;
  idx_out[t] = id;
}

}  // namespace

// Split-K factor of the logits: the tensor-core kernel's where it applies;
// for the FMA kernels ~2 CTAs per SM with K ranges of at least 256 (more splits
// only add partials for the top-k pass).
int router_splits(int T, int H, int E, int num_sms) {
  if (router_tc_applies(H, E)) return router_tc_splits(T, H, E, num_sms);
  if (use_big_tiles(T, E, num_sms)) return 1;
  const int tiles = ((T + kTileT - 1) / kTileT) * ((E + kTileE - 1) / kTileE);
  int s = (2 * num_sms + tiles - 1) / tiles;
  const int smax = H / 256 > 0 ? H / 256 : 1;
  if (s > smax) s = smax;
  if (s < 1) s = 1;
  return s;
}

cudaError_t launch_router(const void* x, const float* w, const float* bias, int T, int H, int E, int top_k,
                          int n_group, int topk_group, float route_scale, int norm, float* weights_out,
                          int64_t* idx_out, float* partial, int splits, int* err, cudaStream_t stream,
                          const RouteVariant* variant) {
  const RouteVariant rv = variant ? *variant : RouteVariant{};
  if (rv.hash && !rv.tid2eid) {
    router_hash_salted_kernel<<<(T + 255) / 256, 256, 0, stream>>>(rv.token_ids, T, E, rv.salt, route_scale,
                                                                   weights_out, idx_out);
    return cudaGetLastError();
  }
  int kchunk = (H + splits - 1) / splits;
  kchunk = (kchunk + kTileK - 1) / kTileK * kTileK;
  const int used = (H + kchunk - 1) / kchunk;
  if (splits == 1 && use_big_tiles(T, E, 148)) {
    dim3 gb((T + kBigT - 1) / kBigT, E / kBigE);
    router_logits_big_kernel<<<gb, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(x), w, T, H, E, partial);
  } else {
    dim3 g1((T + kTileT - 1) / kTileT, (E + kTileE - 1) / kTileE, used);
    router_logits_kernel<<<g1, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(x), w, T, H, E, kchunk, partial);
  }
  return launch_router_topk(partial, used, bias, T, E, top_k, n_group, topk_group, route_scale, norm, weights_out,
                            idx_out, err, stream, &rv);
}

cudaError_t launch_router_topk(const float* partial, int splits, const float* bias, int T, int E, int top_k,
                               int n_group, int topk_group, float route_scale, int norm, float* weights_out,
                               int64_t* idx_out, int* err, cudaStream_t stream, const RouteVariant* variant) {
  const RouteVariant rv = variant ? *variant : RouteVariant{};
  const int used = splits;
  // many splits: a block of kTopkWays warps per token adds them; otherwise a
  // warp per token, with the warps per block spreading small batches over the
  // SMs and packing large ones
  const int ways = splits >= 2 * kTopkWays ? kTopkWays : 1;
  const int wpb = ways > 1 ? kTopkWays : (T >= 8 * 148 ? 8 : (T >= 4 * 148 ? 4 : (T >= 2 * 148 ? 2 : 1)));
  dim3 g2(ways > 1 ? T : (T + wpb - 1) / wpb);
  const int per = (E + 31) / 32;
  cudaError_t e = cudaSuccess;
#define MOSAIC_TOPK(P)                                                                                          \
  e = launch_k(router_topk_kernel<P>, g2, dim3(32 * wpb), 0, stream, partial, used, ways, bias, T, E, top_k, n_group, \
               topk_group, route_scale, norm, weights_out, idx_out, err, rv)
  if (per <= 1)
    MOSAIC_TOPK(1);
  else if (per <= 2)
    MOSAIC_TOPK(2);
  else if (per <= 4)
    MOSAIC_TOPK(4);
  else
    MOSAIC_TOPK(8);
#undef MOSAIC_TOPK
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

bool router_small_applies(int T, int H, int E) { return T >= 1 && T <= kSmallT && H % 64 == 0 && E >= 1 && E <= 256; }

cudaError_t launch_router_small(const void* x, const float* w, const float* bias, int T, int H, int E, int top_k,
                                int n_group, int topk_group, float route_scale, int norm, float* weights_out,
                                int64_t* idx_out, float* logits, int* arrivals, int* err, cudaStream_t stream,
                                const RouteVariant* variant) {
  if (!router_small_applies(T, H, E)) return cudaErrorInvalidValue;
  const RouteVariant rv = variant ? *variant : RouteVariant{};
  const dim3 grid((E + 1) / 2);
  const int per = (E + 31) / 32;
  const __nv_bfloat16* xb = static_cast<const __nv_bfloat16*>(x);
  cudaError_t e = cudaSuccess;
#define MOSAIC_SMALL(P)                                                                                         \
  e = launch_k(router_small_kernel<P>, grid, dim3(256), 0, stream, xb, w, bias, T, H, E, top_k, n_group, topk_group, \
               route_scale, norm, logits, arrivals, weights_out, idx_out, err, rv)
  if (per <= 1)
    MOSAIC_SMALL(1);
  else if (per <= 2)
    MOSAIC_SMALL(2);
  else if (per <= 4)
    MOSAIC_SMALL(4);
  else
    MOSAIC_SMALL(8);
#undef MOSAIC_SMALL
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace mosaic
