// Activation quantisation into packed expert rows, the reference act_quant,
// the MXFP4 weight packer and the weight-scale re-layout.
//
// Reference behaviour:
//   act_quant_ref         mosaicvm/kernels/fp4_source.py:110-129
//   pack_mxfp4_nk         mosaicvm/kernels/fp4_source.py:35-64 with the FLOOR E8M0
//                         scale of mosaicvm/kernels/mxfp4.py:32-43 and the RNE E2M1
//                         rounding of mosaicvm/kernels/mxfp4.py:46-82
//   bank re-layout        mosaicvm/kernels/qpa_mma.py:577-613 (prepack_expert_bank_qpa)
#include "common.cuh"
#include "kernels.h"

namespace mosaic {

namespace {

// hi + lo split on 8 values; the 32-block spans 4 lanes.
__device__ __forceinline__ void split_block32(const float (&v)[8], uint8_t (&hi)[8], uint8_t (&lo)[8], int& eh,
                                              int& el) {
  float m = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) m = fmaxf(m, fabsf(v[i]));
  m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, 2));
  m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, 1));
  eh = max(-126, min(127, pow2_scale_exp(m, 1e-30f)));
  const float ih = exp2i(-eh), sh = exp2i(eh);
  float r[8];
  float m2 = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    hi[i] = f32_to_e4m3(v[i] * ih);
    r[i] = v[i] - e4m3_to_f32(hi[i]) * sh;
    m2 = fmaxf(m2, fabsf(r[i]));
  }
  m2 = fmaxf(m2, __shfl_xor_sync(0xFFFFFFFFu, m2, 2));
  m2 = fmaxf(m2, __shfl_xor_sync(0xFFFFFFFFu, m2, 1));
  el = max(-126, min(127, pow2_scale_exp(m2, fmaxf(m * 1e-7f, 1e-30f))));
  const float il = exp2i(-el);
#pragma unroll
  for (int i = 0; i < 8; ++i) lo[i] = f32_to_e4m3(r[i] * il);
}

// Gather the four per-32 exponents of a 128-block (lanes g, g+4, g+8, g+12 of
// each 16-lane half) into one scale word on the half's first lane.
__device__ __forceinline__ uint32_t gather_word(int e) {
  const int lane = threadIdx.x & 31;
  const int src = lane & ~15;
  uint32_t w = 0;
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const int eg = __shfl_sync(0xFFFFFFFFu, e, src + 4 * g);
    w |= (static_cast<uint32_t>(eg + 127) & 0xFFu) << (8 * g);
  }
  return w;
}

// A block per token row (grid-stride over rows; with T_dev only the first
// *T_dev rows exist, the grid being sized for T); small batches give a row
// gridDim.y blocks, each taking every gridDim.y-th group of 8 chunks.  The row's destinations --
// its k packed rows (row_of) and the shared expert's row -- and their tile
// positions are looked up once into shared memory; each warp then quantises
// 256-value chunks of the row (H % 256 == 0) and writes them to every
// destination row: K-tile-major planes [kt][plane][R_pad][128 B], the scale
// words into the row's token-tile chunk (word (n % 32) * 4 + n / 32 of chunk
// [tile][kt], n = the row's position in its tile; the lo plane of a bf16 tile
// sits at positions rpad + n of the same chunk).
constexpr int kRqThreads = 256;
constexpr int kRqMaxRows = 16;  // top_k (<= 8) + the shared expert's row

__global__ void __launch_bounds__(kRqThreads) rows_quant_kernel(const __nv_bfloat16* __restrict__ x, int T,
                                                                const int* __restrict__ T_dev, int H, int ldx, int k,
                                                                const int* __restrict__ row_of, int shared_base,
                                                                int hilo, int R_pad, const int* __restrict__ row_tile,
                                                                const int* __restrict__ row_pos,
                                                                uint8_t* __restrict__ xq, uint32_t* __restrict__ sft) {
  griddep_wait();  // the layout's row maps are visible
  griddep_launch();
  __shared__ int s_row[kRqMaxRows], s_pos[kRqMaxRows], s_tile[kRqMaxRows];
  const int rows = T_dev ? min(*T_dev, T) : T;
  const int nrows = k + (shared_base >= 0 ? 1 : 0);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int KT = H / 128;
  for (int t = blockIdx.x; t < rows; t += gridDim.x) {
    if (threadIdx.x < nrows) {
      const int s = threadIdx.x;
      const int r = (s < k) ? row_of[static_cast<size_t>(t) * k + s] : shared_base + t;
      s_row[s] = r;
      s_pos[s] = r >= 0 ? row_pos[r] : 0;
      s_tile[s] = r >= 0 ? row_tile[r] : 0;
    }
    __syncthreads();
    // small batches spread a row over gridDim.y blocks
    for (int c = blockIdx.y * (kRqThreads / 32) + warp; c < H / 256; c += gridDim.y * (kRqThreads / 32)) {
      const int k0 = c * 256 + lane * 8;
      const int kt = k0 / 128;
      float v[8];
      load8_bf16(x + static_cast<size_t>(t) * ldx + k0, v);
      if (!hilo) {
        uint8_t q[8];
        const int e = quant_block128(v, q);
        const uint2 pq = pack8(q);
        const uint32_t word = (static_cast<uint32_t>(e + 127) & 0xFFu) * 0x01010101u;
        for (int s = 0; s < nrows; ++s) {
          const int r = s_row[s];
          if (r < 0) continue;
          *reinterpret_cast<uint2*>(xq + (static_cast<size_t>(kt) * R_pad + r) * 128 + (k0 & 127)) = pq;
          if ((lane & 15) == 0) {
            const int n = s_pos[s] & 0xFF;
            sft[(static_cast<size_t>(s_tile[s]) * KT + kt) * 128 + (n & 31) * 4 + (n >> 5)] = word;
          }
        }
      } else {
        uint8_t hi[8], lo[8];
        int eh, el;
        split_block32(v, hi, lo, eh, el);
        const uint32_t wh = gather_word(eh);
        const uint32_t wl = gather_word(el);
        const uint2 ph = pack8(hi), pl = pack8(lo);
        for (int s = 0; s < nrows; ++s) {
          const int r = s_row[s];
          if (r < 0) continue;
          *reinterpret_cast<uint2*>(xq + ((static_cast<size_t>(kt) * 2 + 0) * R_pad + r) * 128 + (k0 & 127)) = ph;
          *reinterpret_cast<uint2*>(xq + ((static_cast<size_t>(kt) * 2 + 1) * R_pad + r) * 128 + (k0 & 127)) = pl;
          if ((lane & 15) == 0) {
            const int pos = s_pos[s];
            const int n = pos & 0xFF, rp = pos >> 8, n2 = rp + n;
            uint32_t* cw = sft + (static_cast<size_t>(s_tile[s]) * KT + kt) * 128;
            cw[(n & 31) * 4 + (n >> 5)] = wh;
            cw[(n2 & 31) * 4 + (n2 >> 5)] = wl;
          }
        }
      }
    }
    __syncthreads();  // s_row / s_pos / s_tile are rewritten for the next row
  }
}

// A warp per E4M3 exchange row: its codes go to packed row p = row_of[r] of
// the K-tile-major plane (one 128-byte line per K-tile, four 16-byte loads in
// flight per lane) and each block exponent, as act_quant_ref's scale word
// (the exponent in all four bytes), into the token tile's scale chunk: what
// rows_quant_kernel writes for the bf16 row in act_quant_ref mode.
constexpr int kPlaceWarps = 8;

__global__ void __launch_bounds__(kPlaceWarps * 32)
    rows_place_e4m3_kernel(const uint8_t* __restrict__ rows, int row_bytes, int R, const int* __restrict__ R_dev,
                           int H, const int* __restrict__ row_of, int R_pad, const int* __restrict__ row_tile,
                           const int* __restrict__ row_pos, uint8_t* __restrict__ xq, uint32_t* __restrict__ sft) {
  griddep_wait();  // the layout's row maps are visible
  griddep_launch();
  const int n = R_dev ? min(*R_dev, R) : R;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KT = H / 128, nv = H / 16;
  for (int r = blockIdx.x * kPlaceWarps + warp; r < n; r += gridDim.x * kPlaceWarps) {
    const int p = row_of[r];
    if (p < 0) continue;
    const uint8_t* row = rows + static_cast<size_t>(r) * row_bytes;
    const uint4* src = reinterpret_cast<const uint4*>(row);
    // 16-byte vector v holds K values [16v, 16v + 16): K-tile v / 8, line offset 16 (v % 8)
    uint8_t* dst = xq + static_cast<size_t>(p) * 128;
    const size_t plane = static_cast<size_t>(R_pad) * 128;
    int v = lane;
    for (; v + 96 < nv; v += 128) {
      const uint4 a = src[v], b = src[v + 32], c = src[v + 64], d = src[v + 96];
      *reinterpret_cast<uint4*>(dst + (v >> 3) * plane + (v & 7) * 16) = a;
      *reinterpret_cast<uint4*>(dst + ((v + 32) >> 3) * plane + (v & 7) * 16) = b;
      *reinterpret_cast<uint4*>(dst + ((v + 64) >> 3) * plane + (v & 7) * 16) = c;
      *reinterpret_cast<uint4*>(dst + ((v + 96) >> 3) * plane + (v & 7) * 16) = d;
    }
    for (; v < nv; v += 32) *reinterpret_cast<uint4*>(dst + (v >> 3) * plane + (v & 7) * 16) = src[v];
    const int tile = row_tile[p], pos = row_pos[p] & 0xFF;
    for (int kt = lane; kt < KT; kt += 32)
      sft[(static_cast<size_t>(tile) * KT + kt) * 128 + (pos & 31) * 4 + (pos >> 5)] =
          static_cast<uint32_t>(row[H + kt]) * 0x01010101u;
  }
}

// Unit rows (one per token and owning rank, K slots): a warp per unit reads
// each 16-byte code vector once and stores it to the packed row of every used
// slot (row_of[u * K + j] >= 0), then the slots' scale words; lane j also
// records slot j's return rank and position under its packed row, for the
// down GEMM's epilogue.
__global__ void __launch_bounds__(kPlaceWarps * 32)
    rows_place_units_kernel(const uint8_t* __restrict__ rows, int row_bytes, int U, const int* __restrict__ U_dev,
                            int H, int K, const int* __restrict__ row_of, const int* __restrict__ a_rank,
                            const int* __restrict__ a_pos, int R_pad, const int* __restrict__ row_tile,
                            const int* __restrict__ row_pos, uint8_t* __restrict__ xq, uint32_t* __restrict__ sft,
                            int* __restrict__ row_rank, int* __restrict__ row_ret) {
  griddep_wait();  // the layout's row maps are visible
  griddep_launch();
  const int n = U_dev ? min(*U_dev, U) : U;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KT = H / 128, nv = H / 16;
  const size_t plane = static_cast<size_t>(R_pad) * 128;
  for (int u = blockIdx.x * kPlaceWarps + warp; u < n; u += gridDim.x * kPlaceWarps) {
    int my_r = -1;
    if (lane < K) {
      my_r = row_of[static_cast<size_t>(u) * K + lane];
      if (my_r >= 0) {
        row_rank[my_r] = a_rank[static_cast<size_t>(u) * K + lane];
        row_ret[my_r] = a_pos[static_cast<size_t>(u) * K + lane];
      }
    }
    int r[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) r[j] = __shfl_sync(0xFFFFFFFFu, my_r, j);
    const uint8_t* row = rows + static_cast<size_t>(u) * row_bytes;
    const uint4* src = reinterpret_cast<const uint4*>(row);
    for (int v = lane; v < nv; v += 32) {
      const uint4 val = src[v];
      const size_t off = (v >> 3) * plane + (v & 7) * 16;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (j < K && r[j] >= 0) *reinterpret_cast<uint4*>(xq + static_cast<size_t>(r[j]) * 128 + off) = val;
    }
    for (int kt = lane; kt < KT; kt += 32) {
      const uint32_t word = static_cast<uint32_t>(row[H + kt]) * 0x01010101u;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (j < K && r[j] >= 0) {
          const int pos = row_pos[r[j]] & 0xFF;
          sft[(static_cast<size_t>(row_tile[r[j]]) * KT + kt) * 128 + (pos & 31) * 4 + (pos >> 5)] = word;
        }
      }
    }
  }
}

// act_quant_ref: grid (M, ceil(K / 1024)), 128 threads.
__global__ void __launch_bounds__(128) act_quant_kernel(const __nv_bfloat16* __restrict__ x, int M, int K,
                                                        uint8_t* __restrict__ q, float* __restrict__ scale) {
  const int m = blockIdx.x;
  const int lane = threadIdx.x & 31;
  const int k0 = blockIdx.y * 1024 + (threadIdx.x >> 5) * 256 + lane * 8;
  const bool valid = k0 < K;
  float v[8];
  if (valid) {
    load8_bf16(x + static_cast<size_t>(m) * K + k0, v);
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = 0.f;
  }
  uint8_t b[8];
  const int e = quant_block128(v, b);
  if (!valid) return;
  *reinterpret_cast<uint2*>(q + static_cast<size_t>(m) * K + k0) = pack8(b);
  if ((lane & 15) == 0) scale[static_cast<size_t>(m) * (K / 128) + k0 / 128] = exp2i(e);
}

// fp32 -> E2M1 code, round to nearest even, saturating at 6.0.
__device__ __forceinline__ uint32_t f32_to_e2m1(float v) {
  const uint32_t sign = (__float_as_uint(v) >> 28) & 0x8u;
  const float a = fabsf(v);
  uint32_t code;
  if (a >= 6.0f) {
    code = 7u;
  } else if (a < 1.0f) {
    // ulp(2^22) == 0.5: the fp32 add rounds a to the 0.5 grid (RNE)
    const float big = 4194304.0f;
    code = __float_as_uint(__fadd_rn(a, big)) - __float_as_uint(big);
  } else {
    const uint32_t b = __float_as_uint(a);
    const uint32_t odd = (b >> 22) & 1u;
    code = (b - (126u << 23) + ((1u << 21) - 1u) + odd) >> 22;
  }
  return (code & 0x7u) | sign;
}

// One thread per 32-element block of a row.
__global__ void pack_mxfp4_kernel(const float* __restrict__ w, int N, int K, uint8_t* __restrict__ packed,
                                  uint8_t* __restrict__ scale) {
  const size_t blk = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const size_t nblk = static_cast<size_t>(N) * (K / 32);
  if (blk >= nblk) return;
  const float* src = w + blk * 32;
  float v[32];
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float4 f = reinterpret_cast<const float4*>(src)[i];
    v[4 * i] = f.x;
    v[4 * i + 1] = f.y;
    v[4 * i + 2] = f.z;
    v[4 * i + 3] = f.w;
  }
  bool nan = false;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    amax = fmaxf(amax, fabsf(v[i]));
    nan |= isnan(v[i]);
  }
  int unb = static_cast<int>((__float_as_uint(amax) >> 23) & 0xFFu) - 127 - 2;
  unb = max(-127, min(128, unb));
  uint32_t sb = static_cast<uint32_t>(unb + 127);
  if (nan) sb = 255u;
  float sf = __uint_as_float(sb << 23);
  sf = fmaxf(sf, __uint_as_float(1u << 23));  // clamp to 2^-126
  uint32_t words[4] = {0u, 0u, 0u, 0u};
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const uint32_t c = f32_to_e2m1(__fdiv_rn(v[i], sf));
    words[i / 8] |= c << (4 * (i % 8));
  }
  *reinterpret_cast<uint4*>(packed + blk * 16) = make_uint4(words[0], words[1], words[2], words[3]);
  scale[blk] = static_cast<uint8_t>(sb);
}

// One thread per output byte of the chunked scale layout
// [n][row block][K-tile][half][512]; chunk byte (r%32)*16 + ((r%128)/32)*4 + kb
// holds row r (of the 128-row block), K32 block kb.
__global__ void prepack_scales_kernel(const uint8_t* __restrict__ in, int n_mats, int rows, int K, int halves,
                                      uint8_t* __restrict__ out) {
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int NB = rows / 128 / halves, KT = K / 128, KB = K / 32;
  const size_t total = static_cast<size_t>(n_mats) * (rows / 128) * KT * 512;
  if (i >= total) return;
  const int b = static_cast<int>(i % 512);
  size_t c = i / 512;
  const int h = static_cast<int>(c % halves);
  c /= halves;
  const int kt = static_cast<int>(c % KT);
  c /= KT;
  const int nb = static_cast<int>(c % NB);
  const int m = static_cast<int>(c / NB);
  const int r_local = (b >> 4) + 32 * ((b & 15) >> 2);
  const int kb = b & 3;
  const int row = h * (rows / halves) + nb * 128 + r_local;
  out[i] = in[(static_cast<size_t>(m) * rows + row) * KB + kt * 4 + kb];
}

// Weight re-layout: packed codes [n][rows][K/2] -> 8 KB tiles of 128 rows x 128
// values, [n][row block][K-tile][half][128][64 B], where with halves = 2 the
// matrix rows split into two halves (gate rows, up rows) whose tiles of the
// same row block and K-tile sit next to each other.  One thread per 16 bytes.
__global__ void repack_weights_kernel(const uint4* __restrict__ in, int n_mats, int rows, int K, int halves,
                                      uint4* __restrict__ out) {
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int NB = rows / 128 / halves, KT = K / 128;
  const size_t total = static_cast<size_t>(n_mats) * rows * (K / 32);  // 16-byte pieces
  if (i >= total) return;
  const int c = static_cast<int>(i & 3);             // piece in the 64-byte row segment
  size_t rest = i >> 2;
  const int r = static_cast<int>(rest % 128);
  rest /= 128;
  const int h = static_cast<int>(rest % halves);
  rest /= halves;
  const int kt = static_cast<int>(rest % KT);
  rest /= KT;
  const int nb = static_cast<int>(rest % NB);
  const int m = static_cast<int>(rest / NB);
  const int row = h * (rows / halves) + nb * 128 + r;
  const size_t src = ((static_cast<size_t>(m) * rows + row) * (K / 2) + kt * 64 + c * 16) / 16;
  out[i] = in[src];
}

}  // namespace

cudaError_t launch_repack_weights(const uint8_t* packed, int n_mats, int rows, int K, int halves, uint8_t* tiled,
                                  cudaStream_t stream) {
  const size_t total = static_cast<size_t>(n_mats) * rows * (K / 32);
  const int threads = 256;
  const unsigned grid = static_cast<unsigned>((total + threads - 1) / threads);
  repack_weights_kernel<<<grid, threads, 0, stream>>>(reinterpret_cast<const uint4*>(packed), n_mats, rows, K, halves,
                                                      reinterpret_cast<uint4*>(tiled));
  return cudaGetLastError();
}

cudaError_t launch_rows_quant(const void* x, int T, const int* T_dev, int H, int ldx, int k, const int* row_of,
                              int shared_base,
                              int hilo, int R_pad, const int* row_tile, const int* row_pos, uint8_t* xq,
                              uint32_t* sft, cudaStream_t stream) {
  if (H % 256 || k + (shared_base >= 0 ? 1 : 0) > kRqMaxRows) return cudaErrorInvalidValue;
  // a block per row, at most 8 per SM of 148 at once (the rest loop); below
  // that, up to one warp per 256-value chunk of a row
  const int gx = T < 1184 ? T : 1184;
  const int warps_per_row = kRqThreads / 32, chunks = H / 256;
  int gy = (1184 + gx - 1) / gx;
  const int gy_max = (chunks + warps_per_row - 1) / warps_per_row;
  if (gy > gy_max) gy = gy_max;
  const cudaError_t e = launch_k(rows_quant_kernel, dim3(gx, gy), dim3(kRqThreads), 0, stream,
                                 static_cast<const __nv_bfloat16*>(x), T, T_dev, H, ldx, k, row_of, shared_base, hilo,
                                 R_pad, row_tile, row_pos, xq, sft);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

cudaError_t launch_rows_place_e4m3(const void* rows, int row_bytes, int R, const int* R_dev, int H, const int* row_of,
                                   int R_pad, const int* row_tile, const int* row_pos, uint8_t* xq, uint32_t* sft,
                                   cudaStream_t stream) {
  if (R <= 0) return cudaSuccess;
  if (H % 128 || row_bytes % 16 || row_bytes < H + H / 128) return cudaErrorInvalidValue;
  int grid = (R + kPlaceWarps - 1) / kPlaceWarps;
  if (grid > 148 * 8) grid = 148 * 8;
  const cudaError_t e = launch_k(rows_place_e4m3_kernel, dim3(grid), dim3(kPlaceWarps * 32), 0, stream,
                                 static_cast<const uint8_t*>(rows), row_bytes, R, R_dev, H, row_of, R_pad, row_tile,
                                 row_pos, xq, sft);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

cudaError_t launch_rows_place_units(const void* rows, int row_bytes, int U, const int* U_dev, int H, int K,
                                    const int* row_of, const int* a_rank, const int* a_pos, int R_pad,
                                    const int* row_tile, const int* row_pos, uint8_t* xq, uint32_t* sft,
                                    int* row_rank, int* row_ret, cudaStream_t stream) {
  if (U <= 0) return cudaSuccess;
  if (H % 128 || row_bytes % 16 || K < 1 || K > 8) return cudaErrorInvalidValue;
  int grid = (U + kPlaceWarps - 1) / kPlaceWarps;
  if (grid > 148 * 8) grid = 148 * 8;
  const cudaError_t e = launch_k(rows_place_units_kernel, dim3(grid), dim3(kPlaceWarps * 32), 0, stream,
                                 static_cast<const uint8_t*>(rows), row_bytes, U, U_dev, H, K, row_of, a_rank, a_pos,
                                 R_pad, row_tile, row_pos, xq, sft, row_rank, row_ret);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

cudaError_t launch_act_quant(const void* x, int M, int K, uint8_t* q, float* scale, cudaStream_t stream) {
  dim3 grid(M, (K + 1023) / 1024);
  act_quant_kernel<<<grid, 128, 0, stream>>>(static_cast<const __nv_bfloat16*>(x), M, K, q, scale);
  return cudaGetLastError();
}

cudaError_t launch_pack_mxfp4(const float* w, int N, int K, uint8_t* packed, uint8_t* scale, cudaStream_t stream) {
  const size_t nblk = static_cast<size_t>(N) * (K / 32);
  const int threads = 256;
  const unsigned grid = static_cast<unsigned>((nblk + threads - 1) / threads);
  pack_mxfp4_kernel<<<grid, threads, 0, stream>>>(w, N, K, packed, scale);
  return cudaGetLastError();
}

cudaError_t launch_prepack_scales(const uint8_t* scale, int n_mats, int rows, int K, int halves, uint8_t* chunks,
                                  cudaStream_t stream) {
  const size_t total = static_cast<size_t>(n_mats) * (rows / 128) * (K / 128) * 512;
  const int threads = 256;
  const unsigned grid = static_cast<unsigned>((total + threads - 1) / threads);
  prepack_scales_kernel<<<grid, threads, 0, stream>>>(scale, n_mats, rows, K, halves, chunks);
  return cudaGetLastError();
}

}  // namespace mosaic
