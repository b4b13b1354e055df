// Assignment layout: histogram -> prefix scan -> stable scatter -> GEMM tile list.
//
// Reference behaviour: mosaicvm/kernels/moe_layout.py:8-27 (layout_assignments:
// bincount, cumsum offsets, a permutation that groups assignments by expert)
// and mosaicvm/kernels/w4a16_grouped.py:41-61,151-169 (emit_tiles: per-expert
// tiles (expert, m_start, rows), tile count kept on the device).  Inside an
// expert segment rows are ordered by flat assignment index (token-major), the
// stable order; the reference's argsort leaves that order unspecified.
//
// One CTA of 1024 threads does everything in shared memory, so the layer
// needs no host round trip.  Ranks inside a chunk of 1024 assignments come
// from per-warp bit masks (one bit per lane, per expert) and a scan over the
// 32 warps; chunks are processed in order and carry per-expert running bases.
// A token may name an expert more than once (the reference's gather-based
// path allows it): each assignment still gets a row of its own.
#include "common.cuh"
#include "kernels.h"

namespace mosaic {

namespace {

// Exclusive scan of n ints by warp 0 (n small); out[n] receives the total.
__device__ void warp0_exclusive_scan(const int* in, int* out, int n) {
  if (threadIdx.x >= 32) return;
  const int lane = threadIdx.x;
  int carry = 0;
  for (int b = 0; b < n; b += 32) {
    const int i = b + lane;
    int v = (i < n) ? in[i] : 0;
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
      if (lane >= o) incl += y;
    }
    if (i < n) out[i] = carry + incl - v;
    carry += __shfl_sync(0xFFFFFFFFu, incl, 31);
  }
  if (lane == 0) out[n] = carry;
}

struct LayoutExtra {
  int64_t* perm;        // optional: packed row -> flat assignment index
  int64_t* sorted_ids;  // optional: packed row -> expert id
};

__global__ void __launch_bounds__(1024) layout_kernel(LayoutParams p, LayoutExtra x) {
  griddep_wait();  // the previous kernel of the chain has finished
  griddep_launch();
  extern __shared__ int sm[];
  const int E = p.E, k = p.k;
  const int T = p.T_dev ? max(0, min(*p.T_dev, p.T)) : p.T;  // device-side count (EP receive side)
  const int NE = E + (p.with_shared ? 1 : 0);
  int* hist = sm;                      // NE
  int* offs = hist + NE;               // NE + 1
  int* base = offs + NE + 1;           // E
  int* ntile = base + E;               // NE
  int* toff = ntile + NE;              // NE + 1
  unsigned* masks = reinterpret_cast<unsigned*>(toff + NE + 1);  // 32 * E
  int* pre = reinterpret_cast<int*>(masks + 32 * E);             // 32 * E
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  for (int i = tid; i < NE; i += 1024) hist[i] = 0;
  for (int i = tid; i < E; i += 1024) base[i] = 0;
  __syncthreads();
  const int A = T * k;
  for (int a = tid; a < A; a += 1024) {
    const int64_t e = p.idx[a];
    if (e < 0 || e >= E) {
      if (!(p.pad_ok && e < 0)) set_error(p.err, MOSAIC_ERR_RANGE);
      continue;
    }
    atomicAdd(&hist[static_cast<int>(e)], 1);
  }
  __syncthreads();
  if (tid == 0 && p.with_shared) hist[E] = T;
  __syncthreads();
  warp0_exclusive_scan(hist, offs, NE);
  for (int i = tid; i < NE; i += 1024) {
    const int tt = (p.with_shared && i == E) ? p.tt_shared : p.tt_routed;
    ntile[i] = (tt > 0) ? (hist[i] + tt - 1) / tt : 0;
  }
  __syncthreads();
  warp0_exclusive_scan(ntile, toff, NE);
  __syncthreads();

  // Ranks: 1024 assignments per chunk in flat (token-major, slot-minor) order.
  // One bit per lane per expert marks the chunk's assignments; a token that
  // names an expert twice (hash tables may) simply has two bits, so every
  // assignment gets its own row and the order inside an expert stays the flat
  // index order.
  for (int c0 = 0; c0 < A; c0 += 1024) {
    const int a = c0 + tid;
    for (int i = tid; i < 32 * E; i += 1024) masks[i] = 0u;
    __syncthreads();
    int e = -1;
    if (a < A) {
      const int64_t v = p.idx[a];
      if (v >= 0 && v < E) {
        e = static_cast<int>(v);
        atomicOr(&masks[warp * E + e], 1u << lane);
      }
    }
    __syncthreads();
    for (int ex = tid; ex < E; ex += 1024) {
      int run = base[ex];
      for (int w = 0; w < 32; ++w) {
        pre[w * E + ex] = run;
        run += __popc(masks[w * E + ex]);
      }
      base[ex] = run;
    }
    __syncthreads();
    if (a < A) {
      int row = -1;
      if (e >= 0) {
        const int t = a / k;
        const unsigned lt = (1u << lane) - 1u;
        const int rank = pre[warp * E + e] + __popc(masks[warp * E + e] & lt);
        row = offs[e] + rank;
        if (p.row_token) p.row_token[row] = t;
        if (p.row_tile) {
          const int tt = p.tt_routed;
          const int ti = rank / tt;
          const int rows_t = min(tt, hist[e] - ti * tt);
          p.row_tile[row] = toff[e] + ti;
          p.row_pos[row] = ((p.rpad_to_tile ? tt : (rows_t + 15) & ~15) << 8) | (rank - ti * tt);
        }
        if (p.row_weight) p.row_weight[row] = p.weights ? p.weights[a] : 1.0f;
        if (x.perm) x.perm[row] = a;
        if (x.sorted_ids) x.sorted_ids[row] = e;
      }
      if (p.row_of) p.row_of[a] = row;
    }
    __syncthreads();
  }
  // Per token, its rows in ascending expert id (the combine order); equal ids
  // (repeated by a hash table) hold equal partials, so their order is free.
  if (p.row_sorted && p.row_of) {
    for (int t = tid; t < T; t += 1024) {
      int ke[8], kr[8];
#pragma unroll
      for (int s = 0; s < 8; ++s) {
        ke[s] = 0x7FFFFFFF;
        kr[s] = 0;
        if (s < k) {
          const int64_t v = p.idx[static_cast<size_t>(t) * k + s];
          ke[s] = (v >= 0 && v < E) ? static_cast<int>(v) : -1;
          kr[s] = p.row_of[static_cast<size_t>(t) * k + s];
        }
      }
      for (int i = 1; i < k; ++i) {
        const int ce = ke[i], cr = kr[i];
        int j = i - 1;
        while (j >= 0 && ke[j] > ce) {
          ke[j + 1] = ke[j];
          kr[j + 1] = kr[j];
          --j;
        }
        ke[j + 1] = ce;
        kr[j + 1] = cr;
      }
      for (int s = 0; s < k; ++s) p.row_sorted[static_cast<size_t>(t) * k + s] = kr[s];
    }
    __syncthreads();
  }
  if (p.with_shared && p.row_token && p.row_weight) {
    for (int t = tid; t < T; t += 1024) {
      const int row = offs[E] + t;
      p.row_token[row] = t;
      p.row_weight[row] = 1.0f;
      if (p.row_tile) {
        const int tt = p.tt_shared;
        const int ti = t / tt;
        const int rows_t = min(tt, T - ti * tt);
        p.row_tile[row] = toff[E] + ti;
        p.row_pos[row] = ((p.rpad_to_tile ? tt : (rows_t + 15) & ~15) << 8) | (t - ti * tt);
      }
    }
  }
  for (int i = tid; i < NE; i += 1024)
    if (p.counts) p.counts[i] = hist[i];
  for (int i = tid; i <= NE; i += 1024)
    if (p.offsets) p.offsets[i] = offs[i];
  if (p.tiles) {
    for (int e = tid; e < NE; e += 1024) {
      const int tt = (p.with_shared && e == E) ? p.tt_shared : p.tt_routed;
      for (int i = 0; i < ntile[e]; ++i) {
        const int j = toff[e] + i;
        if (j < p.max_tiles) {
          p.tiles[3 * j + 0] = e;
          p.tiles[3 * j + 1] = offs[e] + i * tt;
          p.tiles[3 * j + 2] = min(tt, hist[e] - i * tt);
        }
      }
    }
    if (tid == 0) {
      *p.n_tiles = toff[NE];
      if (toff[NE] > p.max_tiles) set_error(p.err, MOSAIC_ERR_WORKSPACE);
    }
  }
}

// ---- multi-CTA layout for large batches (more than one chunk of 1024 assignments).
// The single-CTA kernel above walks the chunks one after another; here each
// chunk is a CTA: (1) count its assignments per expert, (2) one CTA scans the
// counts over chunks (per expert) and over experts and writes the tile list,
// (3) each chunk ranks its assignments from its chunk base, (4) per token: the
// combine order and the shared expert's rows.  Ranks are those of the
// single-CTA kernel: stable by flat assignment index inside each expert.
struct LayoutScratch {
  int* chunk;  // [nchunks][E]: counts, then exclusive chunk bases
  int* hist;   // [NE]
  int* offs;   // [NE + 1]
  int* toff;   // [NE + 1]
};

__device__ __forceinline__ LayoutScratch scratch_of(const LayoutParams& p, int nchunks) {
  const int NE = p.E + (p.with_shared ? 1 : 0);
  LayoutScratch s;
  s.chunk = p.scratch;
  s.hist = p.scratch + static_cast<size_t>(nchunks) * p.E;
  s.offs = s.hist + NE;
  s.toff = s.offs + NE + 1;
  return s;
}

__global__ void __launch_bounds__(1024) layout_count_kernel(LayoutParams p, int nchunks) {
  griddep_wait();  // the previous kernel of the chain has finished
  griddep_launch();
  __shared__ int cnt[260];  // E <= 257 (the per-row pass counts the shared expert as an id)
  const int E = p.E, k = p.k, tid = threadIdx.x, c = blockIdx.x;
  const int T = p.T_dev ? max(0, min(*p.T_dev, p.T)) : p.T;
  const int A = T * k;
  const LayoutScratch sc = scratch_of(p, nchunks);
  for (int e = tid; e < E; e += 1024) cnt[e] = 0;
  __syncthreads();
  const int a = c * 1024 + tid;
  if (a < A) {
    const int64_t v = p.idx[a];
    if (v >= 0 && v < E) {
      atomicAdd(&cnt[static_cast<int>(v)], 1);
    } else if (!(p.pad_ok && v < 0)) {
      set_error(p.err, MOSAIC_ERR_RANGE);
    }
  }
  __syncthreads();
  for (int e = tid; e < E; e += 1024) sc.chunk[static_cast<size_t>(c) * E + e] = cnt[e];
}

__global__ void __launch_bounds__(1024) layout_scan_kernel(LayoutParams p, int nchunks) {
  griddep_wait();  // the previous kernel of the chain has finished
  griddep_launch();
  extern __shared__ int sm[];
  const int E = p.E, tid = threadIdx.x;
  const int T = p.T_dev ? max(0, min(*p.T_dev, p.T)) : p.T;
  const int NE = E + (p.with_shared ? 1 : 0);
  const LayoutScratch sc = scratch_of(p, nchunks);
  int* hist = sm;           // NE
  int* offs = hist + NE;    // NE + 1
  int* ntile = offs + NE + 1;  // NE
  int* toff = ntile + NE;   // NE + 1
  for (int e = tid; e < E; e += 1024) {
    int run = 0;
    for (int c = 0; c < nchunks; ++c) {
      int* q = sc.chunk + static_cast<size_t>(c) * E + e;
      const int v = *q;
      *q = run;
      run += v;
    }
    hist[e] = run;
  }
  if (tid == 0 && p.with_shared) hist[E] = T;
  __syncthreads();
  warp0_exclusive_scan(hist, offs, NE);
  for (int i = tid; i < NE; i += 1024) {
    const int tt = (p.with_shared && i == E) ? p.tt_shared : p.tt_routed;
    ntile[i] = (tt > 0) ? (hist[i] + tt - 1) / tt : 0;
  }
  __syncthreads();
  warp0_exclusive_scan(ntile, toff, NE);
  __syncthreads();
  for (int i = tid; i < NE; i += 1024) {
    sc.hist[i] = hist[i];
    if (p.counts) p.counts[i] = hist[i];
  }
  for (int i = tid; i <= NE; i += 1024) {
    sc.offs[i] = offs[i];
    sc.toff[i] = toff[i];
    if (p.offsets) p.offsets[i] = offs[i];
  }
  if (p.tiles) {
    for (int e = tid; e < NE; e += 1024) {
      const int tt = (p.with_shared && e == E) ? p.tt_shared : p.tt_routed;
      for (int i = 0; i < ntile[e]; ++i) {
        const int j = toff[e] + i;
        if (j < p.max_tiles) {
          p.tiles[3 * j + 0] = e;
          p.tiles[3 * j + 1] = offs[e] + i * tt;
          p.tiles[3 * j + 2] = min(tt, hist[e] - i * tt);
        }
      }
    }
    if (tid == 0) {
      *p.n_tiles = toff[NE];
      if (toff[NE] > p.max_tiles) set_error(p.err, MOSAIC_ERR_WORKSPACE);
    }
  }
}

__global__ void __launch_bounds__(1024) layout_rank_kernel(LayoutParams p, int nchunks, LayoutExtra x) {
  griddep_wait();  // the previous kernel of the chain has finished
  griddep_launch();
  extern __shared__ int sm[];
  const int E = p.E, k = p.k, c = blockIdx.x;
  const int T = p.T_dev ? max(0, min(*p.T_dev, p.T)) : p.T;
  const int A = T * k;
  if (c * 1024 >= A) return;
  const LayoutScratch sc = scratch_of(p, nchunks);
  unsigned* masks = reinterpret_cast<unsigned*>(sm);         // 32 * E
  int* pre = reinterpret_cast<int*>(masks + 32 * E);          // 32 * E
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int i = tid; i < 32 * E; i += 1024) masks[i] = 0u;
  __syncthreads();
  const int a = c * 1024 + tid;
  int e = -1;
  if (a < A) {
    const int64_t v = p.idx[a];
    if (v >= 0 && v < E) {
      e = static_cast<int>(v);
      atomicOr(&masks[warp * E + e], 1u << lane);
    }
  }
  __syncthreads();
  for (int ex = tid; ex < E; ex += 1024) {
    int run = sc.chunk[static_cast<size_t>(c) * E + ex];
    for (int w = 0; w < 32; ++w) {
      pre[w * E + ex] = run;
      run += __popc(masks[w * E + ex]);
    }
  }
  __syncthreads();
  if (a < A) {
    int row = -1;
    if (e >= 0) {
      const unsigned lt = (1u << lane) - 1u;
      const int rank = pre[warp * E + e] + __popc(masks[warp * E + e] & lt);
      row = sc.offs[e] + rank;
      if (p.row_token) p.row_token[row] = a / k;
      if (p.row_tile) {
        const int tt = p.tt_routed;
        const int ti = rank / tt;
        const int rows_t = min(tt, sc.hist[e] - ti * tt);
        p.row_tile[row] = sc.toff[e] + ti;
        p.row_pos[row] = ((p.rpad_to_tile ? tt : (rows_t + 15) & ~15) << 8) | (rank - ti * tt);
      }
      if (p.row_weight) p.row_weight[row] = p.weights ? p.weights[a] : 1.0f;
      if (x.perm) x.perm[row] = a;
      if (x.sorted_ids) x.sorted_ids[row] = e;
    }
    if (p.row_of) p.row_of[a] = row;
  }
}

__global__ void __launch_bounds__(256) layout_finish_kernel(LayoutParams p, int nchunks) {
  griddep_wait();  // the previous kernel of the chain has finished
  griddep_launch();
  const int E = p.E, k = p.k;
  const int T = p.T_dev ? max(0, min(*p.T_dev, p.T)) : p.T;
  const LayoutScratch sc = scratch_of(p, nchunks);
  for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < T; t += gridDim.x * blockDim.x) {
    if (p.row_sorted && p.row_of) {
      int ke[8], kr[8];
#pragma unroll
      for (int s = 0; s < 8; ++s) {
        ke[s] = 0x7FFFFFFF;
        kr[s] = 0;
        if (s < k) {
          const int64_t v = p.idx[static_cast<size_t>(t) * k + s];
          ke[s] = (v >= 0 && v < E) ? static_cast<int>(v) : -1;
          kr[s] = p.row_of[static_cast<size_t>(t) * k + s];
        }
      }
      for (int i = 1; i < k; ++i) {
        const int ce = ke[i], cr = kr[i];
        int j = i - 1;
        while (j >= 0 && ke[j] > ce) {
          ke[j + 1] = ke[j];
          kr[j + 1] = kr[j];
          --j;
        }
        ke[j + 1] = ce;
        kr[j + 1] = cr;
      }
      for (int s = 0; s < k; ++s) p.row_sorted[static_cast<size_t>(t) * k + s] = kr[s];
    }
    if (p.with_shared && p.row_token && p.row_weight) {
      const int row = sc.offs[E] + t;
      p.row_token[row] = t;
      p.row_weight[row] = 1.0f;
      if (p.row_tile) {
        const int tt = p.tt_shared;
        const int ti = t / tt;
        const int rows_t = min(tt, T - ti * tt);
        p.row_tile[row] = sc.toff[E] + ti;
        p.row_pos[row] = ((p.rpad_to_tile ? tt : (rows_t + 15) & ~15) << 8) | (t - ti * tt);
      }
    }
  }
}

size_t layout_smem(int E, int with_shared) {
  const int NE = E + (with_shared ? 1 : 0);
  return sizeof(int) * (static_cast<size_t>(NE) * 4 + 2 + E + 64 * static_cast<size_t>(E));
}

__global__ void emit_tiles_kernel(const int32_t* counts, int E, int block_m, int max_tiles, int32_t* expert_index,
                                  int32_t* m_start, int32_t* n_tiles, int32_t* tile_rows) {
  extern __shared__ int sm[];
  int* nt = sm;
  int* off = sm + E;
  for (int e = threadIdx.x; e < E; e += blockDim.x) nt[e] = (counts[e] + block_m - 1) / block_m;
  __syncthreads();
  warp0_exclusive_scan(nt, off, E);
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    const int c = counts[e];
    for (int i = 0; i < nt[e]; ++i) {
      const int j = off[e] + i;
      if (j < max_tiles) {
        expert_index[j] = e;
        m_start[j] = i * block_m;
        tile_rows[j] = min(block_m, c - i * block_m);
      }
    }
  }
  if (threadIdx.x == 0) *n_tiles = off[E];
}

}  // namespace

size_t layout_scratch_ints(int T, int k, int E) {
  const int nchunks = (T * k + 1023) / 1024;
  return nchunks > 1 ? static_cast<size_t>(nchunks) * E + 3 * static_cast<size_t>(E + 3) : 0;
}

cudaError_t launch_layout(const LayoutParams& p, cudaStream_t stream) {
  const int nchunks = (p.T * p.k + 1023) / 1024;
  cudaError_t e = cudaSuccess;
  if (nchunks > 1 && p.scratch) {
    const int NE = p.E + (p.with_shared ? 1 : 0);
    e = launch_k(layout_count_kernel, dim3(nchunks), dim3(1024), 0, stream, p, nchunks);
    if (e != cudaSuccess) return e;
    e = launch_k(layout_scan_kernel, dim3(1), dim3(1024), sizeof(int) * (4 * NE + 2), stream, p, nchunks);
    if (e != cudaSuccess) return e;
    const size_t rsmem = sizeof(int) * 64 * static_cast<size_t>(p.E);
    e = cudaFuncSetAttribute(layout_rank_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(rsmem));
    if (e != cudaSuccess) return e;
    e = launch_k(layout_rank_kernel, dim3(nchunks), dim3(1024), rsmem, stream, p, nchunks,
                 LayoutExtra{nullptr, nullptr});
    if (e != cudaSuccess) return e;
    const int fb = (p.T + 255) / 256;
    e = launch_k(layout_finish_kernel, dim3(fb < 1184 ? fb : 1184), dim3(256), 0, stream, p, nchunks);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
  }
  const size_t smem = layout_smem(p.E, p.with_shared);
  e = cudaFuncSetAttribute(layout_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  e = launch_k(layout_kernel, dim3(1), dim3(1024), smem, stream, p, LayoutExtra{nullptr, nullptr});
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

cudaError_t launch_layout_assignments(const int64_t* ids, int A, int E, int64_t* sorted_ids, int64_t* perm,
                                      int32_t* offsets, int32_t* counts, cudaStream_t stream) {
  LayoutParams p{};
  p.idx = ids;
  p.weights = nullptr;
  p.T = A;
  p.k = 1;
  p.E = E;
  p.with_shared = 0;
  p.counts = counts;
  p.offsets = offsets;
  p.row_token = nullptr;
  p.row_weight = nullptr;
  p.row_of = nullptr;
  p.row_sorted = nullptr;
  p.tiles = nullptr;
  p.n_tiles = nullptr;
  p.err = nullptr;
  const size_t smem = layout_smem(E, 0);
  cudaError_t err = cudaFuncSetAttribute(layout_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
  if (err != cudaSuccess) return err;
  layout_kernel<<<1, 1024, smem, stream>>>(p, LayoutExtra{perm, sorted_ids});
  return cudaGetLastError();
}

cudaError_t launch_emit_tiles(const int32_t* counts, int E, int block_m, int max_tiles, int32_t* expert_index,
                              int32_t* m_start, int32_t* n_tiles, int32_t* tile_rows, cudaStream_t stream) {
  emit_tiles_kernel<<<1, 256, sizeof(int) * (2 * E + 1), stream>>>(counts, E, block_m, max_tiles, expert_index,
                                                                  m_start, n_tiles, tile_rows);
  return cudaGetLastError();
}

}  // namespace mosaic
