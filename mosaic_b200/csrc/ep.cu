// Expert-parallel dispatch helpers.
//
// Experts are sharded by contiguous ranges: rank d owns experts
// [d*E_local, (d+1)*E_local) (the expert-sharded MoE of
// .mosaicvm/source/inference_model.py:620-627).  The source rank sorts its
// assignments by expert id with the layout kernel, which also groups them by
// destination rank, and ep_pack_kernel gathers the token rows into send rows in
// that order.  The owning rank computes one partial per received row and
// returns the partials in the order it received them, so the source combines
// them in ascending expert id exactly as the single-GPU layer does.
#include "common.cuh"
#include "kernels.h"

namespace mosaic {

namespace {

constexpr int kPackWarps = 8;

// One warp copies one row of n 16-byte vectors, four loads in flight per lane
// (a copy loop with one load per store waits out a load latency per vector).
__device__ __forceinline__ void warp_copy_row(uint4* __restrict__ dst, const uint4* __restrict__ src, int n, int lane) {
  int c = lane;
  for (; c + 96 < n; c += 128) {
    const uint4 a = src[c], b = src[c + 32], d = src[c + 64], e = src[c + 96];
    dst[c] = a;
    dst[c + 32] = b;
    dst[c + 64] = d;
    dst[c + 96] = e;
  }
  for (; c < n; c += 32) dst[c] = src[c];
}


// One warp per send row: 16-byte vector copies of the token row, then the tail.
__global__ void __launch_bounds__(kPackWarps * 32) ep_pack_kernel(const uint4* __restrict__ x, int H, int A, int E,
                                                                  int E_local, const int* __restrict__ offsets,
                                                                  const int* __restrict__ row_token,
                                                                  const float* __restrict__ row_weight,
                                                                  uint4* __restrict__ send) {
  __shared__ int off_s[257];
  for (int i = threadIdx.x; i <= E; i += blockDim.x) off_s[i] = offsets[i];
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int vec_per_row = H / 8;           // 16-byte vectors of token values
  const int stride_vec = vec_per_row + 1;  // + the 16-byte tail
  // Assignments with an out-of-range expert id got no row (the layout records
  // the error), so the valid rows end at offsets[E] <= A.
  const int rows = min(A, off_s[E]);
  for (int r = blockIdx.x * kPackWarps + warp; r < rows; r += gridDim.x * kPackWarps) {
    const int t = row_token[r];
    const uint4* src = x + static_cast<size_t>(t) * vec_per_row;
    uint4* dst = send + static_cast<size_t>(r) * stride_vec;
    warp_copy_row(dst, src, vec_per_row, lane);
    if (lane == 0) {
      // expert of sorted row r: the last e with offsets[e] <= r
      int lo = 0, hi = E;  // invariant: offsets[lo] <= r < offsets[hi]
      while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (off_s[mid] <= r)
          lo = mid;
        else
          hi = mid;
      }
      const int dest = lo / E_local;
      uint4 tail;
      tail.x = static_cast<uint32_t>(lo - dest * E_local);
      tail.y = __float_as_uint(row_weight[r]);
      tail.z = static_cast<uint32_t>(t);
      tail.w = static_cast<uint32_t>(dest);
      dst[vec_per_row] = tail;
    }
  }
}

__global__ void ep_dest_counts_kernel(const int* __restrict__ offsets, int E_local, int world, int* dest_counts) {
  const int d = blockIdx.x * blockDim.x + threadIdx.x;
  if (d < world) dest_counts[d] = offsets[(d + 1) * E_local] - offsets[d * E_local];
}

__global__ void rows_meta_kernel(const int32_t* __restrict__ ids, const float* __restrict__ weights, int stride, int R,
                                 const int* __restrict__ rows_dev, int E, int default_id, int64_t* __restrict__ idx,
                                 float* __restrict__ w, int* err) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= R || (rows_dev && r >= *rows_dev)) return;
  int e = ids ? ids[static_cast<size_t>(r) * stride] : default_id;
  float wt = weights ? weights[static_cast<size_t>(r) * stride] : 1.0f;
  if (e < 0 || e >= E) {
    set_error(err, MOSAIC_ERR_RANGE);
    e = 0;
    wt = 0.f;
  }
  idx[r] = e;
  w[r] = wt;
}

// ------------------------------------------------- peer-memory exchange ---
// Rank r's region holds rows and partials that other ranks write with plain
// stores through their CUDA IPC mapping of it (NVLink peer memory).  A writer
// makes its stores visible (fence at system scope) before it stamps the
// reader's flag with the step's epoch (release); the reader waits on its own
// flags (acquire).  Waits are bounded; a timeout records MOSAIC_ERR_TIMEOUT in
// the waiting rank's region and the kernel returns.

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// true once *flag has reached epoch (epochs only grow; the signed difference
// handles wrap-around); false after budget_ns of the global timer
__device__ __forceinline__ bool wait_epoch(const uint32_t* flag, uint32_t epoch, unsigned long long budget_ns) {
  if (static_cast<int>(ld_acquire_sys(flag) - epoch) >= 0) return true;
  const unsigned long long t0 = global_ns();
  while (static_cast<int>(ld_acquire_sys(flag) - epoch) < 0) {
    if (global_ns() - t0 > budget_ns) return false;
    __nanosleep(64);
  }
  return true;
}

__device__ __forceinline__ EpRegionHeader* hdr_of(const EpPeersDev& P, int r) {
  return reinterpret_cast<EpRegionHeader*>(P.regions[r]);
}

// One CTA: start a step (epoch + 1), publish this rank's row counts to every
// rank, wait for every rank's counts, record the rows this rank receives.
__global__ void ep_counts_kernel(const EpPeersDev P, const int* __restrict__ dest_counts) {
  __shared__ uint32_t epoch;
  EpRegionHeader* own = hdr_of(P, P.rank);
  if (threadIdx.x == 0) {
    epoch = own->epoch + 1;
    own->epoch = epoch;
  }
  __syncthreads();
  const int p = threadIdx.x;
  if (p < P.world) {
    EpRegionHeader* ph = hdr_of(P, p);
    for (int d = 0; d < P.world; ++d) ph->counts[P.rank][d] = dest_counts[d];
    __threadfence_system();
    st_release_sys(&ph->count_flag[P.rank], epoch);
  }
  __syncthreads();
  if (p < P.world && !wait_epoch(&own->count_flag[p], epoch, P.wait_ns)) set_error(&own->err, MOSAIC_ERR_TIMEOUT);
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    int total = 0;
    for (int s = 0; s < P.world; ++s) {
      own->recv_start[s] = total;
      int pos = 0;
      for (int d = 0; d < P.rank; ++d) pos += own->counts[s][d];
      own->src_pos[s] = pos;
      total += own->counts[s][P.rank];
    }
    own->recv_start[P.world] = total;
    if (total > P.max_recv_rows) set_error(&own->err, MOSAIC_ERR_WORKSPACE);
    own->recv_count = min(total, P.max_recv_rows);
  }
}

// Count-matrix geometry of a step, from this rank's copy of the matrix.
struct EpGeom {
  int send_start[MOSAIC_EP_MAX_WORLD + 1];  // this rank's send rows for destination d start here
  int dest_off[MOSAIC_EP_MAX_WORLD];        // ... and land at this receive row of d
  int recv_start[MOSAIC_EP_MAX_WORLD + 1];  // rows received from source s start here
  int src_pos[MOSAIC_EP_MAX_WORLD];         // ... and sit at this send row of s
  bool fits[MOSAIC_EP_MAX_WORLD];           // destination d's receive buffer holds its rows
};

__device__ __forceinline__ void ep_geometry(const EpPeersDev& P, const EpRegionHeader* own, EpGeom& g) {
  const int W = P.world, me = P.rank;
  g.send_start[0] = 0;
  g.recv_start[0] = 0;
  for (int d = 0; d < W; ++d) {
    g.send_start[d + 1] = g.send_start[d] + own->counts[me][d];
    g.recv_start[d + 1] = g.recv_start[d] + own->counts[d][me];
    int off = 0, tot = 0;
    for (int s = 0; s < W; ++s) {
      if (s < me) off += own->counts[s][d];
      tot += own->counts[s][d];
    }
    g.dest_off[d] = off;
    g.fits[d] = tot <= P.max_recv_rows;
    int pos = 0;
    for (int dd = 0; dd < me; ++dd) pos += own->counts[d][dd];
    g.src_pos[d] = pos;  // for d as a source: its send rows for this rank start here
  }
}

// Grid-stride copy of this rank's send rows into the owners' receive buffers;
// the last CTA to finish stamps every owner's data flag.
__global__ void __launch_bounds__(256) ep_send_kernel(const EpPeersDev P, const uint4* __restrict__ send) {
  __shared__ EpGeom g;
  EpRegionHeader* own = hdr_of(P, P.rank);
  if (threadIdx.x == 0) ep_geometry(P, own, g);
  __syncthreads();
  const uint32_t epoch = own->epoch;
  const int cpr = P.row_bytes / 16;
  const int rows = g.send_start[P.world];
  const int lane = threadIdx.x & 31;
  const int nwarps = gridDim.x * (blockDim.x >> 5);
  // a warp per row: the row's destination once, then the row's vectors
  for (int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += nwarps) {
    int d = 0;
    while (r >= g.send_start[d + 1]) ++d;
    if (!g.fits[d]) continue;
    uint4* dst = reinterpret_cast<uint4*>(P.regions[d] + P.recv_off) +
                 static_cast<size_t>(g.dest_off[d] + r - g.send_start[d]) * cpr;
    warp_copy_row(dst, send + static_cast<size_t>(r) * cpr, cpr, lane);
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    if (atomicAdd(&own->send_done, 1u) == gridDim.x - 1) {
      own->send_done = 0;
      __threadfence_system();
      for (int d = 0; d < P.world; ++d) st_release_sys(&hdr_of(P, d)->data_flag[P.rank], epoch);
    }
  }
}

// Grid-stride copy of the partial of every received row back to its source's
// return buffer; the last CTA stamps every source's return flag.
__global__ void __launch_bounds__(256) ep_return_kernel(const EpPeersDev P, const uint4* __restrict__ partials) {
  __shared__ EpGeom g;
  EpRegionHeader* own = hdr_of(P, P.rank);
  if (threadIdx.x == 0) ep_geometry(P, own, g);
  __syncthreads();
  const uint32_t epoch = own->epoch;
  const int cpr = P.ret_row_bytes / 16;
  const int rows = own->recv_count;
  const int lane = threadIdx.x & 31;
  const int nwarps = gridDim.x * (blockDim.x >> 5);
  for (int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += nwarps) {
    int s = 0;
    while (r >= g.recv_start[s + 1]) ++s;
    uint4* dst = reinterpret_cast<uint4*>(P.regions[s] + P.ret_off) +
                 static_cast<size_t>(g.src_pos[s] + r - g.recv_start[s]) * cpr;
    warp_copy_row(dst, partials + static_cast<size_t>(r) * cpr, cpr, lane);
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    if (atomicAdd(&own->ret_done, 1u) == gridDim.x - 1) {
      own->ret_done = 0;
      __threadfence_system();
      for (int s = 0; s < P.world; ++s) st_release_sys(&hdr_of(P, s)->ret_flag[P.rank], epoch);
    }
  }
}

// ----------------------------------------------------------- E4M3 rows ---
// Each token row is quantised once per 128-value block (act_quant_ref, 8 lanes
// x 16 values per block, 512 values per warp pass, two passes per loop trip)
// into an L2-resident scratch row: codes, then the block exponents (collected
// in shared memory).  The send then copies a token's row into the owner's
// receive row for every assignment of the token and adds the meta tail
// {local expert, route weight bits, token, owner}.  No send buffer of
// assignment rows is written.
constexpr int kSendWarps = 8;
constexpr int kMaxKtPad = 128;  // H <= 16384

__device__ __forceinline__ void quant_pass(uint8_t* __restrict__ dst, uint8_t* __restrict__ exps, int k0, bool in,
                                           const float (&v)[16]) {
  uint8_t q[16];
  const int e = quant_block128_x16(v, q);  // every lane takes part in the block shuffles
  if (in) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
      w[i] = q[4 * i] | (q[4 * i + 1] << 8) | (q[4 * i + 2] << 16) | (static_cast<uint32_t>(q[4 * i + 3]) << 24);
    *reinterpret_cast<uint4*>(dst + k0) = make_uint4(w[0], w[1], w[2], w[3]);
    if ((threadIdx.x & 7) == 0) exps[k0 >> 7] = static_cast<uint8_t>((e + 127) & 0xFF);
  }
}

__device__ __forceinline__ void load16_bf16(const __nv_bfloat16* __restrict__ p, bool in, float (&v)[16]) {
  if (in) {
    float a[8], b[8];
    load8_bf16(p, a);
    load8_bf16(p + 8, b);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      v[i] = a[i];
      v[8 + i] = b[i];
    }
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = 0.f;
  }
}

// E4M3 rows quantised once per token: tq[t] = codes [H] | exponents [kt_pad]
// (row stride H + kt_pad, 16-byte aligned), a warp per token.
__global__ void __launch_bounds__(kSendWarps * 32)
    ep_tokens_e4m3_kernel(const __nv_bfloat16* __restrict__ x, int T, int H, uint8_t* __restrict__ tq) {
  __shared__ __align__(16) uint8_t exps_s[kSendWarps][kMaxKtPad];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KT = H / 128, kt_pad = (KT + 15) & ~15, stride = H + kt_pad;
  uint8_t* exps = exps_s[warp];
  for (int t = blockIdx.x * kSendWarps + warp; t < T; t += gridDim.x * kSendWarps) {
    const __nv_bfloat16* src = x + static_cast<size_t>(t) * H;
    uint8_t* dst = tq + static_cast<size_t>(t) * stride;
    for (int base = 0; base < H; base += 1024) {
      const int k0 = base + lane * 16, k1 = k0 + 512;
      float v0[16], v1[16];
      load16_bf16(src + k0, k0 < H, v0);
      load16_bf16(src + k1, k1 < H, v1);
      quant_pass(dst, exps, k0, k0 < H, v0);
      quant_pass(dst, exps, k1, k1 < H, v1);
    }
    for (int i = KT + lane; i < kt_pad; i += 32) exps[i] = 0;
    __syncwarp();
    if (lane < kt_pad / 16) reinterpret_cast<uint4*>(dst + H)[lane] = reinterpret_cast<const uint4*>(exps)[lane];
    __syncwarp();  // exps is rewritten by the next token
  }
}

// The owners' receive rows from the token rows of ep_tokens_e4m3_kernel: each
// warp owns a shared-memory row buffer; per send row, lane 0 bulk-loads the
// token's E4M3 row from L2 (TMA, no multicast), appends the meta tail, and one
// cp.async.bulk store writes the whole receive row into its owner's region
// (NVLink for a peer).  Bulk stores took the phase from 0.61 to 0.56 ms at 4
// GPUs against 16-byte stores from every lane.  Before the last CTA stamps
// the owners' data flags, every warp waits for its stores to complete and
// fences them (async proxy, then system scope).
__device__ __forceinline__ void bulk_store(void* dst_global, const void* src_smem, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst_global),
               "r"(smem_u32(src_smem)), "r"(bytes)
               : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

__global__ void __launch_bounds__(kSendWarps * 32)
    ep_send_rows_e4m3_kernel(const EpPeersDev P, const uint8_t* __restrict__ tq, int H, int E, int E_local,
                             const int* __restrict__ offsets, const int* __restrict__ row_token,
                             const float* __restrict__ row_weight) {
  extern __shared__ __align__(128) uint8_t sbuf[];
  __shared__ EpGeom g;
  __shared__ int off_s[257];
  __shared__ uint64_t lbar[kSendWarps];
  __shared__ int abort_s;
  EpRegionHeader* own = hdr_of(P, P.rank);
  if (threadIdx.x == 0) {
    ep_geometry(P, own, g);
    for (int w = 0; w < kSendWarps; ++w) mbar_init(&lbar[w], 1);
    abort_s = 0;
    fence_mbar_init();
  }
  for (int i = threadIdx.x; i <= E; i += blockDim.x) off_s[i] = offsets[i];
  __syncthreads();
  const uint32_t epoch = own->epoch;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KT = H / 128, kt_pad = (KT + 15) & ~15, stride = H + kt_pad;
  uint8_t* buf = sbuf + warp * ((P.row_bytes + 127) & ~127);
  const int rows = g.send_start[P.world];
  uint32_t ph = 0;
  bool ok = true;
  for (int r = blockIdx.x * kSendWarps + warp; ok && r < rows; r += gridDim.x * kSendWarps) {
    int d = 0;
    while (r >= g.send_start[d + 1]) ++d;
    if (!g.fits[d]) continue;
    if (lane == 0) {
      const int t = row_token[r];
      uint8_t* dst =
          P.regions[d] + P.recv_off + static_cast<size_t>(g.dest_off[d] + r - g.send_start[d]) * P.row_bytes;
      asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");  // the buffer's last store has read it
      mbar_arrive_expect_tx(&lbar[warp], static_cast<uint32_t>(stride));
      bulk_load(buf, tq + static_cast<size_t>(t) * stride, static_cast<uint32_t>(stride), &lbar[warp]);
      if (mbar_wait(&lbar[warp], ph, &abort_s)) {
        int lo = 0, hi = E;  // expert of sorted row r: offsets[lo] <= r < offsets[hi]
        while (hi - lo > 1) {
          const int mid = (lo + hi) >> 1;
          if (off_s[mid] <= r)
            lo = mid;
          else
            hi = mid;
        }
        const int dest = lo / E_local;
        *reinterpret_cast<uint4*>(buf + stride) =
            make_uint4(static_cast<uint32_t>(lo - dest * E_local), __float_as_uint(row_weight[r]),
                       static_cast<uint32_t>(t), static_cast<uint32_t>(dest));
        fence_proxy_async_smem();  // the tail (a generic write) before the bulk store reads the buffer
        bulk_store(dst, buf, static_cast<uint32_t>(P.row_bytes));
      } else {
        set_error(&own->err, MOSAIC_ERR_TIMEOUT);
        ok = false;
      }
    }
    ph ^= 1u;
    ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
  }
  if (lane == 0) {
    if (!ok) {  // a load that never completed: no copy may still write into the buffer at exit
      volatile int never = 0;
      mbar_wait(&lbar[warp], ph ^ 1u, &never);
    }
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");  // every store of this warp complete
    asm volatile("fence.proxy.async.global;" ::: "memory");
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    if (atomicAdd(&own->send_done, 1u) == gridDim.x - 1) {
      own->send_done = 0;
      __threadfence_system();
      for (int d2 = 0; d2 < P.world; ++d2) st_release_sys(&hdr_of(P, d2)->data_flag[P.rank], epoch);
    }
  }
}

// ------------------------------------------------------------ unit rows ---
// A token's row goes once to each rank owning one of its experts.  CTA d lists
// the tokens with an expert on rank d, in token order (a block-wide scan):
// unit_token[d * T_stride + p] = token of d's unit p; dest_counts[d] = units.
__global__ void __launch_bounds__(1024)
    ep_units_kernel(const int64_t* __restrict__ idx, int T, int k, int E_local, int T_stride,
                    int* __restrict__ unit_token, int* __restrict__ dest_counts) {
  __shared__ int warp_pre[32];
  __shared__ int tot_s, carry;
  const int d = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t lo = static_cast<int64_t>(d) * E_local, hi = lo + E_local;
  if (tid == 0) carry = 0;
  __syncthreads();
  for (int t0 = 0; t0 < T; t0 += 1024) {
    const int t = t0 + tid;
    int m = 0;
    if (t < T)
      for (int s = 0; s < k; ++s) {
        const int64_t e = idx[static_cast<size_t>(t) * k + s];
        if (e >= lo && e < hi) m = 1;
      }
    const unsigned b = __ballot_sync(0xFFFFFFFFu, m);
    const int wpre = __popc(b & ((1u << lane) - 1u));
    if (lane == 0) warp_pre[warp] = __popc(b);
    __syncthreads();
    if (warp == 0) {
      const int v = warp_pre[lane];
      int incl = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
        if (lane >= o) incl += y;
      }
      warp_pre[lane] = incl - v;
      if (lane == 31) tot_s = incl;
    }
    __syncthreads();
    if (m) unit_token[static_cast<size_t>(d) * T_stride + carry + warp_pre[warp] + wpre] = t;
    __syncthreads();
    if (tid == 0) carry += tot_s;
    __syncthreads();
  }
  if (tid == 0) dest_counts[d] = carry;
}

// Unit rows into the owners' receive rows (the bulk-store scheme of
// ep_send_rows_e4m3_kernel): lane 0 bulk-loads the token's E4M3 row, lane s < k
// writes the slot of assignment s when its expert is on the owner (slots
// packed in slot order), the other slots up to K are marked unused, lane 0
// writes the header {slots used, token}; one bulk store writes the row.
__global__ void __launch_bounds__(kSendWarps * 32)
    ep_send_units_kernel(const EpPeersDev P, const uint8_t* __restrict__ tq, int H, int T_stride, int k, int E_local,
                         int K, const int64_t* __restrict__ idx, const float* __restrict__ weights,
                         const int* __restrict__ row_of, const int* __restrict__ unit_token) {
  extern __shared__ __align__(128) uint8_t sbuf[];
  __shared__ EpGeom g;
  __shared__ uint64_t lbar[kSendWarps];
  __shared__ int abort_s;
  EpRegionHeader* own = hdr_of(P, P.rank);
  if (threadIdx.x == 0) {
    ep_geometry(P, own, g);
    for (int w = 0; w < kSendWarps; ++w) mbar_init(&lbar[w], 1);
    abort_s = 0;
    fence_mbar_init();
  }
  __syncthreads();
  const uint32_t epoch = own->epoch;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KT = H / 128, kt_pad = (KT + 15) & ~15, stride = H + kt_pad;
  uint8_t* buf = sbuf + warp * ((P.row_bytes + 127) & ~127);
  const int rows = g.send_start[P.world];
  uint32_t ph = 0;
  bool ok = true;
  for (int q = blockIdx.x * kSendWarps + warp; ok && q < rows; q += gridDim.x * kSendWarps) {
    int d = 0;
    while (q >= g.send_start[d + 1]) ++d;
    if (!g.fits[d]) continue;
    const int pu = q - g.send_start[d];
    const int t = unit_token[static_cast<size_t>(d) * T_stride + pu];
    uint8_t* dst = P.regions[d] + P.recv_off + static_cast<size_t>(g.dest_off[d] + pu) * P.row_bytes;
    if (lane == 0) {
      asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");  // the buffer's last store has read it
      mbar_arrive_expect_tx(&lbar[warp], static_cast<uint32_t>(stride));
      bulk_load(buf, tq + static_cast<size_t>(t) * stride, static_cast<uint32_t>(stride), &lbar[warp]);
      ok = mbar_wait(&lbar[warp], ph, &abort_s);
      if (!ok) set_error(&own->err, MOSAIC_ERR_TIMEOUT);
    }
    ph ^= 1u;
    ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
    if (!ok) break;
    int e = -1;
    if (lane < k) {
      const int64_t v = idx[static_cast<size_t>(t) * k + lane];
      const int64_t lo = static_cast<int64_t>(d) * E_local;
      if (v >= lo && v < lo + E_local) e = static_cast<int>(v - lo);
    }
    const unsigned m = __ballot_sync(0xFFFFFFFFu, e >= 0);
    const int c = __popc(m);
    uint4* slot = reinterpret_cast<uint4*>(buf + stride + 16);
    if (e >= 0) {
      const size_t a = static_cast<size_t>(t) * k + lane;
      slot[__popc(m & ((1u << lane) - 1u))] =
          make_uint4(static_cast<uint32_t>(e), __float_as_uint(weights ? weights[a] : 1.0f),
                     static_cast<uint32_t>(row_of[a]), 0u);
    }
    if (lane >= c && lane < K) slot[lane] = make_uint4(0xFFFFFFFFu, 0u, 0u, 0u);
    if (lane == 0) *reinterpret_cast<uint4*>(buf + stride) = make_uint4(static_cast<uint32_t>(c), static_cast<uint32_t>(t), 0u, 0u);
    fence_proxy_async_smem();  // every lane's generic writes before the bulk store reads the buffer
    __syncwarp();
    if (lane == 0) bulk_store(dst, buf, static_cast<uint32_t>(P.row_bytes));
  }
  if (lane == 0) {
    if (!ok) {  // a load that never completed: no copy may still write into the buffer at exit
      volatile int never = 0;
      mbar_wait(&lbar[warp], ph ^ 1u, &never);
    }
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");  // every store of this warp complete
    asm volatile("fence.proxy.async.global;" ::: "memory");
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    if (atomicAdd(&own->send_done, 1u) == gridDim.x - 1) {
      own->send_done = 0;
      __threadfence_system();
      for (int d2 = 0; d2 < P.world; ++d2) st_release_sys(&hdr_of(P, d2)->data_flag[P.rank], epoch);
    }
  }
}

// Received unit rows -> assignments: slot j of unit u is assignment u * K + j
// (id -1: unused), with its route weight, the source rank of the unit and the
// assignment's row in the source's return buffer.
__global__ void ep_units_meta_kernel(const EpPeersDev P, int stride, int K, int U_max, int64_t* __restrict__ idx,
                                     float* __restrict__ w, int* __restrict__ a_rank, int* __restrict__ a_pos) {
  griddep_wait();
  griddep_launch();
  const EpRegionHeader* own = hdr_of(P, P.rank);
  const int n = min(own->recv_count, U_max);
  const int a = blockIdx.x * blockDim.x + threadIdx.x;
  if (a >= n * K) return;
  const int u = a / K, j = a - u * K;
  const uint8_t* row = P.regions[P.rank] + P.recv_off + static_cast<size_t>(u) * P.row_bytes;
  const uint4 sl = *reinterpret_cast<const uint4*>(row + stride + 16 + 16 * j);
  idx[a] = static_cast<int64_t>(static_cast<int32_t>(sl.x));
  w[a] = __uint_as_float(sl.y);
  a_pos[a] = static_cast<int>(sl.z);
  int s = 0;
  while (s + 1 < P.world && u >= own->recv_start[s + 1]) ++s;
  a_rank[a] = s;
}

// One CTA, after the down GEMM wrote this rank's partials into the sources'
// return buffers (its threads fenced them at system scope before exiting):
// stamp every source's return flag.
__global__ void ep_signal_return_kernel(const EpPeersDev P) {
  EpRegionHeader* own = hdr_of(P, P.rank);
  const uint32_t epoch = own->epoch;
  const int s = threadIdx.x;
  __threadfence_system();
  if (s < P.world) st_release_sys(&hdr_of(P, s)->ret_flag[P.rank], epoch);
}

// One CTA: wait until every rank stamped this rank's flags (data or return) with the step's epoch.
__global__ void ep_wait_kernel(const EpPeersDev P, int which) {
  EpRegionHeader* own = hdr_of(P, P.rank);
  const uint32_t epoch = own->epoch;
  const int p = threadIdx.x;
  if (p < P.world) {
    const uint32_t* f = (which == 0) ? &own->data_flag[p] : &own->ret_flag[p];
    if (!wait_epoch(f, epoch, P.wait_ns)) set_error(&own->err, MOSAIC_ERR_TIMEOUT);
  }
}

}  // namespace

cudaError_t launch_ep_pack(const void* x, int H, int A, int E, int E_local, int world, const int* offsets,
                           const int* row_token, const float* row_weight, void* send, int* dest_counts,
                           cudaStream_t stream) {
  if (A > 0) {
    int grid = (A + kPackWarps - 1) / kPackWarps;
    if (grid > 148 * 8) grid = 148 * 8;
    ep_pack_kernel<<<grid, kPackWarps * 32, 0, stream>>>(static_cast<const uint4*>(x), H, A, E, E_local, offsets,
                                                         row_token, row_weight, static_cast<uint4*>(send));
  }
  ep_dest_counts_kernel<<<(world + 127) / 128, 128, 0, stream>>>(offsets, E_local, world, dest_counts);
  return cudaGetLastError();
}

cudaError_t launch_rows_meta(const int32_t* ids, const float* weights, int stride, int R, const int* rows_dev, int E,
                             int default_id, int64_t* idx, float* w, int* err, cudaStream_t stream) {
  if (R <= 0) return cudaSuccess;
  rows_meta_kernel<<<(R + 255) / 256, 256, 0, stream>>>(ids, weights, stride, R, rows_dev, E, default_id, idx, w, err);
  return cudaGetLastError();
}

cudaError_t launch_ep_exchange_rows(const EpPeersDev& P, const void* send_rows, const int* dest_counts, int sms,
                                    cudaStream_t stream) {
  ep_counts_kernel<<<1, 32, 0, stream>>>(P, dest_counts);
  ep_send_kernel<<<2 * sms, 256, 0, stream>>>(P, static_cast<const uint4*>(send_rows));
  ep_wait_kernel<<<1, 32, 0, stream>>>(P, 0);
  return cudaGetLastError();
}

cudaError_t launch_ep_dispatch_send_e4m3(const EpPeersDev& P, const void* x, int T, int H, int E, int E_local,
                                         const int* offsets, const int* row_token, const float* row_weight,
                                         int* dest_counts, uint8_t* tq, int sms, cudaStream_t stream) {
  const int kt_pad = (H / 128 + 15) & ~15;
  if (H % 256 || kt_pad > kMaxKtPad || E > 256 || E_local < 1 ||
      P.row_bytes != H + kt_pad + 16)
    return cudaErrorInvalidValue;
  ep_dest_counts_kernel<<<(P.world + 127) / 128, 128, 0, stream>>>(offsets, E_local, P.world, dest_counts);
  int gq = (T + kSendWarps - 1) / kSendWarps;
  if (gq > 8 * sms) gq = 8 * sms;
  ep_tokens_e4m3_kernel<<<gq, kSendWarps * 32, 0, stream>>>(static_cast<const __nv_bfloat16*>(x), T, H, tq);
  ep_counts_kernel<<<1, 32, 0, stream>>>(P, dest_counts);
  // a row buffer per warp: three CTAs per SM at H = 7168
  const int smem = kSendWarps * ((P.row_bytes + 127) & ~127);
  if (smem > 200 * 1024) return cudaErrorInvalidValue;
  int per_sm = (220 * 1024) / (smem + 2048);
  if (per_sm > 3) per_sm = 3;
  cudaError_t e = cudaFuncSetAttribute(ep_send_rows_e4m3_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  ep_send_rows_e4m3_kernel<<<per_sm * sms, kSendWarps * 32, smem, stream>>>(P, tq, H, E, E_local, offsets, row_token,
                                                                             row_weight);
  ep_wait_kernel<<<1, 32, 0, stream>>>(P, 0);
  return cudaGetLastError();
}

cudaError_t launch_ep_dispatch_send_units(const EpPeersDev& P, const void* x, int T, int H, int k, int E_local,
                                          int K, const int64_t* idx, const float* weights, const int* row_of,
                                          int* dest_counts, int* unit_token, uint8_t* tq, int sms,
                                          cudaStream_t stream) {
  const int kt_pad = (H / 128 + 15) & ~15;
  if (H % 256 || kt_pad > kMaxKtPad || E_local < 1 || K < 1 || K > 8 || k < 1 || k > 8 ||
      P.row_bytes != H + kt_pad + 16 + 16 * K)
    return cudaErrorInvalidValue;
  ep_units_kernel<<<P.world, 1024, 0, stream>>>(idx, T, k, E_local, T, unit_token, dest_counts);
  int gq = (T + kSendWarps - 1) / kSendWarps;
  if (gq > 8 * sms) gq = 8 * sms;
  ep_tokens_e4m3_kernel<<<gq, kSendWarps * 32, 0, stream>>>(static_cast<const __nv_bfloat16*>(x), T, H, tq);
  ep_counts_kernel<<<1, 32, 0, stream>>>(P, dest_counts);
  const int smem = kSendWarps * ((P.row_bytes + 127) & ~127);
  if (smem > 200 * 1024) return cudaErrorInvalidValue;
  int per_sm = (220 * 1024) / (smem + 2048);
  if (per_sm > 3) per_sm = 3;
  cudaError_t e = cudaFuncSetAttribute(ep_send_units_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  ep_send_units_kernel<<<per_sm * sms, kSendWarps * 32, smem, stream>>>(P, tq, H, T, k, E_local, K, idx, weights,
                                                                         row_of, unit_token);
  ep_wait_kernel<<<1, 32, 0, stream>>>(P, 0);
  return cudaGetLastError();
}

cudaError_t launch_ep_units_meta(const EpPeersDev& P, int H, int K, int U_max, int64_t* idx, float* w, int* a_rank,
                                 int* a_pos, cudaStream_t stream) {
  const int stride = H + ((H / 128 + 15) & ~15);
  const int n = U_max * K;
  if (n <= 0) return cudaSuccess;
  const cudaError_t e = launch_k(ep_units_meta_kernel, dim3((n + 255) / 256), dim3(256), 0, stream, P, stride, K,
                                 U_max, idx, w, a_rank, a_pos);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

cudaError_t launch_ep_signal_return(const EpPeersDev& P, cudaStream_t stream) {
  ep_signal_return_kernel<<<1, 32, 0, stream>>>(P);
  ep_wait_kernel<<<1, 32, 0, stream>>>(P, 1);
  return cudaGetLastError();
}

cudaError_t launch_ep_return_partials(const EpPeersDev& P, const void* partials, int sms, cudaStream_t stream) {
  ep_return_kernel<<<2 * sms, 256, 0, stream>>>(P, static_cast<const uint4*>(partials));
  ep_wait_kernel<<<1, 32, 0, stream>>>(P, 1);
  return cudaGetLastError();
}

}  // namespace mosaic
