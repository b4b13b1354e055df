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
    for (int v = lane; v < vec_per_row; v += 32) dst[v] = src[v];
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
                                 int E, int default_id, int64_t* __restrict__ idx, float* __restrict__ w, int* err) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= R) return;
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

cudaError_t launch_rows_meta(const int32_t* ids, const float* weights, int stride, int R, int E, int default_id,
                             int64_t* idx, float* w, int* err, cudaStream_t stream) {
  if (R <= 0) return cudaSuccess;
  rows_meta_kernel<<<(R + 255) / 256, 256, 0, stream>>>(ids, weights, stride, R, E, default_id, idx, w, err);
  return cudaGetLastError();
}

}  // namespace mosaic
