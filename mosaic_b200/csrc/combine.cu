// Ordered combine: per token, the routed partials are summed sequentially in
// fp32 in ascending expert-id order, cast to bf16, then the shared expert's
// bf16 output is added with one more bf16 rounding.
//
// Reference behaviour: mosaicvm/model/layers.py:367-373 (ordered fp32 sum of
// grouped_expert_forward) and :297 (y = out_shared + routed, bf16);
// mosaicvm/kernels/mxint.py:1348-1366 (mxint_routed_reduce).
#include "common.cuh"
#include "kernels.h"

namespace mosaic {

namespace {

template <bool F32>
__device__ __forceinline__ void load8(const void* base, size_t off, float (&v)[8]) {
  if constexpr (F32) {
    const float4 a = *reinterpret_cast<const float4*>(static_cast<const float*>(base) + off);
    const float4 b = *reinterpret_cast<const float4*>(static_cast<const float*>(base) + off + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
    const uint4 raw = *reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(base) + off);
    const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(h2[i]);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  }
}

// grid (T, ceil(H / 2048)), 256 threads x 8 values.
template <bool F32>
__global__ void __launch_bounds__(256) combine_kernel(const void* __restrict__ partial,
                                                      const int* __restrict__ row_sorted, int T, int k, int H,
                                                      int shared_base, __nv_bfloat16* __restrict__ y) {
  griddep_wait();  // the down GEMM's partials are visible
  griddep_launch();
  const int t = blockIdx.x;
  const int h0 = (blockIdx.y * 256 + threadIdx.x) * 8;
  if (h0 >= H) return;
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  for (int s = 0; s < k; ++s) {
    const int r = row_sorted[static_cast<size_t>(t) * k + s];
    if (r < 0) continue;
    float v[8];
    load8<F32>(partial, static_cast<size_t>(r) * H + h0, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = acc[i] + v[i];
  }
  float out[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) out[i] = bf16r(acc[i]);
  if (shared_base >= 0) {
    float v[8];
    load8<F32>(partial, static_cast<size_t>(shared_base + t) * H + h0, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) out[i] = out[i] + v[i];
  }
  uint4 pk;
  __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
  for (int i = 0; i < 4; ++i) o2[i] = __floats2bfloat162_rn(out[2 * i], out[2 * i + 1]);
  *reinterpret_cast<uint4*>(y + static_cast<size_t>(t) * H + h0) = pk;
}

}  // namespace

cudaError_t launch_combine(const void* partial, int partial_f32, const int* row_sorted, int T, int k, int H,
                           int shared_base, void* y, cudaStream_t stream) {
  dim3 grid(T, (H + 2047) / 2048);
  const cudaError_t e = partial_f32 ? launch_k(combine_kernel<true>, grid, dim3(256), 0, stream, partial, row_sorted, T,
                                               k, H, shared_base, static_cast<__nv_bfloat16*>(y))
                                    : launch_k(combine_kernel<false>, grid, dim3(256), 0, stream, partial, row_sorted,
                                               T, k, H, shared_base, static_cast<__nv_bfloat16*>(y));
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace mosaic
