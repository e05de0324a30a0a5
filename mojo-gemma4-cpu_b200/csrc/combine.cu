// combine.cu -- weighted combine of the per-route expert outputs.
//
// Reference: the phase-2 kernels accumulate acc[token] (zero-initialised f32)
// over experts in ascending id order and store bf16(acc)
// (butterquant_kernels/moe.mojo:252-290, kernels/moe_experts.mojo:255-314).
// Here every route's contribution y[pos] = dot*sw*w already sits in f32, and
// this kernel re-creates exactly that summation order per token: the token's
// <=8 local routes are sorted by expert id and added left to right starting
// from 0.0f, then rounded to bf16 with RNE (butterquant/convert.mojo:13-17).
#include "combine_dev.cuh"
#include "gm_kernels.h"
#include "post_moe.cuh"

namespace gm {

constexpr int COMBINE_THREADS = H / 8;  // 352: two float4 column groups per thread and row

__global__ void __launch_bounds__(COMBINE_THREADS)
combine_kernel(const int32_t* __restrict__ route_idx, const int32_t* __restrict__ route_pos,
               const float* __restrict__ ybuf, int T, uint16_t* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  int pos[TOPK];
  routes_by_expert(route_idx, route_pos, t, pos);
  if (gridDim.y == 1) {  // one CTA per row: the thread's two column groups together
    float4 a0, a1;
    sum_routes4x2(ybuf, pos, threadIdx.x, threadIdx.x + COMBINE_THREADS, a0, a1);
    *reinterpret_cast<uint2*>(out + (size_t)t * H + threadIdx.x * 4) = pack_bf16x4(a0);
    *reinterpret_cast<uint2*>(out + (size_t)t * H + (threadIdx.x + COMBINE_THREADS) * 4) = pack_bf16x4(a1);
    return;
  }
  // gridDim.y CTAs share the token's row (column slices)
  const int per = (H / 4) / gridDim.y;
  for (int c4 = blockIdx.y * per + threadIdx.x; c4 < (blockIdx.y + 1) * per; c4 += blockDim.x) {
    const float4 acc = sum_routes4(ybuf, pos, c4);
    uint2 o;
    o.x = (uint32_t)f2bf(acc.x) | ((uint32_t)f2bf(acc.y) << 16);
    o.y = (uint32_t)f2bf(acc.z) | ((uint32_t)f2bf(acc.w) << 16);
    *reinterpret_cast<uint2*>(out + (size_t)t * H + c4 * 4) = o;
  }
}

// The combine followed by the post-MoE tail (post_moe.cuh) on the same row:
// the bf16 MoE row stays in registers.
__global__ void __launch_bounds__(POST_THREADS)
combine_post_kernel(const int32_t* __restrict__ route_idx, const int32_t* __restrict__ route_pos,
                    const float* __restrict__ ybuf, int T, PostParams p) {
  __shared__ float red[POST_THREADS / 32];
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  int pos[TOPK];
  routes_by_expert(route_idx, route_pos, t, pos);
  float m[8];
  float4 acc[2];
  sum_routes4x2(ybuf, pos, threadIdx.x, threadIdx.x + POST_THREADS, acc[0], acc[1]);
#pragma unroll
  for (int g = 0; g < 2; ++g) {
    m[4 * g] = bf2f(f2bf(acc[g].x));
    m[4 * g + 1] = bf2f(f2bf(acc[g].y));
    m[4 * g + 2] = bf2f(f2bf(acc[g].z));
    m[4 * g + 3] = bf2f(f2bf(acc[g].w));
  }
  post_moe_row(m, t, p, red);
}

cudaError_t launch_combine_post(const int32_t* route_idx, const int32_t* route_pos, const float* ybuf,
                                int T, const PostParams& p, cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  return launch_k(combine_post_kernel, dim3(T), dim3(POST_THREADS), 0, s, route_idx, route_pos, ybuf,
                  T, p);
}

cudaError_t launch_combine(const int32_t* route_idx, const int32_t* route_pos, const float* ybuf,
                           int T, uint16_t* out, cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  // small batches: two CTAs per token (half a row each) to spread the reads
  const int split = T < 256 ? 2 : 1;
  return launch_k(combine_kernel, dim3(T, split), dim3(COMBINE_THREADS), 0, s, route_idx, route_pos, ybuf, T, out);
}

}  // namespace gm
