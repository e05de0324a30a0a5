// combine_dev.cuh -- device helpers of the weighted combine kernels
// (combine.cu, and the expert-parallel combine of ep.cu): a token's route
// rows y = facc*sw*w (f32, one row per route) summed in the reference's order,
// ascending expert id from 0.0f (butterquant_kernels/moe.mojo:252-290).
#pragma once
#include "gm_common.cuh"

namespace gm {

// The token's local routes in ascending expert order (its expert ids are
// distinct): pos[j] = schedule position of its route of rank j, -1 past the
// end.  Computed by every thread from the token's 8 (id, position) pairs.
__device__ __forceinline__ void routes_by_expert(const int32_t* __restrict__ route_idx,
                                                 const int32_t* __restrict__ route_pos, size_t t,
                                                 int (&pos)[TOPK]) {
  int ex[TOPK], pp[TOPK];
#pragma unroll
  for (int k = 0; k < TOPK; ++k) {
    pp[k] = __ldg(route_pos + t * TOPK + k);
    ex[k] = __ldg(route_idx + t * TOPK + k);
    pos[k] = -1;
  }
#pragma unroll
  for (int k = 0; k < TOPK; ++k) {
    int rank = 0;
#pragma unroll
    for (int j = 0; j < TOPK; ++j) rank += (pp[j] >= 0 && ex[j] < ex[k]) ? 1 : 0;
#pragma unroll
    for (int j = 0; j < TOPK; ++j)
      if (pp[k] >= 0 && rank == j) pos[j] = pp[k];
  }
}

// Four columns of a token's row: the route rows' values are all requested
// before the first add (one memory round trip, not one per route), then added
// in ascending expert order from 0.0f.
__device__ __forceinline__ float4 sum_routes4(const float* __restrict__ ybuf, const int (&pos)[TOPK],
                                              int c4) {
  float4 y[TOPK];
#pragma unroll
  for (int k = 0; k < TOPK; ++k)
    y[k] = pos[k] >= 0 ? *reinterpret_cast<const float4*>(ybuf + (size_t)pos[k] * H + c4 * 4)
                       : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
  for (int k = 0; k < TOPK; ++k)
    if (pos[k] >= 0) {
      acc.x = __fadd_rn(acc.x, y[k].x);
      acc.y = __fadd_rn(acc.y, y[k].y);
      acc.z = __fadd_rn(acc.z, y[k].z);
      acc.w = __fadd_rn(acc.w, y[k].w);
    }
  return acc;
}

}  // namespace gm
