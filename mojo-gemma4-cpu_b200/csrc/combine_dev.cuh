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

// Two four-column groups c0 and c1 of a token's row, summed as sum_routes4
// does, with both groups' route loads requested before the first add (16
// loads in flight per thread instead of 8).
__device__ __forceinline__ void sum_routes4x2(const float* __restrict__ ybuf, const int (&pos)[TOPK], int c0,
                                              int c1, float4& a0, float4& a1) {
  float4 y0[TOPK], y1[TOPK];
#pragma unroll
  for (int k = 0; k < TOPK; ++k) {
    const float* row = ybuf + (size_t)(pos[k] >= 0 ? pos[k] : 0) * H;
    y0[k] = pos[k] >= 0 ? *reinterpret_cast<const float4*>(row + c0 * 4) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    y1[k] = pos[k] >= 0 ? *reinterpret_cast<const float4*>(row + c1 * 4) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  }
  a0 = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  a1 = a0;
#pragma unroll
  for (int k = 0; k < TOPK; ++k)
    if (pos[k] >= 0) {
      a0.x = __fadd_rn(a0.x, y0[k].x);
      a0.y = __fadd_rn(a0.y, y0[k].y);
      a0.z = __fadd_rn(a0.z, y0[k].z);
      a0.w = __fadd_rn(a0.w, y0[k].w);
      a1.x = __fadd_rn(a1.x, y1[k].x);
      a1.y = __fadd_rn(a1.y, y1[k].y);
      a1.z = __fadd_rn(a1.z, y1[k].z);
      a1.w = __fadd_rn(a1.w, y1[k].w);
    }
}

__device__ __forceinline__ uint2 pack_bf16x4(float4 a) {
  return make_uint2((uint32_t)f2bf(a.x) | ((uint32_t)f2bf(a.y) << 16),
                    (uint32_t)f2bf(a.z) | ((uint32_t)f2bf(a.w) << 16));
}

}  // namespace gm
