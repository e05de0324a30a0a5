// combine_dev.cuh -- the weighted combine fused into the down products
// (tcgen05 kernel in gemm_tc.cu, decode kernel in experts_bq.cu).
//
// Reference: the phase-2 kernels accumulate acc[token] (zero-initialised f32)
// over experts in ascending id order and store bf16(acc)
// (butterquant_kernels/moe.mojo:252-290).  Here each route's weighted output
// y = facc*sw*w is stored as f32 slices of 128 hidden columns, and an arrival
// counter per (token, column slice) finds the token's last route; the warp
// that saw it calls finish_token_slice, which re-creates the reference's sum
// exactly: the token's local routes sorted by expert id, added left to right
// from 0.0f, rounded to bf16 (butterquant/convert.mojo:13-17).
#pragma once
#include "gm_kernels.h"

namespace gm {

// One warp finishes token `tok`'s columns [128*col, 128*col + 128): lane l
// owns 4 of them.  All of the token's slices are requested before the first
// add, so the warp waits for one round trip to L2, not one per route.  The
// result goes to comb.out, or (expert parallel) into the source rank's
// contribution block; the counter is re-armed for the next call.
__device__ __forceinline__ void finish_token_slice(const TcCombine& comb, const float* ybuf, int tok,
                                                   int col, int lane) {
  int ex[TOPK], pp[TOPK], ps[TOPK];
#pragma unroll
  for (int k = 0; k < TOPK; ++k) {
    pp[k] = __ldg(comb.route_pos + (size_t)tok * TOPK + k);
    ex[k] = __ldg(comb.route_idx + (size_t)tok * TOPK + k);
    ps[k] = -1;
  }
  // the token's expert ids are distinct: ps[j] = position of its route of
  // rank j in ascending expert order, -1 past its local routes
#pragma unroll
  for (int k = 0; k < TOPK; ++k) {
    int rank = 0;
#pragma unroll
    for (int j = 0; j < TOPK; ++j) rank += (pp[j] >= 0 && ex[j] < ex[k]) ? 1 : 0;
#pragma unroll
    for (int j = 0; j < TOPK; ++j)
      if (pp[k] >= 0 && rank == j) ps[j] = pp[k];
  }
  const size_t c0 = (size_t)col * 128 + 4 * lane;
  float4 y[TOPK];
#pragma unroll
  for (int k = 0; k < TOPK; ++k)
    y[k] = ps[k] >= 0 ? __ldcg(reinterpret_cast<const float4*>(ybuf + (size_t)ps[k] * H + c0))
                      : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
  for (int k = 0; k < TOPK; ++k)
    if (ps[k] >= 0) {
      acc.x = __fadd_rn(acc.x, y[k].x);
      acc.y = __fadd_rn(acc.y, y[k].y);
      acc.z = __fadd_rn(acc.z, y[k].z);
      acc.w = __fadd_rn(acc.w, y[k].w);
    }
  uint16_t* dst = comb.out ? comb.out + (size_t)tok * H
                           : comb.contrib[tok / comb.cap] + ((size_t)comb.my_rank * comb.cap + tok % comb.cap) * H;
  *reinterpret_cast<uint2*>(dst + c0) = make_uint2((uint32_t)f2bf(acc.x) | ((uint32_t)f2bf(acc.y) << 16),
                                                   (uint32_t)f2bf(acc.z) | ((uint32_t)f2bf(acc.w) << 16));
  if (lane == 0) comb.counts[(size_t)tok * TC_COLS2 + col] = 0;  // re-armed for the next call
}

}  // namespace gm
