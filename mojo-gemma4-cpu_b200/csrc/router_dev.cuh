// router_dev.cuh -- device part of the top-8 selection shared by the router
// and the fused top-8 + schedule kernel.
#pragma once
#include "gm_common.cuh"

namespace gm {

// Top-8 of token t by one warp (lane l holds experts l, l+32, l+64, l+96).
// The split-K partial logits are dots of the un-normalised router input
// (x * router_scale); they are summed in slice order (deterministic), times
// the token's inv_rms (the reference's (x * s) * inv_rms scaling, moved after
// the dot so that the router does not wait for the norm), and the logit is
// written back to slice 0.  moe_router.mojo:44-57 ordering and :276-293
// softmax / per_expert_scale.
__device__ __forceinline__ void topk_token_inv(float* __restrict__ logits, int ksplit,
                                               const uint16_t* __restrict__ pes, float inv, int T, int t,
                                               int lane, int32_t* __restrict__ route_idx,
                                               float* __restrict__ route_w) {
  // all partial loads are issued before any add (independent, one L2 round trip)
  constexpr int MAX_KSPLIT = 11;
  float part[4][MAX_KSPLIT];
#pragma unroll
  for (int j = 0; j < 4; ++j)
#pragma unroll
    for (int z = 0; z < MAX_KSPLIT; ++z)
      part[j][z] = z < ksplit ? logits[(size_t)z * T * E + (size_t)t * E + lane + 32 * j] : 0.0f;
  float v[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float a = part[j][0];
#pragma unroll
    for (int z = 1; z < MAX_KSPLIT; ++z)
      if (z < ksplit) a = __fadd_rn(a, part[j][z]);
    a = __fmul_rn(a, inv);
    logits[(size_t)t * E + lane + 32 * j] = a;
    v[j] = a;
  }
  unsigned taken = 0;
  int sel_e[TOPK];
  float sel_l[TOPK];
#pragma unroll
  for (int k = 0; k < TOPK; ++k) {
    float bv = -INFINITY;
    int bi = 0x7FFFFFFF;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      int id = lane + 32 * j;
      if (!((taken >> j) & 1u) && (v[j] > bv || (v[j] == bv && id < bi))) { bv = v[j]; bi = id; }
    }
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) {
      float ov = __shfl_xor_sync(0xffffffffu, bv, m);
      int oi = __shfl_xor_sync(0xffffffffu, bi, m);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if (bi >= E) bi = 0;  // only reachable with NaN logits; keeps indices in range
    sel_e[k] = bi;
    sel_l[k] = bv;
    if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
  }
  if (lane < TOPK) {
    float maxl = sel_l[0];
    float ev[TOPK];
    float sum = 0.0f;
#pragma unroll
    for (int k = 0; k < TOPK; ++k) {
      ev[k] = fast_exp_softmax_biased(__fsub_rn(sel_l[k], maxl));
      sum = __fadd_rn(sum, ev[k]);
    }
    const float inv_sum = __fdiv_rn(1.0f, sum);
    // lane k stores slot k (all lanes hold the same sel_e / ev)
#pragma unroll
    for (int k = 0; k < TOPK; ++k)
      if (k == lane) {
        route_idx[t * TOPK + k] = sel_e[k];
        route_w[t * TOPK + k] = __fmul_rn(__fmul_rn(ev[k], inv_sum), bf2f(pes[sel_e[k]]));
      }
  }
}

// The same with the token's inv_rms read from inv_rms[t].
__device__ __forceinline__ void topk_token(float* __restrict__ logits, int ksplit, const uint16_t* __restrict__ pes,
                           const float* __restrict__ inv_rms, int T, int t, int lane,
                           int32_t* __restrict__ route_idx, float* __restrict__ route_w) {
  topk_token_inv(logits, ksplit, pes, inv_rms[t], T, t, lane, route_idx, route_w);
}

}  // namespace gm
