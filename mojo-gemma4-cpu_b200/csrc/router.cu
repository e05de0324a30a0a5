// router.cu -- Gemma-4 MoE router on sm_100a.
//
// Reference: kernels/moe_router.mojo:164-191 (RouterExpertKernel: RMSNorm with
// no gain, x*router_scale*inv_rms kept in f32, 128 logits against the bf16
// router projection, per-worker top-8) and :259-293 (RouterMergeKernel: merge
// of the per-worker lists, softmax over the 8 survivors with
// fast_exp_softmax_biased, times per_expert_scale).
//
// B200 shape: the logits are a skinny [T x 2816] x [2816 x 128] product done
// in f32 FMA (the reference's f32-activation x bf16-weight dot, no bf16
// rounding of the activation), tiled through shared memory; top-8 selection is
// one warp per token with 8 rounds of warp arg-max under the reference's
// ordering (logit descending, ties to the lower expert id).
#include "gm_kernels.h"

namespace gm {

template <int TT, int EG, int MT, int ME>
__global__ void __launch_bounds__((TT / MT) * (EG / ME))
router_logits_kernel(const uint16_t* __restrict__ x, const uint16_t* __restrict__ wr,
                     const uint16_t* __restrict__ rscale, int T, int n_experts,
                     float* __restrict__ logits) {
  constexpr int NT = (TT / MT) * (EG / ME);
  constexpr int NW = NT / 32;
  constexpr int KC = 64;
  static_assert(NT % 32 == 0, "whole warps");
  __shared__ float s_inv[TT];
  __shared__ float s_x[KC][TT + 1];
  __shared__ float s_w[KC][EG + 1];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int t0 = blockIdx.x * TT, e0 = blockIdx.y * EG;

  // inv_rms per token (kernels/rmsnorm.mojo:16-17,45-46)
  for (int t = warp; t < TT; t += NW) {
    float ss = 0.0f;
    if (t0 + t < T) {
      const uint16_t* xr = x + (size_t)(t0 + t) * H;
      for (int k = lane * 2; k < H; k += 64) {
        uint32_t v = *reinterpret_cast<const uint32_t*>(xr + k);
        float a = bf2f(v & 0xFFFFu), b = bf2f(v >> 16);
        ss = __fadd_rn(ss, __fmul_rn(a, a));
        ss = __fadd_rn(ss, __fmul_rn(b, b));
      }
      ss = warp_sum(ss);
    }
    if (lane == 0) s_inv[t] = inv_rms_from_sumsq(ss);
  }
  __syncthreads();

  const int tx = tid % (EG / ME), ty = tid / (EG / ME);
  float acc[MT][ME];
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int n = 0; n < ME; ++n) acc[m][n] = 0.0f;

  for (int k0 = 0; k0 < H; k0 += KC) {
    for (int i = tid; i < TT * (KC / 2); i += NT) {
      int t = i / (KC / 2), kp = (i % (KC / 2)) * 2;
      float a = 0.0f, b = 0.0f;
      if (t0 + t < T) {
        uint32_t v = *reinterpret_cast<const uint32_t*>(x + (size_t)(t0 + t) * H + k0 + kp);
        uint32_t rs = *reinterpret_cast<const uint32_t*>(rscale + k0 + kp);
        float inv = s_inv[t];
        // `xv * sv * inv_vec` (moe_router.mojo:175-178): (x*s)*inv, f32
        a = __fmul_rn(__fmul_rn(bf2f(v & 0xFFFFu), bf2f(rs & 0xFFFFu)), inv);
        b = __fmul_rn(__fmul_rn(bf2f(v >> 16), bf2f(rs >> 16)), inv);
      }
      s_x[kp][t] = a;
      s_x[kp + 1][t] = b;
    }
    for (int i = tid; i < EG * (KC / 2); i += NT) {
      int e = i / (KC / 2), kp = (i % (KC / 2)) * 2;
      uint32_t v = 0;
      if (e0 + e < n_experts)
        v = *reinterpret_cast<const uint32_t*>(wr + (size_t)(e0 + e) * H + k0 + kp);
      s_w[kp][e] = bf2f(v & 0xFFFFu);
      s_w[kp + 1][e] = bf2f(v >> 16);
    }
    __syncthreads();
#pragma unroll 8
    for (int k = 0; k < KC; ++k) {
      float xv[MT], wv[ME];
#pragma unroll
      for (int m = 0; m < MT; ++m) xv[m] = s_x[k][ty + m * (TT / MT)];
#pragma unroll
      for (int n = 0; n < ME; ++n) wv[n] = s_w[k][tx + n * (EG / ME)];
#pragma unroll
      for (int m = 0; m < MT; ++m)
#pragma unroll
        for (int n = 0; n < ME; ++n) acc[m][n] = __fmaf_rn(xv[m], wv[n], acc[m][n]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    int t = t0 + ty + m * (TT / MT);
    if (t >= T) continue;
#pragma unroll
    for (int n = 0; n < ME; ++n) {
      int e = e0 + tx + n * (EG / ME);
      if (e < n_experts) logits[(size_t)t * n_experts + e] = acc[m][n];
    }
  }
}

// One warp per token.  Lane l holds experts l, l+32, l+64, l+96.
__global__ void __launch_bounds__(128)
topk_softmax_kernel(const float* __restrict__ logits, const uint16_t* __restrict__ pes, int T,
                    int32_t* __restrict__ route_idx, float* __restrict__ route_w) {
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * 4 + (threadIdx.x >> 5);
  if (t >= T) return;
  float v[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) v[j] = logits[(size_t)t * E + lane + 32 * j];
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
  if (lane == 0) {
    // moe_router.mojo:276-293
    float maxl = sel_l[0];
    float ev[TOPK];
    float sum = 0.0f;
#pragma unroll
    for (int k = 0; k < TOPK; ++k) {
      ev[k] = fast_exp_softmax_biased(__fsub_rn(sel_l[k], maxl));
      sum = __fadd_rn(sum, ev[k]);
    }
    float inv_sum = __fdiv_rn(1.0f, sum);
#pragma unroll
    for (int k = 0; k < TOPK; ++k) {
      route_idx[t * TOPK + k] = sel_e[k];
      route_w[t * TOPK + k] = __fmul_rn(__fmul_rn(ev[k], inv_sum), bf2f(pes[sel_e[k]]));
    }
  }
}

cudaError_t launch_router(const uint16_t* x, const uint16_t* wr, const uint16_t* rscale,
                          const uint16_t* pes, int T, float* logits, int32_t* route_idx,
                          float* route_w, cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  if (T >= 64) {
    dim3 grid((T + 31) / 32, E / 32);
    router_logits_kernel<32, 32, 4, 2><<<grid, 128, 0, s>>>(x, wr, rscale, T, E, logits);
  } else {
    dim3 grid((T + 7) / 8, E / 16);
    router_logits_kernel<8, 16, 1, 1><<<grid, 128, 0, s>>>(x, wr, rscale, T, E, logits);
  }
  topk_softmax_kernel<<<(T + 3) / 4, 128, 0, s>>>(logits, pes, T, route_idx, route_w);
  return cudaGetLastError();
}

}  // namespace gm
