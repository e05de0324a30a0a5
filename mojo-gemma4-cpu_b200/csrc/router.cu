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
// rounding of the activation), split along K into 11 slices of 256 so that
// enough CTAs stream the 720 KB projection at every T.  The dot is taken over
// x * router_scale (exact in f32: a product of two bf16); the token's inv_rms
// (from the activation-norm kernel; the reference computes the same
// rms_reduce_row for both, kernels/rmsnorm.mojo:16-17) multiplies the summed
// dot in the top-8 step, so the logits kernel does not depend on the norm
// kernel and runs beside it: it waits for its predecessor (programmatic
// dependent launch) only after its own stores, which makes its completion
// imply the norm kernel's.  The result differs from the reference's
// per-element (x * s) * inv_rms only by f32 rounding.  Top-8 selection is one
// warp per token with 8 rounds of warp arg-max under the reference's ordering
// (logit descending, ties to the lower expert id).
#include "gm_kernels.h"
#include "router_dev.cuh"

namespace gm {

// Router logits.  CTA = 8 warps, tile = 8 tokens x 32 experts x
// one 256-wide K slice (blockIdx.z).  Lane l owns k = kb+8l..8l+7 of every row
// and reads the bf16 projection straight from global memory (one 16-byte load
// per expert); each warp owns 4 experts.  The 32 (token, expert) lane partials
// are combined by a reduce-scatter butterfly that leaves lane t*4+e holding
// the slice sum of token t and expert e (a fixed, deterministic order).
//
// With tile_count, the K slices of a tile are also reduced here: every CTA
// publishes its partial, and the last of the tile's CTAs to finish (a counter
// per tile, re-armed by that CTA) sums the slices in slice order into slice 0,
// so the top-8 kernel reads T*E logits instead of 11*T*E partials.
__global__ void __launch_bounds__(256)
router_logits_small_kernel(const uint16_t* __restrict__ x, const uint16_t* __restrict__ wr,
                           const uint16_t* __restrict__ rscale, int T, float* __restrict__ logits_base,
                           int* __restrict__ tile_count) {
  constexpr int TT = 8, KS = 256;
  __shared__ __align__(16) float s_s[TT][KS];
  __shared__ int s_last;
  // Launched right after the norm kernel, which triggers only after its own
  // wait: x is complete when this grid starts.  No wait here (see the end).
  pdl_trigger();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int t0 = blockIdx.x * TT, e0 = blockIdx.y * 32, kb = blockIdx.z * KS;
  float* logits = logits_base + (size_t)blockIdx.z * T * E;
  for (int i = tid; i < TT * KS / 2; i += 256) {
    const int t = i / (KS / 2), kp = (i % (KS / 2)) * 2;
    float a = 0.0f, b = 0.0f;
    if (t0 + t < T) {
      const uint32_t v = *reinterpret_cast<const uint32_t*>(x + (size_t)(t0 + t) * H + kb + kp);
      const uint32_t rs = *reinterpret_cast<const uint32_t*>(rscale + kb + kp);
      // `xv * sv` of `xv * sv * inv_vec` (moe_router.mojo:175-178); inv_vec
      // is applied to the summed dot by the top-8 step
      a = __fmul_rn(bf2f(v & 0xFFFFu), bf2f(rs & 0xFFFFu));
      b = __fmul_rn(bf2f(v >> 16), bf2f(rs >> 16));
    }
    s_s[t][kp] = a;
    s_s[t][kp + 1] = b;
  }
  __syncthreads();
  float v[TT * 4];
#pragma unroll
  for (int ee = 0; ee < 4; ++ee) {
    const uint4 w4 = *reinterpret_cast<const uint4*>(wr + (size_t)(e0 + warp * 4 + ee) * H + kb + 8 * lane);
    const float w[8] = {bf2f(w4.x & 0xFFFFu), bf2f(w4.x >> 16), bf2f(w4.y & 0xFFFFu), bf2f(w4.y >> 16),
                        bf2f(w4.z & 0xFFFFu), bf2f(w4.z >> 16), bf2f(w4.w & 0xFFFFu), bf2f(w4.w >> 16)};
#pragma unroll
    for (int t = 0; t < TT; ++t) {
      const float4 s0 = *reinterpret_cast<const float4*>(&s_s[t][8 * lane]);
      const float4 s1 = *reinterpret_cast<const float4*>(&s_s[t][8 * lane + 4]);
      float a = __fmul_rn(s0.x, w[0]);
      a = __fmaf_rn(s0.y, w[1], a);
      a = __fmaf_rn(s0.z, w[2], a);
      a = __fmaf_rn(s0.w, w[3], a);
      a = __fmaf_rn(s1.x, w[4], a);
      a = __fmaf_rn(s1.y, w[5], a);
      a = __fmaf_rn(s1.z, w[6], a);
      a = __fmaf_rn(s1.w, w[7], a);
      v[t * 4 + ee] = a;
    }
  }
#pragma unroll
  for (int m = 16, n = 32; m >= 1; m >>= 1, n >>= 1) {
#pragma unroll
    for (int i = 0; i < n / 2; ++i) {
      const bool up = (lane & m) != 0;
      const float send = up ? v[i] : v[i + n / 2];
      const float keep = up ? v[i + n / 2] : v[i];
      v[i] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, m));
    }
  }
  const int t = t0 + (lane >> 2);
  if (t < T) logits[(size_t)t * E + e0 + warp * 4 + (lane & 3)] = v[0];
  if (tile_count) {
    __threadfence();  // this CTA's partial is visible before it is counted
    __syncthreads();
    int* ctr = tile_count + blockIdx.x * gridDim.y + blockIdx.y;
    if (tid == 0) s_last = atomicAdd(ctr, 1) == (int)gridDim.z - 1;
    __syncthreads();
    if (s_last) {
      __threadfence();
      const int tt = t0 + (tid >> 5), ee = e0 + (tid & 31);
      if (tt < T) {
        float* p = logits_base + (size_t)tt * E + ee;
        float a = __ldcg(p);
        for (int z = 1; z < (int)gridDim.z; ++z) a = __fadd_rn(a, __ldcg(p + (size_t)z * T * E));
        *p = a;
      }
      if (tid == 0) *ctr = 0;  // re-armed for the next call on this stream
    }
  }
  // this grid completes only after its predecessor (the norm kernel) has:
  // the top-8 step, which waits for this grid, then sees inv_rms
  pdl_wait();
}

// inv_rms of each token (one warp per token): kernels/rmsnorm.mojo:16-17,45-46.
__global__ void __launch_bounds__(256)
rms_inv_kernel(const uint16_t* __restrict__ x, int T, float* __restrict__ inv_rms) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (t >= T) return;
  const uint16_t* xr = x + (size_t)t * H;
  float ss = 0.0f;
#pragma unroll
  for (int b = 0; b < H / NORM_BLOCK; ++b) {
    uint2 raw = *reinterpret_cast<const uint2*>(xr + b * NORM_BLOCK + 4 * lane);
    float v[4] = {bf2f(raw.x & 0xFFFFu), bf2f(raw.x >> 16), bf2f(raw.y & 0xFFFFu), bf2f(raw.y >> 16)};
#pragma unroll
    for (int j = 0; j < 4; ++j) ss = __fadd_rn(ss, __fmul_rn(v[j], v[j]));
  }
  ss = warp_sum(ss);
  if (lane == 0) inv_rms[t] = inv_rms_from_sumsq(ss);
}

__global__ void __launch_bounds__(128)
topk_softmax_kernel(float* __restrict__ logits, int ksplit, const uint16_t* __restrict__ pes,
                    const float* __restrict__ inv_rms, int T, int32_t* __restrict__ route_idx,
                    float* __restrict__ route_w) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x * 4 + (threadIdx.x >> 5);
  if (t >= T) return;
  topk_token(logits, ksplit, pes, inv_rms, T, t, threadIdx.x & 31, route_idx, route_w);
}

// The top-8 of topk_softmax_kernel with the token's inv_rms computed first by
// the same warp from its x row (rms_inv_kernel's per-lane chain over the 22
// blocks, then the warp tree), stored for the norm kernel that follows the
// schedule.
__global__ void __launch_bounds__(128)
topk_inv_softmax_kernel(const uint16_t* __restrict__ x, float* __restrict__ logits, int ksplit,
                        const uint16_t* __restrict__ pes, float* __restrict__ inv_rms, int T,
                        int32_t* __restrict__ route_idx, float* __restrict__ route_w) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * 4 + (threadIdx.x >> 5);
  if (t >= T) return;
  const uint16_t* xr = x + (size_t)t * H;
  uint2 raw[H / NORM_BLOCK];  // every load issued before the chain
#pragma unroll
  for (int b = 0; b < H / NORM_BLOCK; ++b) raw[b] = *reinterpret_cast<const uint2*>(xr + b * NORM_BLOCK + 4 * lane);
  float ss = 0.0f;
#pragma unroll
  for (int b = 0; b < H / NORM_BLOCK; ++b) {
    const float v[4] = {bf2f(raw[b].x & 0xFFFFu), bf2f(raw[b].x >> 16), bf2f(raw[b].y & 0xFFFFu),
                        bf2f(raw[b].y >> 16)};
#pragma unroll
    for (int j = 0; j < 4; ++j) ss = __fadd_rn(ss, __fmul_rn(v[j], v[j]));
  }
  const float inv = inv_rms_from_sumsq(warp_sum(ss));  // the same value in every lane
  if (lane == 0) inv_rms[t] = inv;
  topk_token_inv(logits, ksplit, pes, inv, T, t, lane, route_idx, route_w);
}

cudaError_t launch_topk_inv(const uint16_t* x, float* logits, const uint16_t* pes, float* inv_rms, int T,
                            int32_t* route_idx, float* route_w, cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  return launch_k(topk_inv_softmax_kernel, dim3((T + 3) / 4), dim3(128), 0, s, x, logits,
                  router_ksplit(T), pes, inv_rms, T, route_idx, route_w);
}

// Up to 32 tokens the one-CTA top-8 + schedule kernel runs, so the router
// reduces its K slices itself (tile counters); above, the top-8 kernel (T/4
// CTAs) sums the slices while it loads them.
int router_ksplit(int T) {
  return T >= ROUTER_WIDE_MIN_TOKENS ? ROUTER_WIDE_SLICES : T > 32 ? ROUTER_SLICES : 1;
}

int router_tile_counters(int T) { return (T + 7) / 8 * (E / 32); }

// partials [11][T][E], inv_rms [T], one device error word, tile counters
size_t router_workspace_floats(int T) {
  return (size_t)ROUTER_SLICES * T * E + T + 1 + router_tile_counters(T);
}

cudaError_t launch_router_logits(const uint16_t* x, const uint16_t* wr, const uint16_t* rscale, int T,
                                 float* logits, int* err, int* tile_counters, cudaStream_t s,
                                 bool wait_first) {
  if (T <= 0) return cudaSuccess;
  if (T >= ROUTER_TC_MIN_TOKENS && err)
    return launch_router_logits_tc(x, wr, rscale, T, logits, err, s, wait_first);
  if (wait_first) return cudaErrorInvalidValue;  // the FMA kernel always waits last
  if (T >= ROUTER_WIDE_MIN_TOKENS) return cudaErrorInvalidValue;  // the wide slicing is the tcgen05 kernel's
  if (router_ksplit(T) > 1) {
    tile_counters = nullptr;  // ROUTER_SLICES separate partials, summed by the top-8 kernel
  } else if (!tile_counters) {
    return cudaErrorInvalidValue;
  }
  return launch_k(router_logits_small_kernel, dim3((T + 7) / 8, E / 32, ROUTER_SLICES), dim3(256), 0,
                  s, x, wr, rscale, T, logits, tile_counters);
}

cudaError_t launch_rms_inv(const uint16_t* x, int T, float* inv_rms, cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  return launch_k(rms_inv_kernel, dim3((T + 7) / 8), dim3(256), 0, s, x, T, inv_rms);
}

cudaError_t launch_topk(float* logits, const uint16_t* pes, const float* inv_rms, int T,
                        int32_t* route_idx, float* route_w, cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  return launch_k(topk_softmax_kernel, dim3((T + 3) / 4), dim3(128), 0, s, logits,
                  router_ksplit(T), pes, inv_rms, T, route_idx, route_w);
}

// Standalone router (gm_router_select): inv_rms, a device error word and the
// tile counters in the tail of the workspace (cleared here: the caller's
// workspace may hold anything), then logits and top-8.
cudaError_t launch_router(const uint16_t* x, const uint16_t* wr, const uint16_t* rscale,
                          const uint16_t* pes, int T, float* logits, int32_t* route_idx,
                          float* route_w, cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  float* inv = logits + (size_t)ROUTER_SLICES * T * E;
  int* err = reinterpret_cast<int*>(inv + T);
  int* counters = err + 1;
  cudaError_t e = cudaMemsetAsync(err, 0, sizeof(int) * (1 + router_tile_counters(T)), s);
  if (e == cudaSuccess) e = launch_rms_inv(x, T, inv, s);
  if (e == cudaSuccess) e = launch_router_logits(x, wr, rscale, T, logits, err, counters, s);
  if (e == cudaSuccess) e = launch_topk(logits, pes, inv, T, route_idx, route_w, s);
  return e;
}

}  // namespace gm
