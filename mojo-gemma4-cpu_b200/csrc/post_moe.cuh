// post_moe.cuh -- the tail of dispatch_bq_ffn after the MoE
// (modeling/gemma_4_moe_bq.mojo:785-805), applied to one token's finished MoE
// row inside the kernel that produced it, so the MoE output never goes to HBM:
//
//   d1 = bf16(dense * inv_rms(dense) * post_ffn_norm_1)          rms_norm_row
//   d2 = bf16(d1 + (moe * inv_rms(moe)) * post_ffn_norm_2)      norm_residual_add_row
//   xm = bf16(x_main + (d2 * inv_rms(d2)) * post_ffn_norm)      norm_residual_add_row
//   x_main = bf16(xm * layer_scalar)                            scalar_mul_row
//
// (kernels/rmsnorm.mojo:21-67, kernels/elementwise.mojo:75-83).  One CTA of
// 352 threads per token; thread i holds elements [4i, 4i+4) and
// [4(i+352), 4(i+352)+4).
#pragma once
#include "gm_common.cuh"

namespace gm {

struct PostParams {
  const uint16_t* dense;   // [T][H] dense-MLP output (after its all-reduce)
  uint16_t* x_main;        // [T][H] residual stream: the MoE's input, updated in place
  const uint16_t* w1;      // post_feedforward_layernorm_1 [H]
  const uint16_t* w2;      // post_feedforward_layernorm_2 [H]
  const uint16_t* w;       // post_feedforward_layernorm [H]
  float layer_scalar;
};

constexpr int POST_THREADS = H / 8;  // 352

// Sum over the CTA's 352 threads (11 warps) in a fixed order; every thread
// gets the same value.
__device__ __forceinline__ float post_block_sum(float v, float* red) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();  // red[] free (previous use finished)
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < POST_THREADS / 32; ++i) s = __fadd_rn(s, red[i]);
  return s;
}

__device__ __forceinline__ void load_bf16x4(const uint16_t* p, float (&v)[4]) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  v[0] = bf2f(u.x & 0xFFFFu);
  v[1] = bf2f(u.x >> 16);
  v[2] = bf2f(u.y & 0xFFFFu);
  v[3] = bf2f(u.y >> 16);
}

// m: this thread's 8 MoE values, already rounded to bf16 (as the reference's
// moe_out buffer holds them).
__device__ __forceinline__ void post_moe_row(const float (&m)[8], int t, const PostParams& p,
                                             float* red) {
  const int e0 = 4 * threadIdx.x, e1 = 4 * (threadIdx.x + POST_THREADS);
  const size_t row = (size_t)t * H;
  float d[8], x[8], w1[8], w2[8], w[8];
  load_bf16x4(p.dense + row + e0, *reinterpret_cast<float(*)[4]>(d));
  load_bf16x4(p.dense + row + e1, *reinterpret_cast<float(*)[4]>(d + 4));
  load_bf16x4(p.x_main + row + e0, *reinterpret_cast<float(*)[4]>(x));
  load_bf16x4(p.x_main + row + e1, *reinterpret_cast<float(*)[4]>(x + 4));
  load_bf16x4(p.w1 + e0, *reinterpret_cast<float(*)[4]>(w1));
  load_bf16x4(p.w1 + e1, *reinterpret_cast<float(*)[4]>(w1 + 4));
  load_bf16x4(p.w2 + e0, *reinterpret_cast<float(*)[4]>(w2));
  load_bf16x4(p.w2 + e1, *reinterpret_cast<float(*)[4]>(w2 + 4));
  load_bf16x4(p.w + e0, *reinterpret_cast<float(*)[4]>(w));
  load_bf16x4(p.w + e1, *reinterpret_cast<float(*)[4]>(w + 4));
  float ssd = 0.0f, ssm = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    ssd = __fmaf_rn(d[i], d[i], ssd);
    ssm = __fmaf_rn(m[i], m[i], ssm);
  }
  const float inv_d = inv_rms_from_sumsq(post_block_sum(ssd, red));
  const float inv_m = inv_rms_from_sumsq(post_block_sum(ssm, red));
  float d2[8], ss2 = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float d1 = bf2f(f2bf(__fmul_rn(__fmul_rn(d[i], inv_d), w1[i])));
    d2[i] = bf2f(f2bf(__fadd_rn(d1, __fmul_rn(__fmul_rn(m[i], inv_m), w2[i]))));
    ss2 = __fmaf_rn(d2[i], d2[i], ss2);
  }
  const float inv_2 = inv_rms_from_sumsq(post_block_sum(ss2, red));
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 8; i += 2) {
    const float xa = bf2f(f2bf(__fadd_rn(x[i], __fmul_rn(__fmul_rn(d2[i], inv_2), w[i]))));
    const float xb = bf2f(f2bf(__fadd_rn(x[i + 1], __fmul_rn(__fmul_rn(d2[i + 1], inv_2), w[i + 1]))));
    o[i / 2] = (uint32_t)f2bf(__fmul_rn(xa, p.layer_scalar)) |
               ((uint32_t)f2bf(__fmul_rn(xb, p.layer_scalar)) << 16);
  }
  *reinterpret_cast<uint2*>(p.x_main + row + e0) = make_uint2(o[0], o[1]);
  *reinterpret_cast<uint2*>(p.x_main + row + e1) = make_uint2(o[2], o[3]);
}

}  // namespace gm
