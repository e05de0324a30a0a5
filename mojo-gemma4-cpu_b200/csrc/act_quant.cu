// act_quant.cu -- activation preparation of the MoE block.
//
//  * bq_norm_quant: butterquant/runtime.mojo:11-37 prepare_norm_activation
//    [per_block=False, block=128] as dispatched by
//    butterquant_kernels/linear.mojo:58-82: v = x*inv_rms*gamma' (gamma' is the
//    split-gain baked pre_feedforward_layernorm_2), FWHT-128 per block, one
//    absmax over the whole row, int8 = clamp(roundeven(v*127/amax)), sa = amax.
//  * block_quant: butterquant/runtime.mojo:62-79 prepare_block_activation
//    [block=64, apply_fwht=True] (butterquant_kernels/linear.mojo:182-205) on
//    the bf16 bucket: FWHT-64 then per-64-block absmax int8.
//  * rms_norm_bf16: kernels/rmsnorm.mojo:21-47 bf16(x*inv_rms*gamma) for the
//    bf16 expert path (modeling/gemma_4_moe.mojo:537-541).
//
// One warp per row (two for bq_norm_quant).  For the 128-wide FWHT lane l holds elements 4l..4l+3 of
// each block (butterfly strides 1,2 in registers, 4..64 across lanes); for the
// 64-wide FWHT lane l holds 2l, 2l+1 (stride 1 in registers, 2..32 across).
#include "gm_kernels.h"

namespace gm {

// FWHT-128 of the block held as v[0..3] = elements 4*lane+j.
__device__ __forceinline__ void fwht128_lane4(float (&v)[4], int lane) {
  float a, b;
  a = v[0]; b = v[1]; v[0] = __fadd_rn(a, b); v[1] = __fsub_rn(a, b);
  a = v[2]; b = v[3]; v[2] = __fadd_rn(a, b); v[3] = __fsub_rn(a, b);
  a = v[0]; b = v[2]; v[0] = __fadd_rn(a, b); v[2] = __fsub_rn(a, b);
  a = v[1]; b = v[3]; v[1] = __fadd_rn(a, b); v[3] = __fsub_rn(a, b);
#pragma unroll
  for (int m = 1; m <= 16; m <<= 1)
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = fwht_xor_stage(v[j], lane, m);
#pragma unroll
  for (int j = 0; j < 4; ++j) v[j] = __fmul_rn(v[j], fwht_scale_128());
}

// FWHT-64 of the block held as v[0..1] = elements 2*lane+j.
__device__ __forceinline__ void fwht64_lane2(float& v0, float& v1, int lane) {
  float a = v0, b = v1;
  v0 = __fadd_rn(a, b);
  v1 = __fsub_rn(a, b);
#pragma unroll
  for (int m = 1; m <= 16; m <<= 1) {
    v0 = fwht_xor_stage(v0, lane, m);
    v1 = fwht_xor_stage(v1, lane, m);
  }
  v0 = __fmul_rn(v0, fwht_scale_64());
  v1 = __fmul_rn(v1, fwht_scale_64());
}

// Two warps per row: warp h of the pair holds blocks [11h, 11h + 11).  The
// sum of squares keeps the one-warp order exactly: lane l of warp 0 runs its
// chain over blocks 0..10, hands the running sum to lane l of warp 1, which
// continues over blocks 11..21 and does the warp tree; the absmax (a max, so
// order-free) is combined across the pair.  Half the registers per thread and
// twice the warps of a one-warp-per-row kernel.
constexpr int NQ_ROWS = 4;  // rows per 256-thread CTA
__global__ void __launch_bounds__(256)
bq_norm_quant_kernel(const uint16_t* __restrict__ x, const uint16_t* __restrict__ gamma, int T,
                     int8_t* __restrict__ xi8, float* __restrict__ xsa, float* __restrict__ inv_out) {
  __shared__ float s_ss[NQ_ROWS][32];
  __shared__ float s_inv[NQ_ROWS];
  __shared__ float s_amax[NQ_ROWS][2];
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int k = warp >> 1, h = warp & 1;
  const int t = blockIdx.x * NQ_ROWS + k;
  if (t >= T) return;  // both warps of the pair leave together
  constexpr int NBLK = H / NORM_BLOCK;  // 22
  constexpr int NH = NBLK / 2;          // 11 per warp
  const int bar = 1 + k;                // named barrier of the pair (64 threads)
  const uint16_t* xr = x + (size_t)t * H + h * NH * NORM_BLOCK;
  float v[NH][4];
#pragma unroll
  for (int b = 0; b < NH; ++b) {
    uint2 raw = *reinterpret_cast<const uint2*>(xr + b * NORM_BLOCK + 4 * lane);
    v[b][0] = bf2f(raw.x & 0xFFFFu);
    v[b][1] = bf2f(raw.x >> 16);
    v[b][2] = bf2f(raw.y & 0xFFFFu);
    v[b][3] = bf2f(raw.y >> 16);
  }
  float ss = 0.0f;
  if (h == 1) {
    asm volatile("bar.sync %0, 64;" ::"r"(bar) : "memory");  // warp 0's chain is in s_ss
    ss = s_ss[k][lane];
  }
#pragma unroll
  for (int b = 0; b < NH; ++b)
#pragma unroll
    for (int j = 0; j < 4; ++j) ss = __fadd_rn(ss, __fmul_rn(v[b][j], v[b][j]));
  if (h == 0) {
    s_ss[k][lane] = ss;
    asm volatile("bar.sync %0, 64;" ::"r"(bar) : "memory");
  } else {
    ss = warp_sum(ss);
    const float inv = inv_rms_from_sumsq(ss);
    if (lane == 0) {
      s_inv[k] = inv;
      if (inv_out) inv_out[t] = inv;
    }
  }
  asm volatile("bar.sync %0, 64;" ::"r"(bar) : "memory");  // s_inv written
  const float inv = s_inv[k];
  float amax = 0.0f;
#pragma unroll
  for (int b = 0; b < NH; ++b) {
    uint2 g = *reinterpret_cast<const uint2*>(gamma + (h * NH + b) * NORM_BLOCK + 4 * lane);
    float gv[4] = {bf2f(g.x & 0xFFFFu), bf2f(g.x >> 16), bf2f(g.y & 0xFFFFu), bf2f(g.y >> 16)};
#pragma unroll
    for (int j = 0; j < 4; ++j) v[b][j] = __fmul_rn(__fmul_rn(v[b][j], inv), gv[j]);
    fwht128_lane4(v[b], lane);
#pragma unroll
    for (int j = 0; j < 4; ++j) amax = fmaxf(amax, fabsf(v[b][j]));
  }
  amax = warp_max(amax);
  if (lane == 0) s_amax[k][h] = amax;
  asm volatile("bar.sync %0, 64;" ::"r"(bar) : "memory");
  amax = fmaxf(s_amax[k][0], s_amax[k][1]);
  const float qinv = amax > 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
  int8_t* dst = xi8 + (size_t)t * H + h * NH * NORM_BLOCK;
#pragma unroll
  for (int b = 0; b < NH; ++b) {
    uint32_t packed = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) packed |= (uint32_t)(quantize_i8(v[b][j], qinv) & 0xFF) << (8 * j);
    *reinterpret_cast<uint32_t*>(dst + b * NORM_BLOCK + 4 * lane) = packed;
  }
  if (h == 0 && lane == 0) xsa[t] = amax;
}

// bq_norm_quant_kernel for the tcgen05 prefill path: the pair of warps takes
// the token's inv_rms from the top-8 kernel (the same chain and tree, so the
// same bits), and the quantised row is stored once per local route, at
// xg[route_pos[t*8+k]] in schedule order, with the raw amax as that route's
// scale.
__global__ void __launch_bounds__(256)
bq_norm_gather_kernel(const uint16_t* __restrict__ x, const uint16_t* __restrict__ gamma,
                      const float* __restrict__ inv_rms, int T, const int32_t* __restrict__ route_pos,
                      int8_t* __restrict__ xg, float* __restrict__ xg_sa) {
  __shared__ float s_amax[NQ_ROWS][2];
  __shared__ __align__(16) uint32_t s_row[NQ_ROWS][H / 4];  // the pair's int8 row, then copied out
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int k = warp >> 1, h = warp & 1;
  const int t = blockIdx.x * NQ_ROWS + k;
  if (t >= T) return;  // both warps of the pair leave together
  constexpr int NBLK = H / NORM_BLOCK;  // 22
  constexpr int NH = NBLK / 2;          // 11 per warp
  const int bar = 1 + k;                // named barrier of the pair (64 threads)
  const uint16_t* xr = x + (size_t)t * H + h * NH * NORM_BLOCK;
  uint2 raw[NH];
#pragma unroll
  for (int b = 0; b < NH; ++b) raw[b] = *reinterpret_cast<const uint2*>(xr + b * NORM_BLOCK + 4 * lane);
  // lanes 0..7 hold the token's 8 route positions (-1: expert not local)
  const int my_pos = lane < TOPK ? route_pos[t * TOPK + lane] : -1;
  const float inv = inv_rms[t];
  float v[NH][4];
  float amax = 0.0f;
#pragma unroll
  for (int b = 0; b < NH; ++b) {
    const uint2 g = *reinterpret_cast<const uint2*>(gamma + (h * NH + b) * NORM_BLOCK + 4 * lane);
    const float gv[4] = {bf2f(g.x & 0xFFFFu), bf2f(g.x >> 16), bf2f(g.y & 0xFFFFu), bf2f(g.y >> 16)};
    const float xv[4] = {bf2f(raw[b].x & 0xFFFFu), bf2f(raw[b].x >> 16), bf2f(raw[b].y & 0xFFFFu),
                         bf2f(raw[b].y >> 16)};
#pragma unroll
    for (int j = 0; j < 4; ++j) v[b][j] = __fmul_rn(__fmul_rn(xv[j], inv), gv[j]);
    fwht128_lane4(v[b], lane);
#pragma unroll
    for (int j = 0; j < 4; ++j) amax = fmaxf(amax, fabsf(v[b][j]));
  }
  amax = warp_max(amax);
  if (lane == 0) s_amax[k][h] = amax;
  asm volatile("bar.sync %0, 64;" ::"r"(bar) : "memory");
  amax = fmaxf(s_amax[k][0], s_amax[k][1]);
  const float qinv = amax > 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
#pragma unroll
  for (int b = 0; b < NH; ++b) {
    uint32_t packed = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) packed |= (uint32_t)(quantize_i8(v[b][j], qinv) & 0xFF) << (8 * j);
    s_row[k][(h * NH + b) * (NORM_BLOCK / 4) + lane] = packed;
  }
  asm volatile("bar.sync %0, 64;" ::"r"(bar) : "memory");  // the whole row is in s_row[k]
  // the pair's 64 threads copy the row out in 16-byte units, once per local route
  const uint4* src = reinterpret_cast<const uint4*>(s_row[k]);
  const int pt = h * 32 + lane;
#pragma unroll
  for (int r = 0; r < TOPK; ++r) {
    const int pos = __shfl_sync(0xffffffffu, my_pos, r);
    if (pos < 0) continue;
    uint4* dst = reinterpret_cast<uint4*>(xg + (size_t)pos * H);
    for (int c = pt; c < H / 16; c += 64) dst[c] = src[c];
    if (pt == 0) xg_sa[pos] = amax;
  }
}

__global__ void __launch_bounds__(256)
block_quant_kernel(const uint16_t* __restrict__ src, long rows, int8_t* __restrict__ qi8,
                   float* __restrict__ sa) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const long r = (long)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (r >= rows) return;
  const uint16_t* row = src + r * I;
#pragma unroll
  for (int b = 0; b < NB_DOWN; ++b) {
    uint32_t raw = *reinterpret_cast<const uint32_t*>(row + b * DOWN_BLOCK + 2 * lane);
    float v0 = bf2f(raw & 0xFFFFu), v1 = bf2f(raw >> 16);
    fwht64_lane2(v0, v1, lane);
    float amax = warp_max(fmaxf(fabsf(v0), fabsf(v1)));
    float qinv = amax > 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
    uint32_t q = (uint32_t)(quantize_i8(v0, qinv) & 0xFF) | ((uint32_t)(quantize_i8(v1, qinv) & 0xFF) << 8);
    *reinterpret_cast<uint16_t*>(qi8 + r * I + b * DOWN_BLOCK + 2 * lane) = (uint16_t)q;
    if (lane == 0) sa[r * NB_DOWN + b] = amax;
  }
}

__global__ void __launch_bounds__(256)
rms_norm_bf16_kernel(const uint16_t* __restrict__ x, const uint16_t* __restrict__ gamma, int T,
                     uint16_t* __restrict__ out, float* __restrict__ inv_out) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= T) return;
  constexpr int NBLK = H / NORM_BLOCK;
  const uint16_t* xr = x + (size_t)t * H;
  float v[NBLK][4];
  float ss = 0.0f;
#pragma unroll
  for (int b = 0; b < NBLK; ++b) {
    uint2 raw = *reinterpret_cast<const uint2*>(xr + b * NORM_BLOCK + 4 * lane);
    v[b][0] = bf2f(raw.x & 0xFFFFu);
    v[b][1] = bf2f(raw.x >> 16);
    v[b][2] = bf2f(raw.y & 0xFFFFu);
    v[b][3] = bf2f(raw.y >> 16);
#pragma unroll
    for (int j = 0; j < 4; ++j) ss = __fadd_rn(ss, __fmul_rn(v[b][j], v[b][j]));
  }
  ss = warp_sum(ss);
  const float inv = inv_rms_from_sumsq(ss);
  if (inv_out && lane == 0) inv_out[t] = inv;
  uint16_t* dst = out + (size_t)t * H;
#pragma unroll
  for (int b = 0; b < NBLK; ++b) {
    uint2 g = *reinterpret_cast<const uint2*>(gamma + b * NORM_BLOCK + 4 * lane);
    float gv[4] = {bf2f(g.x & 0xFFFFu), bf2f(g.x >> 16), bf2f(g.y & 0xFFFFu), bf2f(g.y >> 16)};
    uint16_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) o[j] = f2bf(__fmul_rn(__fmul_rn(v[b][j], inv), gv[j]));
    uint2 w;
    w.x = (uint32_t)o[0] | ((uint32_t)o[1] << 16);
    w.y = (uint32_t)o[2] | ((uint32_t)o[3] << 16);
    *reinterpret_cast<uint2*>(dst + b * NORM_BLOCK + 4 * lane) = w;
  }
}

// fused_norm_residual_add (kernels/rmsnorm.mojo:48-64 norm_residual_add_row):
// out = bf16(residual + (src * inv_rms(src)) * w).  The decoder layer applies
// it after the attention block's output projection (src = that output,
// residual = x_main, out = x_main: modeling/gemma_4_moe_bq.mojo:1098-1102), so
// out may alias residual: each thread reads its residual elements before it
// stores the same elements.  One CTA of H/8 threads per token, thread i holds
// elements [8i, 8i+8) (16-byte loads); the sum of squares is each thread's
// chain, a warp tree, then the warps' sums in warp order.
constexpr int NRA_THREADS = H / 8;  // 352

__global__ void __launch_bounds__(NRA_THREADS)
norm_residual_add_kernel(const uint16_t* __restrict__ src, const uint16_t* residual,
                         const uint16_t* __restrict__ w, int T, uint16_t* out) {
  __shared__ float red[NRA_THREADS / 32];
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  if (t >= T) return;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const size_t off = (size_t)t * H + 8 * threadIdx.x;
  const uint4 sv = *reinterpret_cast<const uint4*>(src + off);
  const uint4 rv = *reinterpret_cast<const uint4*>(residual + off);
  const uint4 gv = *reinterpret_cast<const uint4*>(w + 8 * threadIdx.x);
  const uint32_t su[4] = {sv.x, sv.y, sv.z, sv.w}, ru[4] = {rv.x, rv.y, rv.z, rv.w},
                 gu[4] = {gv.x, gv.y, gv.z, gv.w};
  float v[8];
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    v[i] = bf2f((su[i >> 1] >> (16 * (i & 1))) & 0xFFFFu);
    ss = __fadd_rn(ss, __fmul_rn(v[i], v[i]));
  }
  ss = warp_sum(ss);
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  float tot = 0.0f;
#pragma unroll
  for (int i = 0; i < NRA_THREADS / 32; ++i) tot = __fadd_rn(tot, red[i]);
  const float inv = inv_rms_from_sumsq(tot);
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint32_t pair = 0;
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const float r = bf2f((ru[i] >> (16 * k)) & 0xFFFFu), g = bf2f((gu[i] >> (16 * k)) & 0xFFFFu);
      pair |= (uint32_t)f2bf(__fadd_rn(r, __fmul_rn(__fmul_rn(v[2 * i + k], inv), g))) << (16 * k);
    }
    o[i] = pair;
  }
  *reinterpret_cast<uint4*>(out + off) = make_uint4(o[0], o[1], o[2], o[3]);
}

// rms_norm_bf16_kernel for the tcgen05 prefill path of bf16 layers: the
// token's inv_rms comes from the top-8 kernel (the same chain and tree), and
// the normalised bf16 row is stored once per local route, at
// xgb[route_pos[t*8+k]] (schedule order, rows of H bf16).
__global__ void __launch_bounds__(256)
rms_norm_gather_bf16_kernel(const uint16_t* __restrict__ x, const uint16_t* __restrict__ gamma,
                            const float* __restrict__ inv_rms, int T, const int32_t* __restrict__ route_pos,
                            uint16_t* __restrict__ xgb) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= T) return;
  constexpr int NBLK = H / NORM_BLOCK;
  const uint16_t* xr = x + (size_t)t * H;
  const int my_pos = lane < TOPK ? route_pos[t * TOPK + lane] : -1;
  const float inv = inv_rms[t];
  uint2 w[NBLK];
#pragma unroll
  for (int b = 0; b < NBLK; ++b) {
    const uint2 raw = *reinterpret_cast<const uint2*>(xr + b * NORM_BLOCK + 4 * lane);
    const uint2 g = *reinterpret_cast<const uint2*>(gamma + b * NORM_BLOCK + 4 * lane);
    const float v[4] = {bf2f(raw.x & 0xFFFFu), bf2f(raw.x >> 16), bf2f(raw.y & 0xFFFFu), bf2f(raw.y >> 16)};
    const float gv[4] = {bf2f(g.x & 0xFFFFu), bf2f(g.x >> 16), bf2f(g.y & 0xFFFFu), bf2f(g.y >> 16)};
    uint16_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) o[j] = f2bf(__fmul_rn(__fmul_rn(v[j], inv), gv[j]));
    w[b].x = (uint32_t)o[0] | ((uint32_t)o[1] << 16);
    w[b].y = (uint32_t)o[2] | ((uint32_t)o[3] << 16);
  }
#pragma unroll
  for (int r = 0; r < TOPK; ++r) {
    const int pos = __shfl_sync(0xffffffffu, my_pos, r);
    if (pos < 0) continue;
    uint16_t* dst = xgb + (size_t)pos * H;
#pragma unroll
    for (int b = 0; b < NBLK; ++b) *reinterpret_cast<uint2*>(dst + b * NORM_BLOCK + 4 * lane) = w[b];
  }
}

cudaError_t launch_rms_norm_gather_bf16(const uint16_t* x, const uint16_t* gamma, const float* inv_rms, int T,
                                        const int32_t* route_pos, uint16_t* xgb, cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  return launch_k(rms_norm_gather_bf16_kernel, dim3((T + 7) / 8), dim3(256), 0, s, x, gamma, inv_rms, T,
                  route_pos, xgb);
}

cudaError_t launch_bq_norm_quant(const uint16_t* x, const uint16_t* gamma, int T, int8_t* xi8,
                                 float* xsa, float* inv_rms, cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  // two warps per token, four tokens per CTA
  return launch_k(bq_norm_quant_kernel, dim3((T + NQ_ROWS - 1) / NQ_ROWS), dim3(256), 0, s, x, gamma, T, xi8,
                  xsa, inv_rms);
}

cudaError_t launch_bq_norm_gather(const uint16_t* x, const uint16_t* gamma, const float* inv_rms, int T,
                                  const int32_t* route_pos, int8_t* xg, float* xg_sa, cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  return launch_k(bq_norm_gather_kernel, dim3((T + NQ_ROWS - 1) / NQ_ROWS), dim3(256), 0, s, x, gamma,
                  inv_rms, T, route_pos, xg, xg_sa);
}

cudaError_t launch_block_quant(const uint16_t* bucket, long rows, int8_t* qi8, float* sa,
                               cudaStream_t s) {
  if (rows <= 0) return cudaSuccess;
  return launch_k(block_quant_kernel, dim3((unsigned)((rows + 7) / 8)), dim3(256), 0, s, bucket, rows,
                  qi8, sa);
}

cudaError_t launch_rms_norm_bf16(const uint16_t* x, const uint16_t* gamma, int T, uint16_t* out,
                                 float* inv_rms, cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  const int wpb = T <= 512 ? 2 : 8;
  return launch_k(rms_norm_bf16_kernel, dim3((T + wpb - 1) / wpb), dim3(32 * wpb), 0, s, x, gamma, T, out,
                  inv_rms);
}

cudaError_t launch_norm_residual_add(const uint16_t* src, const uint16_t* residual, const uint16_t* w, int T,
                                     uint16_t* out, cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  return launch_k(norm_residual_add_kernel, dim3(T), dim3(NRA_THREADS), 0, s, src, residual, w, T, out);
}

}  // namespace gm
