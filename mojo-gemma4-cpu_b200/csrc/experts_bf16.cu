// experts_bf16.cu -- bf16 expert products (the reference's non-quantised model).
//
// Reference: kernels/moe_experts.mojo:16-162 (Phase1GateUpKernel: g and u dots
// of each routed record against the bf16 gate_up rows, bucket =
// bf16(gelu_tanh(g)*u)) and :201-319 (Phase2DownKernel: down dot times the
// route weight, accumulated per token in ascending expert order).
//
// B200 shape: same work decomposition as the butterquant kernels (expert,
// chunk of <=8 routes, output tile) with mma.m16n8k16 bf16.  Row-major weights
// are streamed with 128-bit no-L1 loads; one lane load is 8 consecutive K
// values of one row, which feed two k16 MMAs through a fixed K permutation
// that the activation fragment (also one 16-byte shared load) mirrors.
#include "gm_kernels.h"

namespace gm {

constexpr int RC_BF = 8;
constexpr int XS_BF = H * 2 + 64;   // staged x_normed row (bytes); 64-byte pad
constexpr int BS_BF = I * 2 + 64;   // staged bucket row (bytes)

template <int KSPLIT, int DEPTH>
__global__ void __launch_bounds__(64 * KSPLIT)
bf16_phase1_kernel(const uint16_t* __restrict__ xn, const int32_t* __restrict__ expert_offset,
                   const SparseRoute* __restrict__ routes, const int32_t* __restrict__ chunk_off,
                   int epr, const uint16_t* __restrict__ w_gu, uint16_t* __restrict__ bucket) {
  constexpr int NTILES = I / 32;                 // 22 intermediate tiles
  constexpr int KCH = (H / 32) / KSPLIT;         // 32-wide K chunks per warp
  extern __shared__ __align__(16) uint8_t smem[];
  uint8_t* xs = smem;                                                        // RC x XS_BF
  float* red = reinterpret_cast<float*>(smem + RC_BF * XS_BF);               // (KSPLIT-1)*2*32*8
  float* dots = red + (KSPLIT - 1) * 2 * 32 * 8;                             // [2][32][RC]

  pdl_wait();
  pdl_trigger();
  const int total = __ldg(chunk_off + epr) * NTILES;
  const int task = blockIdx.x;
  if (task >= total) return;
  const int cg = task / NTILES, it = task % NTILES;
  const int e = find_segment(chunk_off, epr, cg);
  const int rbeg = __ldg(expert_offset + e) + (cg - __ldg(chunk_off + e)) * RC_BF;
  const int nr = min(RC_BF, __ldg(expert_offset + e + 1) - rbeg);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, q = lane & 3;
  const int nt = warp & 1, kh = warp >> 1;
  const int row0 = (nt == 0 ? it * 32 : I + it * 32);
  const uint16_t* wt = w_gu + ((size_t)e * GU + row0) * H;

  uint4 buf[DEPTH][4];
#pragma unroll
  for (int d = 0; d < DEPTH; ++d) {
    const int k0 = (kh * KCH + d) * 32 + 8 * q;
#pragma unroll
    for (int u = 0; u < 4; ++u) buf[d][u] = ldg_stream(wt + (size_t)(g + 8 * u) * H + k0);
  }
  for (int i = tid; i < RC_BF * (H / 8); i += blockDim.x) {
    const int r = i / (H / 8), c = i % (H / 8);
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r < nr) v = *reinterpret_cast<const uint4*>(xn + (size_t)routes[rbeg + r].token * H + c * 8);
    *reinterpret_cast<uint4*>(xs + r * XS_BF + c * 16) = v;
  }
  __syncthreads();

  float acc[2][4];
#pragma unroll
  for (int a = 0; a < 2; ++a)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[a][i] = 0.0f;

#pragma unroll
  for (int c = 0; c < KCH; ++c) {
    uint4 R[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) R[u] = buf[c % DEPTH][u];
    if (c + DEPTH < KCH) {
      const int k0 = (kh * KCH + c + DEPTH) * 32 + 8 * q;
#pragma unroll
      for (int u = 0; u < 4; ++u) buf[c % DEPTH][u] = ldg_stream(wt + (size_t)(g + 8 * u) * H + k0);
    }
    const int k0 = (kh * KCH + c) * 32 + 8 * q;
    const uint4 X = *reinterpret_cast<const uint4*>(xs + g * XS_BF + k0 * 2);
#pragma unroll
    for (int rb = 0; rb < 2; ++rb) {
      mma_bf16(acc[rb], R[2 * rb].x, R[2 * rb + 1].x, R[2 * rb].y, R[2 * rb + 1].y, X.x, X.y);
      mma_bf16(acc[rb], R[2 * rb].z, R[2 * rb + 1].z, R[2 * rb].w, R[2 * rb + 1].w, X.z, X.w);
    }
  }

  if (kh > 0) {
    float* dst = red + (((kh - 1) * 2 + nt) * 32 + lane) * 8;
#pragma unroll
    for (int a = 0; a < 2; ++a)
#pragma unroll
      for (int i = 0; i < 4; ++i) dst[a * 4 + i] = acc[a][i];
  }
  __syncthreads();
  if (kh == 0) {
#pragma unroll
    for (int s = 1; s < KSPLIT; ++s) {
      const float* src = red + (((s - 1) * 2 + nt) * 32 + lane) * 8;
#pragma unroll
      for (int a = 0; a < 2; ++a)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[a][i] = __fadd_rn(acc[a][i], src[a * 4 + i]);
    }
#pragma unroll
    for (int a = 0; a < 2; ++a)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int row = g + 8 * (i >> 1) + 16 * a;
        dots[(nt * 32 + row) * RC_BF + 2 * q + (i & 1)] = acc[a][i];
      }
  }
  __syncthreads();
  for (int o = tid; o < RC_BF * 32; o += blockDim.x) {
    const int r = o >> 5, c = o & 31;
    if (r < nr) {
      const float gv = dots[c * RC_BF + r], uv = dots[(32 + c) * RC_BF + r];
      bucket[(size_t)(rbeg + r) * I + it * 32 + c] = f2bf(__fmul_rn(gelu_tanh_f32(gv), uv));
    }
  }
}

template <int NTILE, int DEPTH>
__global__ void __launch_bounds__(32 * NTILE)
bf16_phase2_kernel(const uint16_t* __restrict__ bucket, const int32_t* __restrict__ expert_offset,
                   const SparseRoute* __restrict__ routes, const int32_t* __restrict__ chunk_off,
                   int epr, const uint16_t* __restrict__ w_dn, float* __restrict__ ybuf) {
  constexpr int GROUPS = (H / 32) / NTILE;
  constexpr int KCH = I / 32;
  __shared__ __align__(16) uint8_t xs[RC_BF * BS_BF];
  __shared__ float s_w[RC_BF];

  pdl_wait();
  pdl_trigger();
  const int total = __ldg(chunk_off + epr) * GROUPS;
  const int task = blockIdx.x;
  if (task >= total) return;
  const int cg = task / GROUPS, hg = task % GROUPS;
  const int e = find_segment(chunk_off, epr, cg);
  const int rbeg = __ldg(expert_offset + e) + (cg - __ldg(chunk_off + e)) * RC_BF;
  const int nr = min(RC_BF, __ldg(expert_offset + e + 1) - rbeg);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, q = lane & 3;
  const int tile = hg * NTILE + warp;
  const uint16_t* wt = w_dn + ((size_t)e * H + tile * 32) * I;

  uint4 buf[DEPTH][4];
#pragma unroll
  for (int d = 0; d < DEPTH; ++d)
#pragma unroll
    for (int u = 0; u < 4; ++u) buf[d][u] = ldg_stream(wt + (size_t)(g + 8 * u) * I + d * 32 + 8 * q);
  for (int i = tid; i < RC_BF * (I / 8); i += blockDim.x) {
    const int r = i / (I / 8), c = i % (I / 8);
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r < nr) v = *reinterpret_cast<const uint4*>(bucket + (size_t)(rbeg + r) * I + c * 8);
    *reinterpret_cast<uint4*>(xs + r * BS_BF + c * 16) = v;
  }
  if (tid < RC_BF) s_w[tid] = tid < nr ? routes[rbeg + tid].weight : 0.0f;
  __syncthreads();

  float acc[2][4];
#pragma unroll
  for (int a = 0; a < 2; ++a)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[a][i] = 0.0f;
#pragma unroll
  for (int c = 0; c < KCH; ++c) {
    uint4 R[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) R[u] = buf[c % DEPTH][u];
    if (c + DEPTH < KCH) {
#pragma unroll
      for (int u = 0; u < 4; ++u)
        buf[c % DEPTH][u] = ldg_stream(wt + (size_t)(g + 8 * u) * I + (c + DEPTH) * 32 + 8 * q);
    }
    const uint4 X = *reinterpret_cast<const uint4*>(xs + g * BS_BF + (c * 32 + 8 * q) * 2);
#pragma unroll
    for (int rb = 0; rb < 2; ++rb) {
      mma_bf16(acc[rb], R[2 * rb].x, R[2 * rb + 1].x, R[2 * rb].y, R[2 * rb + 1].y, X.x, X.y);
      mma_bf16(acc[rb], R[2 * rb].z, R[2 * rb + 1].z, R[2 * rb].w, R[2 * rb + 1].w, X.z, X.w);
    }
  }
#pragma unroll
  for (int a = 0; a < 2; ++a)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = 2 * q + (i & 1);
      if (r < nr) {
        const int row = tile * 32 + g + 8 * (i >> 1) + 16 * a;
        ybuf[(size_t)(rbeg + r) * H + row] = __fmul_rn(acc[a][i], s_w[r]);
      }
    }
}

cudaError_t launch_bf16_phase1(const uint16_t* xn, const int32_t* expert_offset,
                               const SparseRoute* routes, const int32_t* chunk_off, int epr, int T,
                               const uint16_t* w_gu, uint16_t* bucket, cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  constexpr int KSPLIT = 4, DEPTH = 4;
  const size_t smem = (size_t)RC_BF * XS_BF + (size_t)(KSPLIT - 1) * 2 * 32 * 8 * 4 +
                      (size_t)2 * 32 * RC_BF * 4;
  const int grid = max_route_chunks(T, epr, RC_BF) * (I / 32);
  auto k = bf16_phase1_kernel<KSPLIT, DEPTH>;
  cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  return launch_k(k, dim3(grid), dim3(64 * KSPLIT), smem, s, xn, expert_offset, routes, chunk_off,
                  epr, w_gu, bucket);
}

cudaError_t launch_bf16_phase2(const uint16_t* bucket, const int32_t* expert_offset,
                               const SparseRoute* routes, const int32_t* chunk_off, int epr, int T,
                               const uint16_t* w_dn, float* ybuf, cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  constexpr int NTILE = 4, DEPTH = 4;
  const int grid = max_route_chunks(T, epr, RC_BF) * ((H / 32) / NTILE);
  return launch_k(bf16_phase2_kernel<NTILE, DEPTH>, dim3(grid), dim3(32 * NTILE), 0, s, bucket,
                  expert_offset, routes, chunk_off, epr, w_dn, ybuf);
}

}  // namespace gm
