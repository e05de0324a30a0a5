// prep.cu -- on-device producer of the butterquant weight format.
//
// Reference (offline quantizer and load-time bakes):
//  * quant/quantizer.mojo:963-1051 do_quant for PerRowQuant/SingleSided:
//    work = f32(W) [* sqrt|gamma| for SplitGamma, quantizer.mojo:923-943 and
//    butterquant/kernels.mojo:28-33]; FWHT along K in `block` chunks
//    (kernels.mojo:81-85); per-row absmax int8, scale = amax/127
//    (kernels.mojo:58-78,105-107).
//  * butterquant/vnni.mojo:31-83 VNNI pack (pure byte permutation).
//  * butterquant/kernels.mojo:171-224 router_center_softmax (W - column mean).
//  * butterquant/kernels.mojo:37-45 bake_split_gain_in_place and
//    modeling/gemma4_topology.mojo:362-388 router-scale bake.
// All of these are exact restatements (IEEE sqrt/div, same rounding order),
// so the device output is bit-identical to the reference procedure.
#include "gm_kernels.h"

namespace gm {

template <int COLS, int BLOCK>
__global__ void __launch_bounds__(256)
quantize_rows_kernel(const uint16_t* __restrict__ w, long rows, const uint16_t* __restrict__ gamma,
                     int8_t* __restrict__ q, float* __restrict__ scale) {
  static_assert(BLOCK == 128 || BLOCK == 64, "FWHT block");
  constexpr int PER = BLOCK / 32;        // values per lane per block
  constexpr int NBLK = COLS / BLOCK;
  const int lane = threadIdx.x & 31;
  const long r = (long)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (r >= rows) return;
  const uint16_t* src = w + r * COLS;
  float v[NBLK][PER];
  float amax = 0.0f;
#pragma unroll
  for (int b = 0; b < NBLK; ++b) {
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const int k = b * BLOCK + PER * lane + j;
      float x = bf2f(src[k]);
      if (gamma) x = __fmul_rn(x, __fsqrt_rn(fabsf(bf2f(gamma[k]))));
      v[b][j] = x;
    }
    if constexpr (PER == 4) {
      float a, c;
      a = v[b][0]; c = v[b][1]; v[b][0] = __fadd_rn(a, c); v[b][1] = __fsub_rn(a, c);
      a = v[b][2]; c = v[b][3]; v[b][2] = __fadd_rn(a, c); v[b][3] = __fsub_rn(a, c);
      a = v[b][0]; c = v[b][2]; v[b][0] = __fadd_rn(a, c); v[b][2] = __fsub_rn(a, c);
      a = v[b][1]; c = v[b][3]; v[b][1] = __fadd_rn(a, c); v[b][3] = __fsub_rn(a, c);
    } else {
      const float a = v[b][0], c = v[b][1];
      v[b][0] = __fadd_rn(a, c);
      v[b][1] = __fsub_rn(a, c);
    }
#pragma unroll
    for (int m = 1; m <= 16; m <<= 1)
#pragma unroll
      for (int j = 0; j < PER; ++j) v[b][j] = fwht_xor_stage(v[b][j], lane, m);
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      v[b][j] = __fmul_rn(v[b][j], BLOCK == 128 ? fwht_scale_128() : fwht_scale_64());
      amax = fmaxf(amax, fabsf(v[b][j]));
    }
  }
  amax = warp_max(amax);
  const float inv = amax > 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
#pragma unroll
  for (int b = 0; b < NBLK; ++b)
#pragma unroll
    for (int j = 0; j < PER; ++j) q[r * COLS + b * BLOCK + PER * lane + j] = (int8_t)quantize_i8(v[b][j], inv);
  if (lane == 0) scale[r] = __fdiv_rn(amax, 127.0f);
}

// Pack (dir=0) or unpack (dir=1) between row-major int8 [rows][cols] and the
// VNNI tile layout.  One thread moves one 4-byte K group of one row.
__global__ void vnni_permute_kernel(const int8_t* __restrict__ src, long rows, int cols,
                                    int8_t* __restrict__ dst, int dir) {
  const long groups = rows * (cols / 4);
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < groups;
       i += (long)gridDim.x * blockDim.x) {
    const long r = i / (cols / 4);
    const int kg = (int)(i % (cols / 4));
    const int k = kg * 4;
    const long t = r / 32;
    const int n = (int)(r % 32);
    const long poff = t * 32L * cols + (long)(k / 64) * 2048 + (n / 16) * 1024 + ((k % 64) / 4) * 64 +
                      (n % 16) * 4;
    const long roff = r * cols + k;
    if (dir == 0)
      *reinterpret_cast<uint32_t*>(dst + poff) = *reinterpret_cast<const uint32_t*>(src + roff);
    else
      *reinterpret_cast<uint32_t*>(dst + roff) = *reinterpret_cast<const uint32_t*>(src + poff);
  }
}

__global__ void router_center_kernel(const uint16_t* __restrict__ w, int rows, int cols,
                                     uint16_t* __restrict__ out) {
  const int k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= cols) return;
  float gsum = 0.0f;
  for (int r = 0; r < rows; ++r) gsum = __fadd_rn(gsum, bf2f(w[(size_t)r * cols + k]));
  const float gauge = __fmul_rn(gsum, __fdiv_rn(1.0f, (float)rows));
  for (int r = 0; r < rows; ++r)
    out[(size_t)r * cols + k] = f2bf(__fsub_rn(bf2f(w[(size_t)r * cols + k]), gauge));
}

__global__ void bake_kernel(const uint16_t* __restrict__ in, uint16_t* __restrict__ out, int n,
                            int kind) {
  const int k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= n) return;
  const float v = bf2f(in[k]);
  if (kind == 0) {
    const float s = __fsqrt_rn(fmaxf(fabsf(v), 1e-12f));
    out[k] = f2bf(v < 0.0f ? -s : s);
  } else {
    const float inv = __fdiv_rn(1.0f, __uint_as_float(0x42544395u));  // 1/sqrt_f32(2816)
    out[k] = f2bf(__fmul_rn(v, inv));
  }
}

cudaError_t launch_quantize_rows(const uint16_t* w, long rows, int cols, const uint16_t* gamma,
                                 int block, int8_t* q, float* scale, cudaStream_t s) {
  if (rows <= 0) return cudaSuccess;
  const unsigned grid = (unsigned)((rows + 7) / 8);
  if (cols == H && block == 128)
    quantize_rows_kernel<H, 128><<<grid, 256, 0, s>>>(w, rows, gamma, q, scale);
  else if (cols == I && block == 64)
    quantize_rows_kernel<I, 64><<<grid, 256, 0, s>>>(w, rows, gamma, q, scale);
  else if (cols == H && block == 64)
    quantize_rows_kernel<H, 64><<<grid, 256, 0, s>>>(w, rows, gamma, q, scale);
  else if (cols == DENSE_I && block == 64)
    quantize_rows_kernel<DENSE_I, 64><<<grid, 256, 0, s>>>(w, rows, gamma, q, scale);
  else
    return cudaErrorInvalidValue;
  return cudaGetLastError();
}

cudaError_t launch_vnni_permute(const int8_t* src, long rows, int cols, int8_t* dst, int dir,
                                cudaStream_t s) {
  if (rows % 32 || cols % 64) return cudaErrorInvalidValue;
  const long groups = rows * (cols / 4);
  const unsigned grid = (unsigned)std::min<long>((groups + 255) / 256, 148L * 32);
  vnni_permute_kernel<<<grid, 256, 0, s>>>(src, rows, cols, dst, dir);
  return cudaGetLastError();
}

cudaError_t launch_router_center(const uint16_t* w, int rows, int cols, uint16_t* out,
                                 cudaStream_t s) {
  router_center_kernel<<<(cols + 127) / 128, 128, 0, s>>>(w, rows, cols, out);
  return cudaGetLastError();
}

cudaError_t launch_bake(const uint16_t* in, uint16_t* out, int n, int kind, cudaStream_t s) {
  bake_kernel<<<(n + 255) / 256, 256, 0, s>>>(in, out, n, kind);
  return cudaGetLastError();
}

}  // namespace gm
