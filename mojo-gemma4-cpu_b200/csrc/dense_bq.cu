// dense_bq.cu -- the dense butterquant MLP that runs beside the MoE in every
// Gemma-4 FFN (dispatch_bq_ffn, modeling/gemma_4_moe_bq.mojo:749-783):
//
//   x_i8, x_sa  = bq_norm_quant(x_main, pre_feedforward_layernorm)   (act_quant.cu)
//   gate, up    = bq_linear(x, gate_proj), bq_linear(x, up_proj)      bf16 [T][2112]
//                 (butterquant/gemm.mojo:115-143: (f32(iacc) - 128*colsum) * (sa/127) * sw)
//   h           = bf16(gelu_tanh(gate) * up)         (kernels/elementwise.mojo:17-24)
//   h_i8, h_sa  = FWHT-64 block quant of h           (butterquant_kernels/linear.mojo:159-205)
//   dense_out   = bq_block_linear(h, down_proj)      bf16 [T][2816]
//                 (butterquant/gemm.mojo:174-216: facc = fma(iacc_b - 128*cs_b, sa_b/127, facc)
//                  over the 33 K-blocks in order, out = facc * sw)
//
// Weights stay in the reference's VNNI-packed layout and stream from HBM into
// mma.m16n8k32 fragments (vnni_stream.cuh).  The dots are signed x signed,
// equal to the reference's u8 x s8 - 128*colsum whenever |iacc| < 2^24.
//
// Kernel 1 (gate/up/GeGLU/block quant) has work items (16-token chunk,
// 64-wide intermediate block j): gate tiles 2j, 2j+1 and up tiles 2j, 2j+1
// (32 rows each) against the chunk's activations, K split over 4 warp
// quarters; the epilogue rounds gate and up to bf16 as the reference stores
// them, applies GeGLU, rounds h, and does FWHT-64 + per-block int8 in
// registers, so only h_i8/h_sa reach HBM.
// Kernel 2 (down) has work items (16-token chunk, 32-row hidden tile); three
// warps each take 11 of the 33 K-blocks, the second and third hand their
// per-block integer dots to the first through shared memory, and the first
// runs the fma chain in block order.
#include "gm_kernels.h"
#include "vnni_stream.cuh"

namespace gm {

namespace {

constexpr int RCD = 16;                // tokens per work item
constexpr int XSTRIDE_D = H + 16;      // staged activation row (bytes)
constexpr int HSTRIDE_D = DENSE_I + 16;  // staged h row (bytes)
constexpr int DSTRIDE_D = 33;          // padded row stride of the kernel-1 dot tile
constexpr int KS2 = 3;                 // K-splits (warps) of kernel 2
constexpr int BPW2 = NB_DENSE / KS2;   // 11 K-blocks per warp
static_assert(NB_DENSE % KS2 == 0, "kernel-2 K split");

template <int KSPLIT, int DEPTH, bool WRITE_BF16>
__global__ void __launch_bounds__(128 * KSPLIT, 2)
dense_gate_up_kernel(const int8_t* __restrict__ xi8, const float* __restrict__ xsa, int T,
                     const int8_t* __restrict__ wg, const float* __restrict__ gsc,
                     const int8_t* __restrict__ wu, const float* __restrict__ usc,
                     int8_t* __restrict__ h_i8, float* __restrict__ h_sa,
                     uint16_t* __restrict__ h_bf16) {
  constexpr int NWARP = 4 * KSPLIT;
  constexpr int KCH = (H / 32) / KSPLIT;
  static_assert(KCH >= DEPTH, "prefetch depth");
  extern __shared__ __align__(16) uint8_t smem[];
  int8_t* xs = reinterpret_cast<int8_t*>(smem);                            // RCD x XSTRIDE_D
  int* red = reinterpret_cast<int*>(smem + RCD * XSTRIDE_D);               // [(KSPLIT-1)*4][16][32]
  int* dots = red + (KSPLIT - 1) * 4 * 16 * 32;                            // [4][RCD][DSTRIDE_D]
  float* s_ad = reinterpret_cast<float*>(dots + 4 * RCD * DSTRIDE_D);      // [RCD]

  pdl_wait();
  pdl_trigger();
  const int total = ((T + RCD - 1) / RCD) * NB_DENSE;
  int task = blockIdx.x;
  if (task >= total) return;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, q = lane & 3;
  const int nt = warp & 3, kh = warp >> 2;
  auto tile_of = [&](int t) -> const int8_t* {
    const int j = t % NB_DENSE;
    return nt < 2 ? wg + (size_t)(2 * j + nt) * 32 * H : wu + (size_t)(2 * j + nt - 2) * 32 * H;
  };

  uint4 buf[DEPTH][2];
  prefetch_chunks<DEPTH>(buf, tile_of(task), kh * KCH, g, q);

  while (true) {
    const int j = task % NB_DENSE, rbeg = (task / NB_DENSE) * RCD;
    const int nr = min(RCD, T - rbeg);
    if (tid < nr) s_ad[tid] = __fmul_rn(xsa[rbeg + tid], INV127);
    // rows >= nr feed only B columns whose results are never stored
    for (int i = tid; i < nr * (H / 16); i += blockDim.x) {
      const int r = i / (H / 16), c = i % (H / 16);
      cp_async16(xs + r * XSTRIDE_D + c * 16, xi8 + (size_t)(rbeg + r) * H + c * 16);
    }
    cp_async_wait_all();
    __syncthreads();

    const int8_t* wt = tile_of(task);
    int acc[2][2][4];
#pragma unroll
    for (int a = 0; a < 2; ++a)
#pragma unroll
      for (int b = 0; b < 2; ++b)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[a][b][i] = 0;
    const bool two_groups = nr > 8;

#pragma unroll
    for (int c = 0; c < KCH; ++c) {
      const uint4 A = buf[c % DEPTH][0], B = buf[c % DEPTH][1];
      if (c + DEPTH < KCH) {
        const int gc = kh * KCH + c + DEPTH;
        const int8_t* p = wt + (gc >> 1) * 2048 + vnni_lane_off(g, q, gc & 1);
        buf[c % DEPTH][0] = ldg_stream(p);
        buf[c % DEPTH][1] = ldg_stream(p + 256);
      }
      const int k0 = (kh * KCH + c) * 32;
      {
        const int8_t* xr = xs + g * XSTRIDE_D + k0 + 4 * q;
        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(xr);
        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(xr + 16);
        mma_s8(acc[0][0], A.x, A.y, B.x, B.y, b0, b1);
        mma_s8(acc[0][1], A.z, A.w, B.z, B.w, b0, b1);
      }
      if (two_groups) {
        const int8_t* xr = xs + (8 + g) * XSTRIDE_D + k0 + 4 * q;
        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(xr);
        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(xr + 16);
        mma_s8(acc[1][0], A.x, A.y, B.x, B.y, b0, b1);
        mma_s8(acc[1][1], A.z, A.w, B.z, B.w, b0, b1);
      }
    }

    const int nxt = task + gridDim.x;
    const bool has_next = nxt < total;
    if (has_next) prefetch_chunks<DEPTH>(buf, tile_of(nxt), kh * KCH, g, q);

    // K-split reduction (integer, order-free) into dots[tile][token][row]
    if (kh > 0) {
      int* dst = red + ((kh - 1) * 4 + nt) * 16 * 32 + lane;
#pragma unroll
      for (int a = 0; a < 2; ++a)
#pragma unroll
        for (int b = 0; b < 2; ++b)
#pragma unroll
          for (int i = 0; i < 4; ++i) dst[((a * 2 + b) * 4 + i) * 32] = acc[a][b][i];
    }
    __syncthreads();
    if (kh == 0) {
#pragma unroll
      for (int s = 1; s < KSPLIT; ++s) {
        const int* src = red + ((s - 1) * 4 + nt) * 16 * 32 + lane;
#pragma unroll
        for (int a = 0; a < 2; ++a)
#pragma unroll
          for (int b = 0; b < 2; ++b)
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[a][b][i] += src[((a * 2 + b) * 4 + i) * 32];
      }
#pragma unroll
      for (int a = 0; a < 2; ++a)
#pragma unroll
        for (int b = 0; b < 2; ++b)
#pragma unroll
          for (int i = 0; i < 4; ++i)
            dots[(nt * RCD + a * 8 + 2 * q + (i & 1)) * DSTRIDE_D + acc_row(g, b, i)] = acc[a][b][i];
    }
    __syncthreads();

    // Epilogue: one warp per token; lane holds h columns 2l, 2l+1 of block j.
    const int c0 = 2 * lane;
    const float sg0 = __ldg(gsc + j * 64 + c0), sg1 = __ldg(gsc + j * 64 + c0 + 1);
    const float su0 = __ldg(usc + j * 64 + c0), su1 = __ldg(usc + j * 64 + c0 + 1);
    for (int r = warp; r < nr; r += NWARP) {
      const float ad = s_ad[r];
      float hv[2];
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int c = c0 + hh;
        const int gd = dots[((c >> 5) * RCD + r) * DSTRIDE_D + (c & 31)];
        const int ud = dots[((2 + (c >> 5)) * RCD + r) * DSTRIDE_D + (c & 31)];
        // gate and up are stored as bf16 by bq_linear, then GeGLU'd
        const float gv = bf2f(f2bf(__fmul_rn(__fmul_rn((float)gd, ad), hh ? sg1 : sg0)));
        const float uv = bf2f(f2bf(__fmul_rn(__fmul_rn((float)ud, ad), hh ? su1 : su0)));
        hv[hh] = bf2f(f2bf(__fmul_rn(gelu_tanh_f32(gv), uv)));
      }
      const size_t row = (size_t)(rbeg + r);
      if (WRITE_BF16) {
        const uint32_t pk = (uint32_t)f2bf(hv[0]) | ((uint32_t)f2bf(hv[1]) << 16);
        *reinterpret_cast<uint32_t*>(h_bf16 + row * DENSE_I + j * 64 + c0) = pk;
      }
      float v0 = hv[0], v1 = hv[1];
      {
        const float a = v0, b = v1;
        v0 = __fadd_rn(a, b);
        v1 = __fsub_rn(a, b);
      }
#pragma unroll
      for (int m = 1; m <= 16; m <<= 1) {
        v0 = fwht_xor_stage(v0, lane, m);
        v1 = fwht_xor_stage(v1, lane, m);
      }
      v0 = __fmul_rn(v0, fwht_scale_64());
      v1 = __fmul_rn(v1, fwht_scale_64());
      const float amax = warp_max(fmaxf(fabsf(v0), fabsf(v1)));
      const float qinv = amax > 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
      const uint32_t qp = (uint32_t)(quantize_i8(v0, qinv) & 0xFF) |
                          ((uint32_t)(quantize_i8(v1, qinv) & 0xFF) << 8);
      *reinterpret_cast<uint16_t*>(h_i8 + row * DENSE_I + j * 64 + c0) = (uint16_t)qp;
      if (lane == 0) h_sa[row * NB_DENSE + j] = amax;
    }
    __syncthreads();  // smem of this item fully consumed
    if (!has_next) break;
    task = nxt;
  }
}

template <int DEPTH>
__global__ void __launch_bounds__(32 * KS2, 2)
dense_down_kernel(const int8_t* __restrict__ hi8, const float* __restrict__ hsa, int T,
                  const int8_t* __restrict__ wd, const float* __restrict__ dsc,
                  uint16_t* __restrict__ out) {
  constexpr int TILES = H / 32;     // 88 hidden tiles
  constexpr int KCH = 2 * BPW2;     // 22 K chunks per warp
  extern __shared__ __align__(16) uint8_t smem[];
  int8_t* xs = reinterpret_cast<int8_t*>(smem);                               // RCD x HSTRIDE_D
  float* s_adv = reinterpret_cast<float*>(smem + RCD * HSTRIDE_D);            // [RCD][NB_DENSE]
  int* pd = reinterpret_cast<int*>(s_adv + RCD * NB_DENSE);                   // [KS2-1][BPW2][16][32]

  const int total = ((T + RCD - 1) / RCD) * TILES;
  int task = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, kw = tid >> 5;
  const int g = lane >> 2, q = lane & 3;
  auto tile_ptr = [&](int t) { return wd + (size_t)(t % TILES) * 32 * DENSE_I; };
  uint4 buf[DEPTH][2];
  // the weights are not written by the predecessor: start streaming first
  if (task < total) prefetch_chunks<DEPTH>(buf, tile_ptr(task), kw * KCH, g, q);
  pdl_wait();
  pdl_trigger();
  if (task >= total) return;

  while (true) {
    const int tile = task % TILES, rbeg = (task / TILES) * RCD;
    const int nr = min(RCD, T - rbeg);
    for (int i = tid; i < nr * (DENSE_I / 16); i += blockDim.x) {
      const int r = i / (DENSE_I / 16), c = i % (DENSE_I / 16);
      cp_async16(xs + r * HSTRIDE_D + c * 16, hi8 + (size_t)(rbeg + r) * DENSE_I + c * 16);
    }
    for (int i = tid; i < nr * NB_DENSE; i += blockDim.x)
      s_adv[i] = __fmul_rn(hsa[(size_t)rbeg * NB_DENSE + i], INV127);
    cp_async_wait_all();
    __syncthreads();

    const int8_t* wt = tile_ptr(task);
    const bool two_groups = nr > 8;
    int iacc[2][2][4];
    float facc[2][2][4];
#pragma unroll
    for (int a = 0; a < 2; ++a)
#pragma unroll
      for (int b = 0; b < 2; ++b)
#pragma unroll
        for (int i = 0; i < 4; ++i) { iacc[a][b][i] = 0; facc[a][b][i] = 0.0f; }

#pragma unroll
    for (int c = 0; c < KCH; ++c) {
      const uint4 A = buf[c % DEPTH][0], B = buf[c % DEPTH][1];
      if (c + DEPTH < KCH) {
        const int gc = kw * KCH + c + DEPTH;
        const int8_t* p = wt + (gc >> 1) * 2048 + vnni_lane_off(g, q, gc & 1);
        buf[c % DEPTH][0] = ldg_stream(p);
        buf[c % DEPTH][1] = ldg_stream(p + 256);
      }
      const int k0 = (kw * KCH + c) * 32;
      {
        const int8_t* xr = xs + g * HSTRIDE_D + k0 + 4 * q;
        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(xr);
        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(xr + 16);
        mma_s8(iacc[0][0], A.x, A.y, B.x, B.y, b0, b1);
        mma_s8(iacc[0][1], A.z, A.w, B.z, B.w, b0, b1);
      }
      if (two_groups) {
        const int8_t* xr = xs + (8 + g) * HSTRIDE_D + k0 + 4 * q;
        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(xr);
        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(xr + 16);
        mma_s8(iacc[1][0], A.x, A.y, B.x, B.y, b0, b1);
        mma_s8(iacc[1][1], A.z, A.w, B.z, B.w, b0, b1);
      }
      if (c & 1) {  // K-block complete
        const int lb = c >> 1, blk = kw * BPW2 + lb;
        if (kw == 0) {  // the first warp owns the chain: facc = fma(dot_b, sa_b/127, facc)
#pragma unroll
          for (int a = 0; a < 2; ++a)
#pragma unroll
            for (int b = 0; b < 2; ++b)
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const int r = a * 8 + 2 * q + (i & 1);
                facc[a][b][i] =
                    __fmaf_rn((float)iacc[a][b][i], s_adv[r * NB_DENSE + blk], facc[a][b][i]);
              }
        } else {        // later blocks: hand the integer dots to the first warp
          int* dst = pd + ((kw - 1) * BPW2 + lb) * 16 * 32 + lane;
#pragma unroll
          for (int a = 0; a < 2; ++a)
#pragma unroll
            for (int b = 0; b < 2; ++b)
#pragma unroll
              for (int i = 0; i < 4; ++i) dst[((a * 2 + b) * 4 + i) * 32] = iacc[a][b][i];
        }
#pragma unroll
        for (int a = 0; a < 2; ++a)
#pragma unroll
          for (int b = 0; b < 2; ++b)
#pragma unroll
            for (int i = 0; i < 4; ++i) iacc[a][b][i] = 0;
      }
    }

    const int nxt = task + gridDim.x;
    const bool has_next = nxt < total;
    if (has_next) prefetch_chunks<DEPTH>(buf, tile_ptr(nxt), kw * KCH, g, q);
    __syncthreads();  // handed-over dots visible

    if (kw == 0) {
      for (int w = 1; w < KS2; ++w) {
#pragma unroll 1
        for (int lb = 0; lb < BPW2; ++lb) {
          const int blk = w * BPW2 + lb;
          const int* src = pd + ((w - 1) * BPW2 + lb) * 16 * 32 + lane;
#pragma unroll
          for (int a = 0; a < 2; ++a)
#pragma unroll
            for (int b = 0; b < 2; ++b)
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const int r = a * 8 + 2 * q + (i & 1);
                facc[a][b][i] = __fmaf_rn((float)src[((a * 2 + b) * 4 + i) * 32],
                                          s_adv[r * NB_DENSE + blk], facc[a][b][i]);
              }
        }
      }
      // out[token][n] = bf16(facc * sw[n])   (gemm.mojo:211-215)
      const float* wsc = dsc + tile * 32;
      const int rbase = 16 * (g >> 2) + 4 * (g & 3);
      float sw[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) sw[u] = __ldg(wsc + rbase + u);
#pragma unroll
      for (int a = 0; a < 2; ++a) {
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int r = a * 8 + 2 * q + hh;
          if (r < nr) {
            uint2 o;
            o.x = (uint32_t)f2bf(__fmul_rn(facc[a][0][hh], sw[0])) |
                  ((uint32_t)f2bf(__fmul_rn(facc[a][0][2 + hh], sw[1])) << 16);
            o.y = (uint32_t)f2bf(__fmul_rn(facc[a][1][hh], sw[2])) |
                  ((uint32_t)f2bf(__fmul_rn(facc[a][1][2 + hh], sw[3])) << 16);
            *reinterpret_cast<uint2*>(out + (size_t)(rbeg + r) * H + tile * 32 + rbase) = o;
          }
        }
      }
    }
    __syncthreads();  // smem of this item fully consumed
    if (!has_next) break;
    task = nxt;
  }
}

size_t gate_up_smem(int ksplit) {
  return (size_t)RCD * XSTRIDE_D + (size_t)(ksplit - 1) * 4 * 16 * 32 * 4 +
         (size_t)4 * RCD * DSTRIDE_D * 4 + RCD * 4;
}

constexpr size_t DOWN_SMEM = (size_t)RCD * HSTRIDE_D + (size_t)RCD * NB_DENSE * 4 +
                             (size_t)(KS2 - 1) * BPW2 * 16 * 32 * 4;

int sm_count() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

template <typename K>
int fill_grid(K kern, int threads, size_t smem, int items) {
  int per_sm = 1;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, smem);
  per_sm = std::max(per_sm, 1);
  return std::max(1, std::min(items, per_sm * sm_count()));
}

}  // namespace

cudaError_t launch_dense_gate_up(const int8_t* xi8, const float* xsa, int T, const int8_t* wg,
                                 const float* gsc, const int8_t* wu, const float* usc,
                                 int8_t* h_i8, float* h_sa, uint16_t* h_bf16, cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  constexpr int KSPLIT = 4, DEPTH = 4;
  const size_t smem = gate_up_smem(KSPLIT);
  auto k = h_bf16 ? dense_gate_up_kernel<KSPLIT, DEPTH, true> : dense_gate_up_kernel<KSPLIT, DEPTH, false>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const int items = ((T + RCD - 1) / RCD) * NB_DENSE;
  const int grid = fill_grid(k, 128 * KSPLIT, smem, items);
  return launch_k(k, dim3(grid), dim3(128 * KSPLIT), smem, s, xi8, xsa, T, wg, gsc, wu, usc, h_i8,
                  h_sa, h_bf16);
}

cudaError_t launch_dense_down(const int8_t* hi8, const float* hsa, int T, const int8_t* wd,
                              const float* dsc, uint16_t* out, cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  constexpr int DEPTH = 4;
  auto k = dense_down_kernel<DEPTH>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)DOWN_SMEM);
  if (e != cudaSuccess) return e;
  const int items = ((T + RCD - 1) / RCD) * (H / 32);
  const int grid = fill_grid(k, 32 * KS2, DOWN_SMEM, items);
  return launch_k(k, dim3(grid), dim3(32 * KS2), DOWN_SMEM, s, hi8, hsa, T, wd, dsc, out);
}

}  // namespace gm
