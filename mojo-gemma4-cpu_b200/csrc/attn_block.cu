// attn_block.cu -- the products of the butterquant attention block around the
// attention core (modeling/gemma_4_moe_bq.mojo:418-627):
//
//  * bq_linear (butterquant_kernels/linear.mojo:86-150, butterquant/gemm.mojo:
//    115-143): out[t][n] = bf16((f32(iacc) - 128*colsum[n]) * (sa[t]/127) *
//    sw[n]) over the K = 2816 FWHT-128 activation; dispatch_bq_qkv
//    (linear.mojo:273-328) runs it for the q, k and v projections of one
//    attention layer over the same activation, in one launch here.
//  * block quant (butterquant/runtime.mojo:62-79 prepare_block_activation
//    [block, apply_fwht]): per block of `block` columns, optional FWHT, absmax,
//    int8 = clamp(roundeven(v*127/amax)), sa = amax.  The attention output is
//    quantised per head (block = head_dim, no FWHT: it is already in the
//    FWHT-rotated basis of the cache).
//  * block linear (butterquant/gemm.mojo:174-216 gemm_i8_per_block_panel):
//    out[t][n] = bf16(facc * sw[n]), facc = fma(f32(iacc_b) - 128*cs[b][n],
//    sa[t][b]/127, facc) over the k/block blocks in order; the attention
//    output projection (o_proj, FWHT-rotated per head block,
//    PlainPerRowBlockCs[head_dim], modeling/gemma_4_moe_bq.mojo:96-120).
//
// Weights stay in the reference's VNNI-packed layout and stream from HBM into
// mma.m16n8k32 fragments (vnni_stream.cuh), exactly as the dense MLP's kernels
// (dense_bq.cu) do; the dots are signed x signed, equal to the reference's
// u8 x s8 - 128*colsum.  Work items are (16-token chunk, weight tile group),
// so the weights are read once per 16 tokens: HBM-bound for decode batches.
#include "gm_kernels.h"
#include "vnni_stream.cuh"

namespace gm {

namespace {

constexpr int RCA = 16;             // tokens per work item
constexpr int XSTRIDE_A = H + 16;   // staged activation row (bytes)
constexpr int DSTR = 33;            // padded row stride of the dot tile

// ---------------------------------------------------------------- bq_linear
// Up to three products over the same activation.  Item = (token chunk, group
// of 4 consecutive 32-row tiles of one product); warp (nt, kh) computes tile
// nt of the group over K quarter kh, the quarters' integer dots are summed
// through shared memory, then one warp per token writes the group's 128
// outputs.
struct LinearSeg {
  const int8_t* w;       // VNNI-packed [n_rows][2816]
  const float* scale;    // [n_rows]
  uint16_t* out;         // bf16 [T][n_rows]
  int n_rows;            // multiple of 32
  int groups;            // ceil(n_rows / 128)
};
struct LinearSegs {
  LinearSeg s[3];
  int nseg;
  int groups;            // total tile groups
};

template <int DEPTH>
__global__ void __launch_bounds__(512, 2)
bq_linear_kernel(const int8_t* __restrict__ xi8, const float* __restrict__ xsa, int T,
                 const __grid_constant__ LinearSegs segs) {
  constexpr int KSPLIT = 4;
  constexpr int KCH = (H / 32) / KSPLIT;  // 22 K chunks of 32 per warp
  static_assert(KCH >= DEPTH, "prefetch depth");
  extern __shared__ __align__(16) uint8_t smem[];
  int8_t* xs = reinterpret_cast<int8_t*>(smem);                           // RCA x XSTRIDE_A
  int* red = reinterpret_cast<int*>(smem + RCA * XSTRIDE_A);              // [(KSPLIT-1)*4][16][32]
  int* dots = red + (KSPLIT - 1) * 4 * 16 * 32;                           // [4][RCA][DSTR]
  float* s_ad = reinterpret_cast<float*>(dots + 4 * RCA * DSTR);          // [RCA]

  const int total = ((T + RCA - 1) / RCA) * segs.groups;
  int task = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, q = lane & 3;
  const int nt = warp & 3, kh = warp >> 2;
  // (segment, first tile) of a group index
  auto locate = [&](int grp, int& seg, int& tile0) {
    seg = 0;
    while (seg + 1 < segs.nseg && grp >= segs.s[seg].groups) grp -= segs.s[seg++].groups;
    tile0 = grp * 4;
  };
  auto tile_ptr = [&](int t, bool& ok) -> const int8_t* {
    int seg, tile0;
    locate(t % segs.groups, seg, tile0);
    const int tile = tile0 + nt;
    ok = tile * 32 < segs.s[seg].n_rows;
    return segs.s[seg].w + (size_t)(ok ? tile : 0) * 32 * H;
  };
  uint4 buf[DEPTH][2];
  // the weights are not written by the predecessor: start streaming first
  if (task < total) {
    bool ok;
    prefetch_chunks<DEPTH>(buf, tile_ptr(task, ok), kh * KCH, g, q);
  }
  pdl_wait();
  pdl_trigger();
  if (task >= total) return;

  while (true) {
    int seg, tile0;
    locate(task % segs.groups, seg, tile0);
    const LinearSeg& S = segs.s[seg];
    const int rbeg = (task / segs.groups) * RCA;
    const int nr = min(RCA, T - rbeg);
    if (tid < nr) s_ad[tid] = __fmul_rn(xsa[rbeg + tid], INV127);
    // rows >= nr feed only B columns whose results are never stored
    for (int i = tid; i < nr * (H / 16); i += blockDim.x) {
      const int r = i / (H / 16), c = i % (H / 16);
      cp_async16(xs + r * XSTRIDE_A + c * 16, xi8 + (size_t)(rbeg + r) * H + c * 16);
    }
    cp_async_wait_all();
    __syncthreads();

    bool tile_ok;
    const int8_t* wt = tile_ptr(task, tile_ok);
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
        const int8_t* xr = xs + g * XSTRIDE_A + k0 + 4 * q;
        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(xr);
        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(xr + 16);
        mma_s8(acc[0][0], A.x, A.y, B.x, B.y, b0, b1);
        mma_s8(acc[0][1], A.z, A.w, B.z, B.w, b0, b1);
      }
      if (two_groups) {
        const int8_t* xr = xs + (8 + g) * XSTRIDE_A + k0 + 4 * q;
        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(xr);
        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(xr + 16);
        mma_s8(acc[1][0], A.x, A.y, B.x, B.y, b0, b1);
        mma_s8(acc[1][1], A.z, A.w, B.z, B.w, b0, b1);
      }
    }

    const int nxt = task + gridDim.x;
    const bool has_next = nxt < total;
    if (has_next) {
      bool ok;
      prefetch_chunks<DEPTH>(buf, tile_ptr(nxt, ok), kh * KCH, g, q);
    }

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
            dots[(nt * RCA + a * 8 + 2 * q + (i & 1)) * DSTR + acc_row(g, b, i)] = acc[a][b][i];
    }
    __syncthreads();

    // one warp per token; lane l writes rows 4l..4l+3 of the group (gemm.mojo:
    // 136-143: (corr * (sa/127)) * sw, stored as bf16)
    const int rows_here = min(128, S.n_rows - tile0 * 32);
    const int c0 = 4 * lane;
    if (c0 < rows_here) {
      float sw[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) sw[u] = __ldg(S.scale + tile0 * 32 + c0 + u);
      for (int r = warp; r < nr; r += 16) {
        const float ad = s_ad[r];
        uint16_t o[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int c = c0 + u;
          const int d = dots[((c >> 5) * RCA + r) * DSTR + (c & 31)];
          o[u] = f2bf(__fmul_rn(__fmul_rn((float)d, ad), sw[u]));
        }
        *reinterpret_cast<uint2*>(S.out + (size_t)(rbeg + r) * S.n_rows + tile0 * 32 + c0) =
            make_uint2((uint32_t)o[0] | ((uint32_t)o[1] << 16), (uint32_t)o[2] | ((uint32_t)o[3] << 16));
      }
    }
    __syncthreads();  // smem of this item fully consumed
    if (!has_next) break;
    task = nxt;
  }
}

// ---------------------------------------------------------------- block quant
// One warp per (row, block); lane l holds elements [l*V, l*V + V) of the block
// (V = block/32).  FWHT (block 64 only) as block_quant_kernel of act_quant.cu.
template <int BLOCK, bool FWHT>
__global__ void __launch_bounds__(256)
block_quant_ex_kernel(const uint16_t* __restrict__ src, long rows, int cols, int8_t* __restrict__ qi8,
                      float* __restrict__ sa) {
  constexpr int V = BLOCK / 32;
  static_assert(!FWHT || BLOCK == 64, "FWHT is applied to 64-wide blocks");
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int nb = cols / BLOCK;
  const long item = (long)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (item >= rows * nb) return;
  const long r = item / nb;
  const int b = (int)(item % nb);
  const uint16_t* p = src + r * cols + (long)b * BLOCK + lane * V;
  float v[V];
#pragma unroll
  for (int j = 0; j < V; ++j) v[j] = bf2f(p[j]);
  if constexpr (FWHT) {
    const float a = v[0], c = v[1];
    v[0] = __fadd_rn(a, c);
    v[1] = __fsub_rn(a, c);
#pragma unroll
    for (int m = 1; m <= 16; m <<= 1) {
      v[0] = fwht_xor_stage(v[0], lane, m);
      v[1] = fwht_xor_stage(v[1], lane, m);
    }
    v[0] = __fmul_rn(v[0], fwht_scale_64());
    v[1] = __fmul_rn(v[1], fwht_scale_64());
  }
  float amax = 0.0f;
#pragma unroll
  for (int j = 0; j < V; ++j) amax = fmaxf(amax, fabsf(v[j]));
  amax = warp_max(amax);
  const float qinv = amax > 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
  int8_t* d = qi8 + r * cols + (long)b * BLOCK + lane * V;
#pragma unroll
  for (int j = 0; j < V; ++j) d[j] = (int8_t)quantize_i8(v[j], qinv);
  if (lane == 0) sa[r * nb + b] = amax;
}

// ---------------------------------------------------------------- block linear
// Item = (16-token chunk, 32-row output tile); warp w of BL_WARPS (4, or 3
// when the block count is not a multiple of 4) takes the contiguous K blocks
// [w*BPW, (w+1)*BPW).  Warp 0 runs the fma chain over its own blocks while it
// streams them; the later warps hand their per-block integer dots to it
// through shared memory, and it continues the chain in block order.
template <int BLOCK, int DEPTH, int BL_WARPS>
__global__ void __launch_bounds__(32 * BL_WARPS, 1)
block_linear_kernel(const int8_t* __restrict__ hi8, const float* __restrict__ hsa, int T, int k,
                    const int8_t* __restrict__ w, const float* __restrict__ wsc, int n_rows,
                    uint16_t* __restrict__ out) {
  constexpr int CPB = BLOCK / 32;  // K chunks of 32 per block
  extern __shared__ __align__(16) uint8_t smem[];
  const int nb = k / BLOCK, bpw = nb / BL_WARPS, kch = bpw * CPB;
  const int xstride = k + 16;
  int8_t* xs = reinterpret_cast<int8_t*>(smem);                               // RCA x xstride
  float* s_adv = reinterpret_cast<float*>(smem + (size_t)RCA * xstride);       // [RCA][nb]
  int* pd = reinterpret_cast<int*>(s_adv + RCA * nb);                         // [BL_WARPS-1][bpw][16][32]

  const int tiles = n_rows / 32;
  const int total = ((T + RCA - 1) / RCA) * tiles;
  int task = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, kw = tid >> 5;
  const int g = lane >> 2, q = lane & 3;
  auto tile_ptr = [&](int t) { return w + (size_t)(t % tiles) * 32 * k; };
  uint4 buf[DEPTH][2];
  if (task < total) prefetch_chunks<DEPTH>(buf, tile_ptr(task), kw * kch, g, q);
  pdl_wait();
  pdl_trigger();
  if (task >= total) return;

  while (true) {
    const int tile = task % tiles, rbeg = (task / tiles) * RCA;
    const int nr = min(RCA, T - rbeg);
    for (int i = tid; i < nr * (k / 16); i += blockDim.x) {
      const int r = i / (k / 16), c = i % (k / 16);
      cp_async16(xs + (size_t)r * xstride + c * 16, hi8 + (size_t)(rbeg + r) * k + c * 16);
    }
    for (int i = tid; i < nr * nb; i += blockDim.x) s_adv[i] = __fmul_rn(hsa[(size_t)rbeg * nb + i], INV127);
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

    for (int c = 0; c < kch; ++c) {
      const int slot = c % DEPTH;
      uint4 A, B;
#pragma unroll
      for (int d = 0; d < DEPTH; ++d)
        if (d == slot) { A = buf[d][0]; B = buf[d][1]; }
      if (c + DEPTH < kch) {
        const int gc = kw * kch + c + DEPTH;
        const int8_t* p = wt + (gc >> 1) * 2048 + vnni_lane_off(g, q, gc & 1);
        const uint4 n0 = ldg_stream(p), n1 = ldg_stream(p + 256);
#pragma unroll
        for (int d = 0; d < DEPTH; ++d)
          if (d == slot) { buf[d][0] = n0; buf[d][1] = n1; }
      }
      const int k0 = (kw * kch + c) * 32;
      {
        const int8_t* xr = xs + g * xstride + k0 + 4 * q;
        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(xr);
        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(xr + 16);
        mma_s8(iacc[0][0], A.x, A.y, B.x, B.y, b0, b1);
        mma_s8(iacc[0][1], A.z, A.w, B.z, B.w, b0, b1);
      }
      if (two_groups) {
        const int8_t* xr = xs + (8 + g) * xstride + k0 + 4 * q;
        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(xr);
        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(xr + 16);
        mma_s8(iacc[1][0], A.x, A.y, B.x, B.y, b0, b1);
        mma_s8(iacc[1][1], A.z, A.w, B.z, B.w, b0, b1);
      }
      if ((c + 1) % CPB == 0) {  // K block complete
        const int lb = c / CPB, blk = kw * bpw + lb;
        if (kw == 0) {  // the first warp owns the chain: facc = fma(dot_b, sa_b/127, facc)
#pragma unroll
          for (int a = 0; a < 2; ++a)
#pragma unroll
            for (int b = 0; b < 2; ++b)
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const int r = a * 8 + 2 * q + (i & 1);
                facc[a][b][i] = __fmaf_rn((float)iacc[a][b][i], s_adv[r * nb + blk], facc[a][b][i]);
              }
        } else {
          int* dst = pd + ((size_t)(kw - 1) * bpw + lb) * 16 * 32 + lane;
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
    if (has_next) prefetch_chunks<DEPTH>(buf, tile_ptr(nxt), kw * kch, g, q);
    __syncthreads();  // handed-over dots visible

    if (kw == 0) {
      for (int wv = 1; wv < BL_WARPS; ++wv) {
        for (int lb = 0; lb < bpw; ++lb) {
          const int blk = wv * bpw + lb;
          const int* src = pd + ((size_t)(wv - 1) * bpw + lb) * 16 * 32 + lane;
#pragma unroll
          for (int a = 0; a < 2; ++a)
#pragma unroll
            for (int b = 0; b < 2; ++b)
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const int r = a * 8 + 2 * q + (i & 1);
                facc[a][b][i] =
                    __fmaf_rn((float)src[((a * 2 + b) * 4 + i) * 32], s_adv[r * nb + blk], facc[a][b][i]);
              }
        }
      }
      // out[token][n] = bf16(facc * sw[n])   (gemm.mojo:211-215)
      const int rbase = 16 * (g >> 2) + 4 * (g & 3);
      float sw[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) sw[u] = __ldg(wsc + tile * 32 + rbase + u);
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
            *reinterpret_cast<uint2*>(out + (size_t)(rbeg + r) * n_rows + tile * 32 + rbase) = o;
          }
        }
      }
    }
    __syncthreads();  // smem of this item fully consumed
    if (!has_next) break;
    task = nxt;
  }
}

int num_sms_ab() {
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
int grid_for(K kern, int threads, size_t smem, int items) {
  int per_sm = 1;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, smem);
  per_sm = std::max(per_sm, 1);
  return std::max(1, std::min(items, per_sm * num_sms_ab()));
}

}  // namespace

cudaError_t launch_bq_linear_multi(const int8_t* xi8, const float* xsa, int T, int nseg,
                                   const int8_t* const* w, const float* const* scale, uint16_t* const* out,
                                   const int* n_rows, cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  if (nseg < 1 || nseg > 3) return cudaErrorInvalidValue;
  LinearSegs segs = {};
  segs.nseg = nseg;
  for (int i = 0; i < nseg; ++i) {
    if (n_rows[i] <= 0 || n_rows[i] % 32) return cudaErrorInvalidValue;
    segs.s[i] = LinearSeg{w[i], scale[i], out[i], n_rows[i], (n_rows[i] + 127) / 128};
    segs.groups += segs.s[i].groups;
  }
  constexpr int DEPTH = 4;
  constexpr size_t smem = (size_t)RCA * XSTRIDE_A + (size_t)3 * 4 * 16 * 32 * 4 + (size_t)4 * RCA * DSTR * 4 +
                          RCA * 4;
  auto k = bq_linear_kernel<DEPTH>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const int items = ((T + RCA - 1) / RCA) * segs.groups;
  const int grid = grid_for(k, 512, smem, items);
  return launch_k(k, dim3(grid), dim3(512), smem, s, xi8, xsa, T, segs);
}

cudaError_t launch_block_quant_ex(const uint16_t* src, long rows, int cols, int block, int fwht,
                                  int8_t* qi8, float* sa, cudaStream_t s) {
  if (rows <= 0) return cudaSuccess;
  if (block <= 0 || cols % block) return cudaErrorInvalidValue;
  const long items = rows * (cols / block);
  const dim3 grid((unsigned)((items + 7) / 8)), blk(256);
  if (fwht) {
    if (block != 64) return cudaErrorInvalidValue;
    return launch_k(block_quant_ex_kernel<64, true>, grid, blk, 0, s, src, rows, cols, qi8, sa);
  }
  switch (block) {
    case 64: return launch_k(block_quant_ex_kernel<64, false>, grid, blk, 0, s, src, rows, cols, qi8, sa);
    case 128: return launch_k(block_quant_ex_kernel<128, false>, grid, blk, 0, s, src, rows, cols, qi8, sa);
    case 256: return launch_k(block_quant_ex_kernel<256, false>, grid, blk, 0, s, src, rows, cols, qi8, sa);
    case 512: return launch_k(block_quant_ex_kernel<512, false>, grid, blk, 0, s, src, rows, cols, qi8, sa);
    default: return cudaErrorInvalidValue;
  }
}

size_t block_linear_smem(int k, int block, int warps) {
  const int nb = k / block;
  return (size_t)RCA * (k + 16) + (size_t)RCA * nb * 4 + (size_t)(warps - 1) * (nb / warps) * 16 * 32 * 4;
}

cudaError_t launch_block_linear_ex(const int8_t* hi8, const float* hsa, int T, int k, int block,
                                   const int8_t* w, const float* wsc, int n_rows, uint16_t* out,
                                   cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  if (block <= 0 || k % block || n_rows <= 0 || n_rows % 32 || k % 64) return cudaErrorInvalidValue;
  const int nb = k / block;
  // K split over as many warps as the block count allows (16 for the output
  // projections, whose 16 head blocks give one block per warp): more weight
  // loads in flight per SM, and the token chunk staged by more threads
  const int warps = nb % 16 == 0 ? 16 : nb % 8 == 0 ? 8 : nb % 4 == 0 ? 4 : nb % 3 == 0 ? 3 : 0;
  if (!warps) return cudaErrorInvalidValue;
  const size_t smem = block_linear_smem(k, block, warps);
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  const int items = ((T + RCA - 1) / RCA) * (n_rows / 32);
  auto run = [&](auto kern) -> cudaError_t {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    const int grid = grid_for(kern, 32 * warps, smem, items);
    return launch_k(kern, dim3(grid), dim3(32 * warps), smem, s, hi8, hsa, T, k, w, wsc, n_rows, out);
  };
  if (warps == 16) {
    switch (block) {
      case 64: return run(block_linear_kernel<64, 4, 16>);
      case 128: return run(block_linear_kernel<128, 4, 16>);
      case 256: return run(block_linear_kernel<256, 4, 16>);
      case 512: return run(block_linear_kernel<512, 4, 16>);
      default: return cudaErrorInvalidValue;
    }
  }
  if (warps == 8) {
    switch (block) {
      case 64: return run(block_linear_kernel<64, 4, 8>);
      case 128: return run(block_linear_kernel<128, 4, 8>);
      case 256: return run(block_linear_kernel<256, 4, 8>);
      case 512: return run(block_linear_kernel<512, 4, 8>);
      default: return cudaErrorInvalidValue;
    }
  }
  if (warps == 4) {
    switch (block) {
      case 64: return run(block_linear_kernel<64, 4, 4>);
      case 128: return run(block_linear_kernel<128, 4, 4>);
      case 256: return run(block_linear_kernel<256, 4, 4>);
      case 512: return run(block_linear_kernel<512, 4, 4>);
      default: return cudaErrorInvalidValue;
    }
  }
  switch (block) {
    case 64: return run(block_linear_kernel<64, 4, 3>);
    case 128: return run(block_linear_kernel<128, 4, 3>);
    case 256: return run(block_linear_kernel<256, 4, 3>);
    case 512: return run(block_linear_kernel<512, 4, 3>);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace gm
