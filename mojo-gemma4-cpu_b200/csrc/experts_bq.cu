// experts_bq.cu -- butterquant expert products streamed from the reference's
// VNNI-packed int8 layout.
//
// Reference:
//  * phase 1 (butterquant_kernels/moe.mojo:26-129): per expert, per 32-row
//    intermediate tile, iacc = sum_k u8(x)*s8(w) (butterquant/gemm.mojo:36-75),
//    val = (iacc - 128*colsum)*(sa/127)*sw, bucket = bf16(gelu_tanh(g)*u);
//    then dispatch_bq_block_quant (butterquant_kernels/linear.mojo:182-205):
//    FWHT-64 + per-64-block int8 of the bucket.
//  * phase 2 (butterquant_kernels/moe.mojo:168-295): per record and 32-row
//    hidden tile, facc = fma(iacc_b - 128*cs[b], sa[b]/127, facc) over the 11
//    K-blocks, res = facc*sw*route_weight, accumulated per token.
//
// B200 shape.  The packed layout (butterquant/vnni.mojo:31-83: per 32-row
// N-tile and 64-col K-step a 2048-byte tile, two 16-row halves, byte
// (k/4)*64 + n*4 + k%4) is streamed as-is with 128-bit no-L1 loads.  One lane
// load returns one 4-byte K-group for 4 consecutive rows; two such loads (K
// groups q and q+4 of a 32-wide K chunk) are exactly the A fragments of two
// mma.m16n8k32 s8 tiles whose logical rows are permuted physical rows, so the
// weights go from HBM to the tensor core without a shared-memory transpose.
// The activations (<=16 routed rows per work item) sit in shared memory as the
// B operand.  The dot is signed x signed, which equals the reference's
// u8 x s8 - 128*colsum identity (quantization_docs/butterquant.md 1.4, 2.5), so
// the colsum is not read.
//
// Work items: (expert, chunk of <=16 routes, output block).  The kernels are
// persistent: each CTA walks a strided list of work items and issues the first
// weight loads of its next item before the reduction/epilogue of the current
// one, so the HBM stream does not drain between items.  Phase 1's epilogue
// holds the 64 gate and 64 up outputs of one FWHT-64 block for every route, so
// GeGLU, the bf16 rounding of the bucket, FWHT-64 and the per-block int8
// quantisation run in registers and only bucket_i8/bucket_sa reach HBM.
// Phase 2 writes per-route f32 rows y = facc*sw*w; combine.cu sums them per
// token in ascending expert order (the reference's accumulation order).
#include "gm_kernels.h"
#include "vnni_stream.cuh"

namespace gm {

constexpr int RC_BQ = 16;                 // routes per work item
constexpr int XSTRIDE = H + 16;           // staged activation row (bytes)
constexpr int BSTRIDE = I + 16;           // staged bucket row (bytes)
constexpr int DSTRIDE = 33;               // padded row stride of the phase-1 dot tile

struct Task {
  int e, rbeg, nr, blk;
};

// Work item `task` of a kernel whose items are (route chunk, blk) with
// `per_chunk` output blocks per route chunk.
__device__ __forceinline__ bool decode_task(int task, int total, int per_chunk,
                                            const int32_t* __restrict__ chunk_off,
                                            const int32_t* __restrict__ expert_offset, int epr,
                                            Task& t) {
  if (task >= total) return false;
  const int cg = task / per_chunk;
  t.blk = task % per_chunk;
  t.e = find_segment(chunk_off, epr, cg);
  t.rbeg = __ldg(expert_offset + t.e) + (cg - __ldg(chunk_off + t.e)) * RC_BQ;
  t.nr = min(RC_BQ, __ldg(expert_offset + t.e + 1) - t.rbeg);
  return true;
}

__device__ __forceinline__ const int8_t* p1_tile(const int8_t* w_gu, const Task& t, int nt) {
  const int tile = (nt < 2) ? (2 * t.blk + nt) : (I / 32 + 2 * t.blk + (nt - 2));
  return w_gu + (size_t)t.e * GU * H + (size_t)tile * 32 * H;
}

template <int KSPLIT, int DEPTH, bool WRITE_BF16>
__global__ void __launch_bounds__(128 * KSPLIT, 2)
bq_phase1_kernel(const int8_t* __restrict__ xi8, const float* __restrict__ xsa,
                 const int32_t* __restrict__ expert_offset, const SparseRoute* __restrict__ routes,
                 const int32_t* __restrict__ chunk_off, int epr,
                 const int8_t* __restrict__ w_gu, const float* __restrict__ gu_scale,
                 int8_t* __restrict__ bucket_i8, float* __restrict__ bucket_sa,
                 uint16_t* __restrict__ bucket_bf16) {
  constexpr int NWARP = 4 * KSPLIT;
  constexpr int KCH = (H / 32) / KSPLIT;  // 32-wide K chunks per warp
  static_assert(KCH >= DEPTH, "prefetch depth");
  extern __shared__ __align__(16) uint8_t smem[];
  int8_t* xs = reinterpret_cast<int8_t*>(smem);                              // RC x XSTRIDE
  int* red = reinterpret_cast<int*>(smem + RC_BQ * XSTRIDE);                 // [(KSPLIT-1)*4][16][32]
  int* dots = red + (KSPLIT - 1) * 4 * 16 * 32;                              // [4][RC][DSTRIDE]
  float* s_ad = reinterpret_cast<float*>(dots + 4 * RC_BQ * DSTRIDE);        // [RC]
  int* s_tok = reinterpret_cast<int*>(s_ad + RC_BQ);                         // [RC]

  pdl_wait();
  pdl_trigger();
  const int total = __ldg(chunk_off + epr) * NB_DOWN;
  int task = blockIdx.x;
  Task cur;
  if (!decode_task(task, total, NB_DOWN, chunk_off, expert_offset, epr, cur)) return;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, q = lane & 3;
  const int nt = warp & 3, kh = warp >> 2;

  uint4 buf[DEPTH][2];
  prefetch_chunks<DEPTH>(buf, p1_tile(w_gu, cur, nt), kh * KCH, g, q);

  while (true) {
    const int nr = cur.nr, rbeg = cur.rbeg, j = cur.blk;
    // Stage the nr routed activation rows with asynchronous copies (rows >= nr
    // feed only B columns whose results are never stored).
    if (tid < nr) {
      const int tok = routes[rbeg + tid].token;
      s_tok[tid] = tok;
      s_ad[tid] = __fmul_rn(xsa[tok], INV127);
    }
    __syncthreads();
    for (int i = tid; i < nr * (H / 16); i += blockDim.x) {
      const int r = i / (H / 16), c = i % (H / 16);
      cp_async16(xs + r * XSTRIDE + c * 16, xi8 + (size_t)s_tok[r] * H + c * 16);
    }
    cp_async_wait_all();
    __syncthreads();

    const int8_t* wt = p1_tile(w_gu, cur, nt);
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
        const int8_t* xr = xs + g * XSTRIDE + k0 + 4 * q;
        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(xr);
        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(xr + 16);
        mma_s8(acc[0][0], A.x, A.y, B.x, B.y, b0, b1);
        mma_s8(acc[0][1], A.z, A.w, B.z, B.w, b0, b1);
      }
      if (two_groups) {
        const int8_t* xr = xs + (8 + g) * XSTRIDE + k0 + 4 * q;
        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(xr);
        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(xr + 16);
        mma_s8(acc[1][0], A.x, A.y, B.x, B.y, b0, b1);
        mma_s8(acc[1][1], A.z, A.w, B.z, B.w, b0, b1);
      }
    }

    // Keep HBM busy: the next item's first chunks are in flight during the
    // reduction and epilogue below.
    Task nxt;
    const bool has_next =
        decode_task(task + gridDim.x, total, NB_DOWN, chunk_off, expert_offset, epr, nxt);
    if (has_next) prefetch_chunks<DEPTH>(buf, p1_tile(w_gu, nxt, nt), kh * KCH, g, q);

    // K-split reduction (integer, order-free) into dots[tile][route][row];
    // partials are stored register-major ([slot][lane]) so lanes hit distinct banks.
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
            dots[(nt * RC_BQ + a * 8 + 2 * q + (i & 1)) * DSTRIDE + acc_row(g, b, i)] = acc[a][b][i];
    }
    __syncthreads();

    // Epilogue: one warp per route; lane holds bucket columns 2l, 2l+1 of block j.
    const float* wsc = gu_scale + (size_t)cur.e * GU;
    const int c0 = 2 * lane;
    const float sg0 = __ldg(wsc + j * 64 + c0), sg1 = __ldg(wsc + j * 64 + c0 + 1);
    const float su0 = __ldg(wsc + I + j * 64 + c0), su1 = __ldg(wsc + I + j * 64 + c0 + 1);
    for (int r = warp; r < nr; r += NWARP) {
      const float ad = s_ad[r];
      float hv[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int c = c0 + h;
        const int gd = dots[((c >> 5) * RC_BQ + r) * DSTRIDE + (c & 31)];
        const int ud = dots[((2 + (c >> 5)) * RC_BQ + r) * DSTRIDE + (c & 31)];
        const float gv = __fmul_rn(__fmul_rn((float)gd, ad), h ? sg1 : sg0);
        const float uv = __fmul_rn(__fmul_rn((float)ud, ad), h ? su1 : su0);
        hv[h] = bf2f(f2bf(__fmul_rn(gelu_tanh_f32(gv), uv)));
      }
      const size_t row = (size_t)(rbeg + r);
      if (WRITE_BF16) {
        const uint32_t pk = (uint32_t)f2bf(hv[0]) | ((uint32_t)f2bf(hv[1]) << 16);
        *reinterpret_cast<uint32_t*>(bucket_bf16 + row * I + j * 64 + c0) = pk;
      }
      // FWHT-64 (stride 1 in registers, 2..32 across lanes), per-block int8.
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
      *reinterpret_cast<uint16_t*>(bucket_i8 + row * I + j * 64 + c0) = (uint16_t)qp;
      if (lane == 0) bucket_sa[row * NB_DOWN + j] = amax;
    }
    __syncthreads();  // smem of this item fully consumed
    if (!has_next) break;
    cur = nxt;
    task += gridDim.x;
  }
}

// `prologue_prefetch`: the schedule (two launches back) is complete when the
// kernel starts, so the first weight chunks are issued before waiting for
// phase 1's bucket.  Only the fused forward sets it (it always runs phase 1
// between the schedule and this kernel).
template <int NTILE, int DEPTH>
__global__ void __launch_bounds__(32 * NTILE, 4)
bq_phase2_kernel(const int8_t* __restrict__ bi8, const float* __restrict__ bsa,
                 const int32_t* __restrict__ expert_offset, const SparseRoute* __restrict__ routes,
                 const int32_t* __restrict__ chunk_off, int epr,
                 const int8_t* __restrict__ w_dn, const float* __restrict__ dn_scale,
                 float* __restrict__ ybuf, int prologue_prefetch) {
  constexpr int GROUPS = (H / 32) / NTILE;  // hidden tile groups per expert
  constexpr int KCH = I / 32;               // 22 K chunks, 2 per K-block
  __shared__ __align__(16) int8_t xs2[2][RC_BQ * BSTRIDE];
  __shared__ float s_adv2[2][RC_BQ * NB_DOWN];
  __shared__ float s_w2[2][RC_BQ];

  if (!prologue_prefetch) pdl_wait();
  const int total = __ldg(chunk_off + epr) * GROUPS;
  int task = blockIdx.x;
  Task cur;
  const bool any = decode_task(task, total, GROUPS, chunk_off, expert_offset, epr, cur);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, q = lane & 3;
  uint4 buf[DEPTH][2];
  if (any) {
    const int8_t* wt0 = w_dn + (size_t)cur.e * H * I + (size_t)(cur.blk * NTILE + warp) * 32 * I;
    prefetch_chunks<DEPTH>(buf, wt0, 0, g, q);
  }
  if (prologue_prefetch) pdl_wait();
  pdl_trigger();
  if (!any) return;
  // a task's nr bucket rows, their block scales and route weights, by
  // asynchronous copy into buffer b (the next task's while this one computes)
  auto stage = [&](const Task& tk, int b) {
    for (int i = tid; i < tk.nr * (I / 16); i += blockDim.x) {
      const int r = i / (I / 16), c = i % (I / 16);
      cp_async16(xs2[b] + r * BSTRIDE + c * 16, bi8 + (size_t)(tk.rbeg + r) * I + c * 16);
    }
    for (int i = tid; i < tk.nr * NB_DOWN; i += blockDim.x) cp_async4(&s_adv2[b][i], bsa + (size_t)tk.rbeg * NB_DOWN + i);
    if (tid < tk.nr) cp_async4(&s_w2[b][tid], &routes[tk.rbeg + tid].weight);
    cp_async_commit();
  };
  stage(cur, 0);
  int xb = 0;

  while (true) {
    const int nr = cur.nr, rbeg = cur.rbeg;
    const int tile = cur.blk * NTILE + warp;
    const int8_t* wt = w_dn + (size_t)cur.e * H * I + (size_t)tile * 32 * I;
    cp_async_wait_all();
    __syncthreads();
    const int8_t* xs = xs2[xb];
    const float* s_adv = s_adv2[xb];
    const float* s_w = s_w2[xb];

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
        const int cn = c + DEPTH;
        const int8_t* p = wt + (cn >> 1) * 2048 + vnni_lane_off(g, q, cn & 1);
        buf[c % DEPTH][0] = ldg_stream(p);
        buf[c % DEPTH][1] = ldg_stream(p + 256);
      }
      const int k0 = c * 32;
      {
        const int8_t* xr = xs + g * BSTRIDE + k0 + 4 * q;
        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(xr);
        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(xr + 16);
        mma_s8(iacc[0][0], A.x, A.y, B.x, B.y, b0, b1);
        mma_s8(iacc[0][1], A.z, A.w, B.z, B.w, b0, b1);
      }
      if (two_groups) {
        const int8_t* xr = xs + (8 + g) * BSTRIDE + k0 + 4 * q;
        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(xr);
        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(xr + 16);
        mma_s8(iacc[1][0], A.x, A.y, B.x, B.y, b0, b1);
        mma_s8(iacc[1][1], A.z, A.w, B.z, B.w, b0, b1);
      }
      if (c & 1) {  // K-block (c>>1) complete: facc = fma(dot_b, sa_b/127, facc)
        const int blk = c >> 1;
#pragma unroll
        for (int a = 0; a < 2; ++a)
#pragma unroll
          for (int b = 0; b < 2; ++b)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int r = a * 8 + 2 * q + (i & 1);
              facc[a][b][i] =
                  __fmaf_rn((float)iacc[a][b][i], __fmul_rn(s_adv[r * NB_DOWN + blk], INV127), facc[a][b][i]);
              iacc[a][b][i] = 0;
            }
      }
    }

    Task nxt;
    const bool has_next =
        decode_task(task + gridDim.x, total, GROUPS, chunk_off, expert_offset, epr, nxt);
    if (has_next) {
      const int8_t* wtn = w_dn + (size_t)nxt.e * H * I + (size_t)(nxt.blk * NTILE + warp) * 32 * I;
      prefetch_chunks<DEPTH>(buf, wtn, 0, g, q);
      stage(nxt, xb ^ 1);
    }

    // y[route][n] = facc * sw[n] * w_route  (moe.mojo:218-225)
    const float* wsc = dn_scale + (size_t)cur.e * H + tile * 32;
    const int rbase = 16 * (g >> 2) + 4 * (g & 3);
    float sw[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) sw[u] = __ldg(wsc + rbase + u);
#pragma unroll
    for (int a = 0; a < 2; ++a) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int r = a * 8 + 2 * q + h;
        if (r < nr) {
          const float wr = s_w[r];
          float4 o;
          o.x = __fmul_rn(__fmul_rn(facc[a][0][h], sw[0]), wr);
          o.y = __fmul_rn(__fmul_rn(facc[a][0][2 + h], sw[1]), wr);
          o.z = __fmul_rn(__fmul_rn(facc[a][1][h], sw[2]), wr);
          o.w = __fmul_rn(__fmul_rn(facc[a][1][2 + h], sw[3]), wr);
          *reinterpret_cast<float4*>(ybuf + (size_t)(rbeg + r) * H + tile * 32 + rbase) = o;
        }
      }
    }
    if (!has_next) break;
    cur = nxt;
    task += gridDim.x;
    xb ^= 1;
  }
}

static size_t phase1_smem(int ksplit) {
  return (size_t)RC_BQ * XSTRIDE + (size_t)(ksplit - 1) * 4 * 16 * 32 * 4 +
         (size_t)4 * RC_BQ * DSTRIDE * 4 + RC_BQ * 4 + RC_BQ * 4;
}

int max_route_chunks(int T, int epr, int rc) {
  // sum_e ceil(n_e/rc) <= floor(R/rc) + (number of non-empty experts), and
  // never more than R chunks of one route.
  const int R = T * TOPK;
  return std::min(R, R / rc + std::min(epr, R));
}

static int num_sms() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

// Bulk L2 prefetch of a byte range (no destination, no completion tracking):
// the weights phase 1 reads first are pulled into L2 while the router and the
// schedule -- latency-bound kernels that leave HBM idle -- run.  It reads
// nothing another kernel writes, so it does not wait on its predecessor.
// Prefetches n_units units of unit_bytes: unit k starts at base + (first +
// stride*k) * unit_bytes.
__global__ void __launch_bounds__(256) l2_prefetch_kernel(const uint8_t* __restrict__ base, size_t unit_bytes,
                                                         int n_units, int first, int stride) {
  pdl_trigger();
  constexpr size_t CHUNK = 32768;
  const size_t bytes = unit_bytes * (size_t)n_units;
  for (size_t off = ((size_t)blockIdx.x * blockDim.x + threadIdx.x) * CHUNK; off < bytes;
       off += (size_t)gridDim.x * blockDim.x * CHUNK) {
    const size_t k = off / unit_bytes, in = off % unit_bytes;
    const uint32_t n = (uint32_t)min((size_t)CHUNK, unit_bytes - in) & ~15u;
    const uint8_t* p = base + ((size_t)first + (size_t)stride * k) * unit_bytes + in;
    if (n) asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(n) : "memory");
  }
}

cudaError_t launch_l2_prefetch(const void* base, size_t unit_bytes, int n_units, int first, int stride,
                               cudaStream_t s) {
  if (!unit_bytes || n_units <= 0) return cudaSuccess;
  const size_t chunks = (unit_bytes * n_units + 32767) / 32768;
  const int blocks = (int)std::min<size_t>(148, (chunks + 255) / 256);
  return launch_k(l2_prefetch_kernel, dim3(blocks), dim3(256), 0, s, static_cast<const uint8_t*>(base), unit_bytes,
                  n_units, first, stride);
}

template <typename K>
static int resident_grid(K kern, int threads, size_t smem, int max_items) {
  int per_sm = 1;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, smem);
  per_sm = std::max(per_sm, 1);
  return std::max(1, std::min(max_items, per_sm * num_sms()));
}

cudaError_t launch_bq_phase1(const int8_t* xi8, const float* xsa, const int32_t* expert_offset,
                             const SparseRoute* routes, const int32_t* chunk_off, int epr, int T,
                             const int8_t* w_gu, const float* gu_scale, int8_t* bucket_i8,
                             float* bucket_sa, uint16_t* bucket_bf16, cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  constexpr int KSPLIT = 4, DEPTH = 4;
  const size_t smem = phase1_smem(KSPLIT);
  const int items = max_route_chunks(T, epr, RC_BQ) * NB_DOWN;
  auto k = bucket_bf16 ? bq_phase1_kernel<KSPLIT, DEPTH, true> : bq_phase1_kernel<KSPLIT, DEPTH, false>;
  cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  const int grid = resident_grid(k, 128 * KSPLIT, smem, items);
  return launch_k(k, dim3(grid), dim3(128 * KSPLIT), smem, s, xi8, xsa, expert_offset, routes,
                  chunk_off, epr, w_gu, gu_scale, bucket_i8, bucket_sa, bucket_bf16);
}

cudaError_t launch_bq_phase2(const int8_t* bi8, const float* bsa, const int32_t* expert_offset,
                             const SparseRoute* routes, const int32_t* chunk_off, int epr, int T,
                             const int8_t* w_dn, const float* dn_scale, float* ybuf,
                             bool after_phase1, cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  // 8 chunks (8 KB per warp) in flight: 52.2 us at 64 tokens against 54.8 with 4
  constexpr int NTILE = 4, DEPTH = 8;
  const int items = max_route_chunks(T, epr, RC_BQ) * ((H / 32) / NTILE);
  auto k = bq_phase2_kernel<NTILE, DEPTH>;
  const int grid = resident_grid(k, 32 * NTILE, 0, items);
  if (after_phase1)
    return launch_k(k, dim3(grid), dim3(32 * NTILE), 0, s, bi8, bsa, expert_offset, routes,
                    chunk_off, epr, w_dn, dn_scale, ybuf, 1);
  // standalone: an ordinary stream-ordered launch (the prologue may then read
  // the schedule before any wait)
  k<<<grid, 32 * NTILE, 0, s>>>(bi8, bsa, expert_offset, routes, chunk_off, epr, w_dn, dn_scale,
                                ybuf, 0);
  return cudaGetLastError();
}

}  // namespace gm
