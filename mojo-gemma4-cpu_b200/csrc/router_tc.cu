// router_tc.cu -- router logits for many tokens on the tcgen05 tensor cores.
//
// Same product as router_logits_small_kernel (kernels/moe_router.mojo:
// 164-191: logit = sum_k (x_k * router_scale_k) * w_k with the bf16 router
// projection; the top-8 step multiplies the sum by inv_rms), for
// T >= ROUTER_TC_MIN_TOKENS:
//
//  * s = x * router_scale is a product of two bf16, exact in f32 with at most
//    16 significant bits, so it splits exactly into two bf16 parts,
//    s = hi + lo (hi = bf16(s), lo = s - hi: the rounding residual has at most
//    8 significant bits), and a bf16 x bf16 product is exact in f32, so the
//    two kind::f16 MMAs (f32 accumulate) give the f32 dot up to the
//    accumulation order -- the same class of difference as the reference's
//    own split across workers;
//  * one CTA = 128 tokens x all 128 experts x one 256-wide K slice (the same
//    11 slices, and the same [slice][T][E] partial layout, as the FMA kernel,
//    so the top-8 kernels are shared);
//  * the kernel reads only x and the router weights, so it runs beside the
//    norm kernel launched just before it (that kernel triggers only after its
//    own wait, so x is complete); it waits for its predecessor only after its
//    stores, so its completion implies the norm kernel's (router.cu);
//  * the router slice (64 KB) is fetched with cp.async, the activation parts
//    are produced by all 256 threads into a 2-stage ring in the
//    128-byte-swizzled K-major layout the MMA descriptors read, and the TMEM
//    accumulator is staged through shared memory for coalesced stores.
//
// Every mbarrier wait is bounded (tc::mbar_wait, ~1 s); on expiry the kernel
// writes 1 into *err, skips the remaining MMAs, still frees its TMEM and
// returns.
#include "gm_kernels.h"
#include "tc_prims.cuh"

namespace gm {

namespace tc {

constexpr int RT_BM = 128;               // tokens per CTA (TMEM lanes)
constexpr int RT_KS = 256;               // K slice per CTA
constexpr int RT_BK = 64;                // bf16 per 128-byte swizzle row
constexpr int RT_NCH = RT_KS / RT_BK;    // 4 K chunks per slice
constexpr int RT_THREADS = 256;
constexpr int RT_TILE = 128 * 128;       // bytes of one [128 rows][64 bf16] operand tile
constexpr int RT_YSTR = E + 4;           // output staging row stride (floats)

// kind::f16: D = f32 (bits 4-5 = 1), A = B = bf16 (bits 7-9, 10-12 = 1), both
// K-major, N = 128 (bits 17-22 = N>>3), M = 128 (bits 24-28 = M>>4).
constexpr uint32_t IDESC_BF16 = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(E >> 3) << 17) |
                                ((uint32_t)(RT_BM >> 4) << 24);

struct RouterSmem {
  uint8_t b[RT_NCH][RT_TILE];     // router rows (experts) x 64 bf16 per chunk; 1024-aligned
  uint8_t a[2][3][RT_TILE];       // 2 stages x {hi, lo, (output staging room)} x [128 tokens][64 bf16]
  uint64_t done[2];
  uint32_t tmem_base;
  int failed;
};
static_assert(sizeof(float) * RT_BM * RT_YSTR <= sizeof(((RouterSmem*)0)->a), "staging fits in a[]");

__device__ __forceinline__ void mma_bf16_ss(uint32_t d_tmem, uint64_t da, uint64_t db, uint32_t accumulate) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }"
      ::"r"(d_tmem), "l"(da), "l"(db), "r"(IDESC_BF16), "r"(accumulate)
      : "memory");
}

// Byte offset of 16-byte unit j (0..7) of row r in a 128-byte-swizzled tile.
__device__ __forceinline__ int sw128(int r, int j) { return r * 128 + ((j ^ (r & 7)) << 4); }

__device__ __forceinline__ uint32_t pack_bf16(uint16_t lo, uint16_t hi) {
  return (uint32_t)lo | ((uint32_t)hi << 16);
}

__global__ void __launch_bounds__(RT_THREADS, 1)
router_tc_kernel(const uint16_t* __restrict__ x, const uint16_t* __restrict__ wr,
                 const uint16_t* __restrict__ rscale, int T, float* __restrict__ logits,
                 int* __restrict__ err) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  RouterSmem& s =
      *reinterpret_cast<RouterSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int t0 = blockIdx.x * RT_BM, kb = blockIdx.y * RT_KS;

  // router slice: 128 experts x 256 K = 4 chunks of [128][64] bf16
  for (int i = tid; i < E * (RT_KS / 8); i += RT_THREADS) {
    const int e = i / (RT_KS / 8), u = i % (RT_KS / 8), c = u >> 3, j = u & 7;
    cp_async16(s.b[c] + sw128(e, j), wr + (size_t)e * H + kb + u * 8);
  }
  if (tid == 0) {
    mbar_init(&s.done[0], 1);
    mbar_init(&s.done[1], 1);
    s.failed = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&s.tmem_base)),
                 "r"(128u));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;

  pdl_trigger();  // no wait before reading x: see the file comment

  // 8 consecutive router_scale values of each 16-byte unit this thread owns
  // (the unit column j = tid & 7 is the same for all 4 of its units)
  const int j = tid & 7;
  for (int c = 0; c < RT_NCH; ++c) {
    const int st = c & 1;
    if (c >= 2) mbar_wait(&s.done[st], 0, &s.failed);  // MMAs of chunk c-2 read this stage
    const int k0 = kb + c * RT_BK + j * 8;
    const uint4 rs4 = *reinterpret_cast<const uint4*>(rscale + k0);
    const uint32_t rsw[4] = {rs4.x, rs4.y, rs4.z, rs4.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int r = (tid >> 3) + q * (RT_THREADS / 8);  // token row in the tile
      const int t = t0 + r;
      uint32_t hi[4] = {0, 0, 0, 0}, lo[4] = {0, 0, 0, 0};
      if (t < T) {
        const uint4 xv = *reinterpret_cast<const uint4*>(x + (size_t)t * H + k0);
        const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          uint16_t h2[2], l2[2];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const float xs = bf2f(h ? xw[p] >> 16 : xw[p] & 0xFFFFu);
            const float ss = bf2f(h ? rsw[p] >> 16 : rsw[p] & 0xFFFFu);
            const float sv = __fmul_rn(xs, ss);                   // x*s, exact
            h2[h] = f2bf(sv);
            l2[h] = f2bf(__fsub_rn(sv, bf2f(h2[h])));             // exact residual (<= 8 bits)
          }
          hi[p] = pack_bf16(h2[0], h2[1]);
          lo[p] = pack_bf16(l2[0], l2[1]);
        }
      }
      const int off = sw128(r, j);
      *reinterpret_cast<uint4*>(s.a[st][0] + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
      *reinterpret_cast<uint4*>(s.a[st][1] + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    }
    if (c == 0) cp_async_wait_all();
    // generic-proxy shared-memory writes -> visible to the tensor core (async proxy)
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    if (tid == 0 && !*(volatile int*)&s.failed) {
      tc_fence_after();
#pragma unroll
      for (int k = 0; k < RT_BK / 16; ++k) {
        const uint64_t db = kmajor_sw128_desc(smem_u32(s.b[c]) + k * 32);
#pragma unroll
        for (int p = 0; p < 2; ++p)
          mma_bf16_ss(tmem, kmajor_sw128_desc(smem_u32(s.a[st][p]) + k * 32), db,
                      (c | k | p) != 0);
      }
      mma_commit(&s.done[st]);
    }
  }
  // chunk 2 -> second completion of done[0], chunk 3 -> second of done[1]
  mbar_wait(&s.done[0], 1, &s.failed);
  mbar_wait(&s.done[1], 1, &s.failed);
  tc_fence_after();

  // epilogue: warp w reads TMEM lanes 32*(w&3).. and columns 64*(w>>2)..,
  // stages the f32 tile in shared memory (reusing the operand ring), then
  // whole 512-byte rows are stored
  float* ystage = reinterpret_cast<float*>(&s.a[0][0][0]);
  __syncthreads();  // every thread is past its last read of the ring
  {
    const int q = warp & 3, half = warp >> 2, row = q * 32 + lane;
    float* dst = ystage + row * RT_YSTR + half * 64;
#pragma unroll
    for (int cc = 0; cc < 2; ++cc) {
      int v[32];
      tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + half * 64 + cc * 32, v);
      tmem_ld_wait();
#pragma unroll
      for (int i = 0; i < 32; i += 4)
        *reinterpret_cast<float4*>(dst + cc * 32 + i) =
            make_float4(__int_as_float(v[i]), __int_as_float(v[i + 1]), __int_as_float(v[i + 2]),
                        __int_as_float(v[i + 3]));
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(128u));
  float* out = logits + (size_t)blockIdx.y * T * E;
  for (int r = warp; r < RT_BM; r += RT_THREADS / 32) {
    const int t = t0 + r;
    if (t >= T) break;
    *reinterpret_cast<float4*>(out + (size_t)t * E + lane * 4) =
        *reinterpret_cast<const float4*>(ystage + r * RT_YSTR + lane * 4);
  }
  if (tid == 0 && *(volatile int*)&s.failed) atomicExch(err, 1);
  // this grid completes only after its predecessor (the norm kernel) has
  pdl_wait();
}

}  // namespace tc

cudaError_t launch_router_logits_tc(const uint16_t* x, const uint16_t* wr, const uint16_t* rscale, int T,
                                    float* logits, int* err, cudaStream_t s) {
  const size_t smem = sizeof(tc::RouterSmem) + 1024;
  cudaError_t e = cudaFuncSetAttribute(tc::router_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e != cudaSuccess) return e;
  return launch_k(tc::router_tc_kernel, dim3((T + tc::RT_BM - 1) / tc::RT_BM, H / tc::RT_KS),
                  dim3(tc::RT_THREADS), smem, s, x, wr, rscale, T, logits, err);
}

}  // namespace gm
