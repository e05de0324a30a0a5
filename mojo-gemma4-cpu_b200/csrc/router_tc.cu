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
//  * one CTA = 128 tokens x all 128 experts x one K slice, written as the
//    same [slice][T][E] partial layout as the FMA kernel so that the top-8
//    kernels are shared: the FMA kernel's 11 slices of 256 below
//    ROUTER_WIDE_MIN_TOKENS, 4 slices of 704 from there on (about one CTA per
//    SM at 4096 tokens, and fewer partials for the top-8 to sum);
//  * the kernel reads only x and the router weights, so it runs beside the
//    norm kernel launched just before it (that kernel triggers only after its
//    own wait, so x is complete); it waits for its predecessor only after its
//    stores, so its completion implies the norm kernel's (router.cu).  On the
//    tcgen05 prefill path the router is the forward's first kernel (the norm
//    follows the schedule there) and waits before reading x (wait_first);
//  * the router chunks (64 K each) arrive by cp.async in a 6-stage ring, two
//    chunks ahead; each thread loads its x units two chunks ahead into
//    registers; the activation parts are produced by all 256 threads (packed
//    f32x2 products and bf16x2 roundings) into a 4-stage ring in the
//    128-byte-swizzled K-major layout the MMA descriptors read, so a chunk's
//    MMAs have four chunk periods to complete before its stages are reused;
//    the TMEM accumulator is staged through shared memory for coalesced
//    stores.
//
// Every mbarrier wait is bounded (tc::mbar_wait, ~1 s); on expiry the kernel
// writes 1 into *err, skips the remaining MMAs, still frees its TMEM and
// returns.
#include "gm_kernels.h"
#include "tc_prims.cuh"

namespace gm {

namespace tc {

constexpr int RT_BM = 128;               // tokens per CTA (TMEM lanes)
constexpr int RT_BK = 64;                // bf16 per 128-byte swizzle row (one K chunk)
constexpr int RT_CHUNKS = H / RT_BK;     // 44 K chunks in all
constexpr int RT_THREADS = 256;
constexpr int RT_TILE = 128 * 128;       // bytes of one [128 rows][64 bf16] operand tile
constexpr int RT_AST = 4;                // activation (hi, lo) stages
constexpr int RT_XLA = 2;                // x chunks loaded ahead into registers
constexpr int RT_BST = RT_AST + 2;       // router chunk ring, filled two chunks ahead
// chunk c's activation stage c % RT_AST and router stage (c + 2) % RT_BST were
// both last read by the MMAs of chunk c - RT_AST
constexpr int RT_YSTR = E + 4;           // output staging row stride (floats)

// kind::f16: D = f32 (bits 4-5 = 1), A = B = bf16 (bits 7-9, 10-12 = 1), both
// K-major, N = 128 (bits 17-22 = N>>3), M = 128 (bits 24-28 = M>>4).
constexpr uint32_t IDESC_BF16 = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(E >> 3) << 17) |
                                ((uint32_t)(RT_BM >> 4) << 24);

struct RouterSmem {
  uint8_t b[RT_BST][RT_TILE];     // router rows (experts) x 64 bf16 per chunk; 1024-aligned
  uint8_t a[RT_AST][2][RT_TILE];  // RT_AST stages x {hi, lo} x [128 tokens][64 bf16]
  uint64_t done[RT_AST];          // MMAs of the chunks using A stage 0..RT_AST-1 complete
  uint32_t tmem_base;
  int failed;
};
static_assert(sizeof(RouterSmem) + 1024 <= 227 * 1024, "router shared memory (plus alignment) fits one CTA");
static_assert(sizeof(float) * RT_BM * RT_YSTR <= sizeof(((RouterSmem*)0)->b) + sizeof(((RouterSmem*)0)->a),
              "output staging fits in the operand rings");

__device__ __forceinline__ void mma_bf16_ss(uint32_t d_tmem, uint64_t da, uint64_t db, uint32_t accumulate) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }"
      ::"r"(d_tmem), "l"(da), "l"(db), "r"(IDESC_BF16), "r"(accumulate)
      : "memory");
}

// Byte offset of 16-byte unit j (0..7) of row r in a 128-byte-swizzled tile.
__device__ __forceinline__ int sw128(int r, int j) { return r * 128 + ((j ^ (r & 7)) << 4); }

// (element 0 = low half, element 1 = high half) of a bf16 pair, as floats
__device__ __forceinline__ float2 unpack_bf16x2(uint32_t w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
}
// round-to-nearest-even bf16 pair: v.x -> low half, v.y -> high half
__device__ __forceinline__ uint32_t pack_bf16x2_rn(float2 v) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(v.y), "f"(v.x));
  return r;
}
__device__ __forceinline__ float2 sub2(float2 a, float2 b) {
  float2 c;
  asm("sub.rn.f32x2 %0, %1, %2;"
      : "=l"(reinterpret_cast<uint64_t&>(c))
      : "l"(reinterpret_cast<const uint64_t&>(a)), "l"(reinterpret_cast<const uint64_t&>(b)));
  return c;
}

// One CTA: 128 tokens x all 128 experts x K chunks [blockIdx.y*CPS, +CPS).
// Per chunk c: the router chunk arrives by cp.async two chunks ahead (6-stage
// ring), the thread's x units RT_XLA chunks ahead in registers; x*s is split
// into its hi / lo bf16 parts in A stage c%4 (after the MMAs of chunk c-4,
// which read that stage, complete), and thread 0 issues the chunk's 8 MMAs,
// which then run while the threads prepare the next chunks.
template <int CPS>
__global__ void __launch_bounds__(RT_THREADS, 1)
router_tc_kernel(const uint16_t* __restrict__ x, const uint16_t* __restrict__ wr,
                 const uint16_t* __restrict__ rscale, int T, float* __restrict__ logits,
                 int* __restrict__ err, int wait_first) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  RouterSmem& s =
      *reinterpret_cast<RouterSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5;
  const int t0 = blockIdx.x * RT_BM, kb = blockIdx.y * CPS * RT_BK;
  // this thread's 16-byte unit column j of token rows (tid >> 3) + 32q, and of
  // expert rows (tid >> 3) + 32q in the router chunks
  const int j = tid & 7, r0 = tid >> 3;

  auto issue_b = [&](int c) {  // router chunk c -> ring stage c % RT_BST, one commit group
    if (c < CPS) {
      uint8_t* dst = s.b[c % RT_BST];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int e = r0 + 32 * q;
        cp_async16(dst + sw128(e, j), wr + (size_t)e * H + kb + c * RT_BK + j * 8);
      }
    }
    cp_async_commit();
  };
  auto load_x = [&](int c, uint4 (&v)[4], uint4& rs) {
    const int k0 = kb + c * RT_BK + j * 8;
    rs = *reinterpret_cast<const uint4*>(rscale + k0);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int t = t0 + r0 + 32 * q;
      v[q] = t < T ? __ldg(reinterpret_cast<const uint4*>(x + (size_t)t * H + k0)) : make_uint4(0, 0, 0, 0);
    }
  };

  issue_b(0);
  issue_b(1);
  if (tid == 0) {
    for (int i = 0; i < RT_AST; ++i) mbar_init(&s.done[i], 1);
    s.failed = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&s.tmem_base)),
                 "r"(128u));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
  }
  // no wait before reading x when a norm kernel that waited is the
  // predecessor (see the file comment); as the forward's first kernel
  // (wait_first) x may still be being written by the previous one
  if (wait_first) pdl_wait();
  pdl_trigger();
  uint4 xv[RT_XLA + 1][4], rs[RT_XLA + 1];
#pragma unroll
  for (int c = 0; c < RT_XLA && c < CPS; ++c) load_x(c, xv[c], rs[c]);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;

#pragma unroll
  for (int c = 0; c < CPS; ++c) {
    const int st = c % RT_AST;
    if (c + RT_XLA < CPS) load_x(c + RT_XLA, xv[(c + RT_XLA) % (RT_XLA + 1)], rs[(c + RT_XLA) % (RT_XLA + 1)]);
    // stage st and router stage (c+2) % RT_BST were read by the MMAs of chunk
    // c - RT_AST (both rings are fresh before that)
    if (c >= RT_AST) {
      const int cw = c - RT_AST;
      mbar_wait(&s.done[cw % RT_AST], (uint32_t)((cw / RT_AST) & 1), &s.failed);
    }
    issue_b(c + 2);
    const uint4 rc = rs[c % (RT_XLA + 1)];
    const uint32_t rsw[4] = {rc.x, rc.y, rc.z, rc.w};
    float2 ss[4];  // this thread's 8 router scales of the chunk, as pairs
#pragma unroll
    for (int p = 0; p < 4; ++p) ss[p] = unpack_bf16x2(rsw[p]);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint4 v = xv[c % (RT_XLA + 1)][q];
      const uint32_t xw[4] = {v.x, v.y, v.z, v.w};
      uint32_t hi[4], lo[4];
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        const float2 sv = mul2(unpack_bf16x2(xw[p]), ss[p]);  // x*s, exact
        hi[p] = pack_bf16x2_rn(sv);
        lo[p] = pack_bf16x2_rn(sub2(sv, unpack_bf16x2(hi[p])));  // exact residual (<= 8 bits)
      }
      const int off = sw128(r0 + 32 * q, j);
      *reinterpret_cast<uint4*>(s.a[st][0] + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
      *reinterpret_cast<uint4*>(s.a[st][1] + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    }
    cp_async_wait_group<2>();  // router chunk c (two later groups may still fly)
    // generic-proxy shared-memory writes -> visible to the tensor core (async proxy)
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    if (tid == 0 && !*(volatile int*)&s.failed) {
      tc_fence_after();
#pragma unroll
      for (int k = 0; k < RT_BK / 16; ++k) {
        const uint64_t db = kmajor_sw128_desc(smem_u32(s.b[c % RT_BST]) + k * 32);
#pragma unroll
        for (int p = 0; p < 2; ++p)
          mma_bf16_ss(tmem, kmajor_sw128_desc(smem_u32(s.a[st][p]) + k * 32), db, (c | k | p) != 0);
      }
      mma_commit(&s.done[st]);
    }
  }
  // every chunk's MMAs complete (in order: the last commit covers them all)
  mbar_wait(&s.done[(CPS - 1) % RT_AST], (uint32_t)(((CPS - 1) / RT_AST) & 1), &s.failed);
  tc_fence_after();

  // epilogue: warp w reads TMEM lanes 32*(w&3).. and columns 64*(w>>2)..,
  // stages the f32 tile in shared memory (reusing the operand rings), then
  // whole 512-byte rows are stored
  float* ystage = reinterpret_cast<float*>(&s.b[0][0]);
  cp_async_wait_all();
  __syncthreads();  // every thread is past its last read of the rings
  {
    const int q = warp & 3, half = warp >> 2, row = q * 32 + (tid & 31);
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
  const int lane = tid & 31;
  for (int r = warp; r < RT_BM; r += RT_THREADS / 32) {
    const int t = t0 + r;
    if (t >= T) break;
    *reinterpret_cast<float4*>(out + (size_t)t * E + lane * 4) =
        *reinterpret_cast<const float4*>(ystage + r * RT_YSTR + lane * 4);
  }
  if (tid == 0 && *(volatile int*)&s.failed) atomicExch(err, 1);
  // this grid completes only after its predecessor (the norm kernel) has
  // completed (with wait_first the wait came before the x loads)
  if (!wait_first) pdl_wait();
}

}  // namespace tc

cudaError_t launch_router_logits_tc(const uint16_t* x, const uint16_t* wr, const uint16_t* rscale, int T,
                                    float* logits, int* err, cudaStream_t s, bool wait_first) {
  const size_t smem = sizeof(tc::RouterSmem) + 1024;
  // router_ksplit(T) K slices: 11 chunks each for wide batches (about one CTA
  // per SM at 4096 tokens), 4 chunks each below (more CTAs for fewer tokens)
  const int ns = router_ksplit(T);
  if (ns != ROUTER_WIDE_SLICES && ns != ROUTER_SLICES) return cudaErrorInvalidValue;
  auto k = ns == ROUTER_WIDE_SLICES ? tc::router_tc_kernel<tc::RT_CHUNKS / ROUTER_WIDE_SLICES>
                                    : tc::router_tc_kernel<tc::RT_CHUNKS / ROUTER_SLICES>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  return launch_k(k, dim3((T + tc::RT_BM - 1) / tc::RT_BM, ns), dim3(tc::RT_THREADS), smem, s, x, wr, rscale, T,
                  logits, err, wait_first ? 1 : 0);
}

}  // namespace gm
