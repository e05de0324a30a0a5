// tc_prims.cuh -- sm_100a primitives shared by the tcgen05 kernels: shared
// memory mbarriers with bounded waits, 2-D TMA loads, the K-major 128-byte
// swizzle shared-memory descriptor, tcgen05 commit / fences / TMEM loads, and
// packed f32x2 arithmetic.
#pragma once
#include <cuda.h>

#include "gm_common.cuh"

namespace gm {
namespace tc {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait for the phase with parity `parity` to complete.  Returns false
// (and flags the CTA) after ~1 s.  With SUSPEND each try_wait may suspend the
// thread in hardware for up to 20 us (it resumes when the phase completes),
// so waiting warps leave the issue slots to the working warps; without it the
// thread polls, which reacts faster in a tight producer/consumer ping-pong.
template <bool SUSPEND = true>
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity, int* failed) {
  const uint32_t a = smem_u32(b);
  uint64_t t0 = 0;
  for (uint32_t it = 0;; ++it) {
    uint32_t ok;
    if (SUSPEND)
      asm volatile(
          "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3; selp.u32 %0, 1, 0, p; }"
          : "=r"(ok)
          : "r"(a), "r"(parity), "r"(20000u)
          : "memory");
    else
      asm volatile(
          "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
          : "=r"(ok)
          : "r"(a), "r"(parity)
          : "memory");
    if (ok) return true;
    if (*(volatile int*)failed) return false;
    if ((it & (SUSPEND ? 3 : 63)) == 0) {
      const uint64_t t = global_ns();
      if (t0 == 0) t0 = t;
      else if (t - t0 > 1000000000ull) {
        atomicExch(failed, 1);
        return false;
      }
    }
  }
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
      ::"r"(smem_u32(dst)), "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// L2 prefetch of one 2-D TMA box (no shared-memory destination, no barrier).
__device__ __forceinline__ void tma_prefetch_2d(const CUtensorMap* map, int x, int y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(map), "r"(x), "r"(y)
               : "memory");
}

// K-major operand, 128-byte swizzle: rows of 128 bytes, 8-row atoms 1024 bytes
// apart (SBO), version 1 (sm100), layout type 2 (SWIZZLE_128B).
__device__ __forceinline__ uint64_t kmajor_sw128_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, int (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, int (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]),
        "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]),
        "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
      ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Packed two-lane f32 arithmetic of sm_100 (one instruction, two IEEE
// round-to-nearest results; identical to the scalar operations).
__device__ __forceinline__ float2 add2(float2 a, float2 b) {
  float2 c;
  asm("add.rn.f32x2 %0, %1, %2;"
      : "=l"(reinterpret_cast<uint64_t&>(c))
      : "l"(reinterpret_cast<const uint64_t&>(a)), "l"(reinterpret_cast<const uint64_t&>(b)));
  return c;
}
__device__ __forceinline__ float2 mul2(float2 a, float2 b) {
  float2 c;
  asm("mul.rn.f32x2 %0, %1, %2;"
      : "=l"(reinterpret_cast<uint64_t&>(c))
      : "l"(reinterpret_cast<const uint64_t&>(a)), "l"(reinterpret_cast<const uint64_t&>(b)));
  return c;
}
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;"
      : "=l"(reinterpret_cast<uint64_t&>(d))
      : "l"(reinterpret_cast<const uint64_t&>(a)), "l"(reinterpret_cast<const uint64_t&>(b)),
        "l"(reinterpret_cast<const uint64_t&>(c)));
  return d;
}

// Exact int32 -> f32 for |d| < 2^22 (the 64-wide down-block dots are < 2^21):
// 1.5*2^23 + d is representable, so its bits are those of 0x4B400000 + d, and
// subtracting 1.5*2^23 is exact.  Two lanes at a time.
__device__ __forceinline__ float2 small_ints_to_float2(int d0, int d1) {
  const float2 biased = make_float2(__int_as_float(0x4B400000 + d0), __int_as_float(0x4B400000 + d1));
  return add2(biased, make_float2(-12582912.0f, -12582912.0f));
}

// ------------------------------------------------ grouped-GEMM tile tables
// Routes of one expert are contiguous (schedule order); an expert with n
// routes spans ceil(n / TILE_M) m-tiles of TILE_M routes.
constexpr int TILE_M = 128;

struct TileTable {
  int eoff[E + 1];   // expert_offset of this rank
  int moff[E + 1];   // prefix of ceil(n_e / TILE_M): m-tiles before expert e
};

// Named barrier for the 4 epilogue warps of one TMEM lane quarter.
__device__ __forceinline__ void quarter_sync(int q) {
  asm volatile("bar.sync %0, 128;" ::"r"(1 + q) : "memory");
}

struct TileInfo {
  int e, row0, nvalid, col;
};

// Tile t = (m-tile of an expert, column tile); m-tiles enumerated expert by
// expert so that consecutive tiles reuse the same weights (L2-resident).
__device__ __forceinline__ TileInfo tile_info(const TileTable& tt, int epr, int ncol, int t) {
  const int mg = t / ncol;
  TileInfo ti;
  ti.col = t % ncol;
  int lo = 0, hi = epr;  // tt.moff[lo] <= mg < tt.moff[hi]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (tt.moff[mid] <= mg) lo = mid; else hi = mid;
  }
  ti.e = lo;
  ti.row0 = tt.eoff[lo] + (mg - tt.moff[lo]) * TILE_M;
  ti.nvalid = min(TILE_M, tt.eoff[lo + 1] - ti.row0);
  return ti;
}

// m-tile prefix over this rank's experts (one warp, 4 experts per lane).
__device__ __forceinline__ void build_tile_table(TileTable& tt, const int32_t* expert_offset, int epr,
                                                 int lane) {
  int c[4], sum = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int e = lane * 4 + j;
    const int n = e < epr ? expert_offset[e + 1] - expert_offset[e] : 0;
    c[j] = (n + TILE_M - 1) / TILE_M;
    sum += c[j];
  }
  int inc = sum;
#pragma unroll
  for (int m = 1; m < 32; m <<= 1) {
    const int o = __shfl_up_sync(0xffffffffu, inc, m);
    if (lane >= m) inc += o;
  }
  int run = inc - sum;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int e = lane * 4 + j;
    if (e < epr) {
      tt.moff[e] = run;
      tt.eoff[e] = expert_offset[e];
    }
    run += c[j];
  }
  if (lane == 31) {  // end entries (e = epr, up to 128)
    tt.moff[epr] = run;
    tt.eoff[epr] = expert_offset[epr];
  }
}

}  // namespace tc
}  // namespace gm
