// gemm_tc_bf16.cu -- prefill expert products of bf16 layers on the tcgen05
// tensor cores (kind::f16 with bf16 operands, f32 accumulators in TMEM).
//
// Same mathematics as the bf16 decode kernels of experts_bf16.cu
// (kernels/moe_experts.mojo:16-162 phase 1, :201-319 phase 2), organised as a
// grouped GEMM over the schedule's contiguous per-expert route segments:
//
//  * phase 1: A = the routed normalised activation rows in schedule order
//    ([R][2816] bf16, gathered once per call), B = 64 gate rows + the matching
//    64 up rows of the expert (the registered row-major [epr][1408][2816]
//    layout is already K-major), D = 128 routes x 128 f32 columns.  Epilogue:
//    bucket[route][j] = bf16(gelu_tanh(g_j) * u_j).
//  * phase 2: A = the bucket rows ([R][704] bf16), B = 128 rows of the
//    expert's [2816][704] down matrix, D = 128 routes x 128 hidden columns.
//    Epilogue: y[route][n] = D * w_route (f32), staged per row and written as
//    whole 512-byte rows; the combine kernel sums a token's routes in expert
//    order as for every other path.
//
// Persistent CTAs (one per SM), warp-specialised like gemm_tc.cu: warp 0
// issues TMA loads into a shared-memory ring, warp 1 allocates TMEM and issues
// the MMAs from one thread (K = 16 per instruction, 4 per 64-element stage)
// into two accumulators so that the epilogue of one tile overlaps the MMAs of
// the next, warps 2..17 are the epilogue (4 per TMEM lane quarter, one route
// row per thread).  Every mbarrier wait is bounded; on expiry the kernel
// writes 1 into *err, stops issuing work and still frees its TMEM.
#include <cuda.h>

#include "gm_kernels.h"
#include "tc_prims.cuh"

namespace gm {

namespace tcb {

using namespace tc;

constexpr int BN = 128;                  // accumulator columns
constexpr int BKE = 64;                  // bf16 elements per 128-byte stage row
constexpr int A_BYTES = TILE_M * 128;    // 16 KB
constexpr int B_BYTES = BN * 128;        // 16 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int STAGES1 = 6;
constexpr int STAGES2 = 4;
constexpr int KS1 = H / BKE;             // 44 K stages (gate/up)
constexpr int KS2 = I / BKE;             // 11 K stages (down)
constexpr int NJ1 = I / 64;              // 11 column tiles of 64 intermediate outputs
constexpr int NT2 = H / BN;              // 22 hidden tiles
constexpr int EPI_WARPS = 16;
constexpr int THREADS = 64 + 32 * EPI_WARPS;
constexpr uint32_t TMEM_COLS = 2 * BN;   // two accumulators
constexpr int YSTR = BN + 4;
constexpr int ERR_TIMEOUT = 1;

// kind::f16: D = f32, A = B = bf16, both K-major, N = 128, M = 128.
constexpr uint32_t IDESC = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                           ((uint32_t)(TILE_M >> 4) << 24);

struct Smem1 {
  uint8_t stage[STAGES1][STAGE_BYTES];  // first member: 1024-byte aligned
  uint64_t full[STAGES1];
  uint64_t empty[STAGES1];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint32_t tmem_base;
  int failed;
  TileTable tt;
};

struct Smem2 {
  uint8_t stage[STAGES2][STAGE_BYTES];
  float ystage[TILE_M][YSTR];
  uint64_t full[STAGES2];
  uint64_t empty[STAGES2];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint32_t tmem_base;
  int failed;
  TileTable tt;
};

__device__ __forceinline__ void mma_bf16(uint32_t d, uint64_t da, uint64_t db, uint32_t accumulate) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }"
      ::"r"(d), "l"(da), "l"(db), "r"(IDESC), "r"(accumulate)
      : "memory");
}

template <typename S>
__device__ __forceinline__ void setup(S& s, const int32_t* expert_offset, int epr, int warp, int lane) {
  if (threadIdx.x == 0) {
    constexpr int NS = sizeof(s.full) / sizeof(s.full[0]);
    for (int i = 0; i < NS; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.acc_full[i], 1);
      mbar_init(&s.acc_empty[i], EPI_WARPS);  // one arrival per epilogue warp
    }
    s.failed = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 2) build_tile_table(s.tt, expert_offset, epr, lane);
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&s.tmem_base)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
}

template <typename S>
__device__ __forceinline__ void teardown(S& s, uint32_t tmem, int warp, int* err) {
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
  }
  if (threadIdx.x == 0 && s.failed) atomicExch(err, ERR_TIMEOUT);
}

// MMA issuer shared by both phases: KS stages of 4 K=16 instructions per tile,
// accumulator t&1 of this CTA's tile sequence.
template <int KS, int NS, typename S>
__device__ __forceinline__ void mma_loop(S& s, uint32_t tmem, int total) {
  int stage = 0, acc = 0;
  uint32_t phase = 0, aphase = 0;
  for (int t = blockIdx.x; t < total; t += gridDim.x) {
    if (!mbar_wait(&s.acc_empty[acc], aphase ^ 1, &s.failed)) return;
    tc_fence_after();
    const uint32_t d = tmem + (uint32_t)(acc * BN);
    for (int k = 0; k < KS; ++k) {
      if (!mbar_wait(&s.full[stage], phase, &s.failed)) return;
      tc_fence_after();
      const uint32_t a0 = smem_u32(s.stage[stage]);
      const uint32_t b0 = a0 + A_BYTES;
#pragma unroll
      for (int kk = 0; kk < BKE / 16; ++kk)
        mma_bf16(d, kmajor_sw128_desc(a0 + kk * 32), kmajor_sw128_desc(b0 + kk * 32), (k | kk) != 0);
      mma_commit(&s.empty[stage]);
      if (++stage == NS) { stage = 0; phase ^= 1; }
    }
    mma_commit(&s.acc_full[acc]);
    if (++acc == 2) { acc = 0; aphase ^= 1; }
  }
}

__global__ void __launch_bounds__(THREADS, 1)
tcb_phase1_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                  const int32_t* __restrict__ expert_offset, int epr, uint16_t* __restrict__ bucket,
                  int* __restrict__ err, int max_rows, int max_tiles) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  Smem1& s = *reinterpret_cast<Smem1*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  pdl_wait();
  pdl_trigger();
  setup(s, expert_offset, epr, warp, lane);
  const uint32_t tmem = s.tmem_base;
  int total = s.tt.moff[epr] * NJ1;
  if (total < 0 || total > max_tiles || s.tt.eoff[epr] > max_rows) {
    if (tid == 0) atomicExch(err, 2);
    total = 0;
  }
  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int t = blockIdx.x; t < total; t += gridDim.x) {
        const TileInfo ti = tile_info(s.tt, epr, NJ1, t);
        const int gate_row = ti.e * GU + ti.col * 64;
        for (int k = 0; k < KS1; ++k) {
          if (!mbar_wait(&s.empty[stage], phase ^ 1, &s.failed)) goto done;
          uint8_t* st = s.stage[stage];
          mbar_expect_tx(&s.full[stage], STAGE_BYTES);
          tma_load_2d(st, &map_a, k * BKE, ti.row0, &s.full[stage]);
          tma_load_2d(st + A_BYTES, &map_b, k * BKE, gate_row, &s.full[stage]);
          tma_load_2d(st + A_BYTES + B_BYTES / 2, &map_b, k * BKE, gate_row + I, &s.full[stage]);
          if (++stage == STAGES1) { stage = 0; phase ^= 1; }
        }
      }
    done:;
    }
  } else if (warp == 1) {
    if (lane == 0) mma_loop<KS1, STAGES1>(s, tmem, total);
  } else {
    // epilogue warp (q, cb): lanes 32q.., gate columns 16cb..16cb+15 and the
    // matching up columns 64+16cb..
    const int q = warp & 3, cb = (warp - 2) >> 2, r = q * 32 + lane;
    int acc = 0;
    uint32_t aphase = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x) {
      const TileInfo ti = tile_info(s.tt, epr, NJ1, t);
      (void)__all_sync(0xffffffffu, mbar_wait(&s.acc_full[acc], aphase, &s.failed));
      tc_fence_after();
      int g[16], u[16];
      const uint32_t base = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN);
      tmem_ld16(base + 16 * cb, g);
      tmem_ld16(base + 64 + 16 * cb, u);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.acc_empty[acc]);
      if (++acc == 2) { acc = 0; aphase ^= 1; }
      if (r < ti.nvalid) {
        uint32_t o[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float v0 = __fmul_rn(gelu_tanh_f32(__int_as_float(g[2 * i])), __int_as_float(u[2 * i]));
          const float v1 =
              __fmul_rn(gelu_tanh_f32(__int_as_float(g[2 * i + 1])), __int_as_float(u[2 * i + 1]));
          o[i] = (uint32_t)f2bf(v0) | ((uint32_t)f2bf(v1) << 16);
        }
        uint4* dst = reinterpret_cast<uint4*>(bucket + (size_t)(ti.row0 + r) * I + ti.col * 64 + 16 * cb);
        dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
        dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
      }
    }
  }
  teardown(s, tmem, warp, err);
}

__global__ void __launch_bounds__(THREADS, 1)
tcb_phase2_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                  const int32_t* __restrict__ expert_offset, int epr,
                  const SparseRoute* __restrict__ routes, float* __restrict__ ybuf,
                  int* __restrict__ err, int max_rows, int max_tiles) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  Smem2& s = *reinterpret_cast<Smem2*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  pdl_wait();
  pdl_trigger();
  setup(s, expert_offset, epr, warp, lane);
  const uint32_t tmem = s.tmem_base;
  int total = s.tt.moff[epr] * NT2;
  if (total < 0 || total > max_tiles || s.tt.eoff[epr] > max_rows) {
    if (tid == 0) atomicExch(err, 2);
    total = 0;
  }
  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int t = blockIdx.x; t < total; t += gridDim.x) {
        const TileInfo ti = tile_info(s.tt, epr, NT2, t);
        for (int k = 0; k < KS2; ++k) {
          if (!mbar_wait(&s.empty[stage], phase ^ 1, &s.failed)) goto done;
          uint8_t* st = s.stage[stage];
          mbar_expect_tx(&s.full[stage], STAGE_BYTES);
          tma_load_2d(st, &map_a, k * BKE, ti.row0, &s.full[stage]);
          tma_load_2d(st + A_BYTES, &map_b, k * BKE, ti.e * H + ti.col * BN, &s.full[stage]);
          if (++stage == STAGES2) { stage = 0; phase ^= 1; }
        }
      }
    done:;
    }
  } else if (warp == 1) {
    if (lane == 0) mma_loop<KS2, STAGES2>(s, tmem, total);
  } else {
    // epilogue warp (q, cb): lanes 32q.., hidden columns 32cb..32cb+31
    const int q = warp & 3, cb = (warp - 2) >> 2, r = q * 32 + lane;
    int acc = 0;
    uint32_t aphase = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x) {
      const TileInfo ti = tile_info(s.tt, epr, NT2, t);
      const float wr = r < ti.nvalid ? routes[ti.row0 + r].weight : 0.0f;
      (void)__all_sync(0xffffffffu, mbar_wait(&s.acc_full[acc], aphase, &s.failed));
      tc_fence_after();
      int d[32];
      tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN + 32 * cb), d);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.acc_empty[acc]);
      if (++acc == 2) { acc = 0; aphase ^= 1; }
      float4* ys = reinterpret_cast<float4*>(&s.ystage[r][32 * cb]);
#pragma unroll
      for (int v = 0; v < 8; ++v)
        ys[v] = make_float4(__fmul_rn(__int_as_float(d[4 * v]), wr), __fmul_rn(__int_as_float(d[4 * v + 1]), wr),
                            __fmul_rn(__int_as_float(d[4 * v + 2]), wr), __fmul_rn(__int_as_float(d[4 * v + 3]), wr));
      quarter_sync(q);
      // the 4 warps of quarter q write its 32 rows: 8 rows each, one 512-byte row per warp store
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int rr = q * 32 + cb * 8 + j;
        if (rr < ti.nvalid) {
          const float4 v = reinterpret_cast<const float4*>(&s.ystage[rr][0])[lane];
          reinterpret_cast<float4*>(ybuf + (size_t)(ti.row0 + rr) * H + ti.col * BN)[lane] = v;
        }
      }
      quarter_sync(q);  // staging rows read before the next tile overwrites them
    }
  }
  teardown(s, tmem, warp, err);
}

}  // namespace tcb

namespace {
int sm_count_b() {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}
}  // namespace

cudaError_t launch_tcb_phase1(const void* map_a, const void* map_b, const int32_t* expert_offset,
                              int epr, int T, uint16_t* bucket, int* err, cudaStream_t s) {
  const int max_rows = T * TOPK;
  const int max_tiles = (max_rows / tc::TILE_M + epr) * tcb::NJ1;
  const size_t smem = sizeof(tcb::Smem1) + 1024;
  cudaError_t e = cudaFuncSetAttribute(tcb::tcb_phase1_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e != cudaSuccess) return e;
  return launch_k(tcb::tcb_phase1_kernel, dim3(sm_count_b()), dim3(tcb::THREADS), smem, s,
                  *reinterpret_cast<const CUtensorMap*>(map_a),
                  *reinterpret_cast<const CUtensorMap*>(map_b), expert_offset, epr, bucket, err,
                  max_rows, max_tiles);
}

cudaError_t launch_tcb_phase2(const void* map_a, const void* map_b, const int32_t* expert_offset,
                              int epr, int T, const SparseRoute* routes, float* ybuf, int* err,
                              cudaStream_t s) {
  const int max_rows = T * TOPK;
  const int max_tiles = (max_rows / tc::TILE_M + epr) * tcb::NT2;
  const size_t smem = sizeof(tcb::Smem2) + 1024;
  cudaError_t e = cudaFuncSetAttribute(tcb::tcb_phase2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e != cudaSuccess) return e;
  return launch_k(tcb::tcb_phase2_kernel, dim3(sm_count_b()), dim3(tcb::THREADS), smem, s,
                  *reinterpret_cast<const CUtensorMap*>(map_a),
                  *reinterpret_cast<const CUtensorMap*>(map_b), expert_offset, epr, routes, ybuf, err,
                  max_rows, max_tiles);
}

}  // namespace gm
