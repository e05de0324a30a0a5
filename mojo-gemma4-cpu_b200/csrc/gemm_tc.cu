// gemm_tc.cu -- prefill expert products on the 5th-generation tensor cores
// (tcgen05 + TMEM + TMA), sm_100a.
//
// Same mathematics as the decode kernels of experts_bq.cu, organised for many
// routes per expert:
//
//  * phase 1 (butterquant_kernels/moe.mojo:26-129, then the bucket FWHT-64
//    quantisation of linear.mojo:182-205): A = the routed activation rows of
//    one expert in schedule order (gathered once per call into a contiguous
//    [R][2816] int8 buffer so that a 2-D TMA box covers 128 routes), B = 64 gate
//    rows + the matching 64 up rows from a row-major (K-contiguous) int8 copy of
//    the packed weights (gm_vnni_unpack: the VNNI tile order is a permutation),
//    D = 128 routes x 128 int32 columns in TMEM, exact signed dots
//    (tcgen05.mma kind::i8, K = 32 per instruction, 22 stages of 128 K bytes).
//  * phase 2 (butterquant_kernels/moe.mojo:168-225): the down product with the
//    reference's per-64-K-block dequantisation; each K block's exact int32 dot
//    goes to one of 4 TMEM regions (128 columns), the epilogue folds it into
//    facc = fma(f32(dot_b), sa[b]/127, facc) in block order and frees the
//    region, so the MMA warp runs up to 4 blocks ahead.  y = facc*sw*w_route.
//
// Persistent CTAs (one per SM), warp-specialised: warp 0 issues TMA loads into
// a shared-memory ring, warp 1 allocates TMEM and issues the MMAs from one
// thread, warps 2..17 are the epilogue: 4 warps per TMEM lane quarter (one
// route row per thread), each owning a quarter of the tile's columns.  In
// phase 1 the FWHT-64 stages of stride 16 and 32 and the row absmax cross
// those column blocks through shared memory (named barrier per quarter); in
// phase 2 the f32 output rows are staged in shared memory and written with
// whole-row coalesced stores.
//
// Every mbarrier wait is bounded (1 s of globaltimer); on expiry the kernel
// records GM_ERR_TIMEOUT in *err, stops issuing work, still meets the final
// barrier and frees its TMEM.
#include <cuda.h>

#include "gm_kernels.h"
#include "tc_prims.cuh"

namespace gm {

namespace tc {

constexpr int BM = 128;            // routes per tile (TMEM lanes)
constexpr int BN = 128;            // phase 1: 64 gate + 64 up rows; phase 2: 128 hidden rows
constexpr int BK = 128;            // K bytes per stage (one 128-byte swizzle row)
constexpr int KB1 = H / BK;        // 22 K stages for gate/up
constexpr int NJ1 = I / 64;        // 11 column tiles of 64 intermediate outputs
constexpr int NT2 = H / BN;        // 22 hidden tiles
constexpr int KC2 = (I + BK - 1) / BK;  // 6 K stages of 128 bytes (last half zero-filled)
constexpr int A_BYTES = BM * BK;   // 16 KB
constexpr int B_BYTES = BN * BK;   // 16 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int STAGES1 = 6;          // the FWHT exchange lives in TMEM, so a 6th stage fits
constexpr int STAGES2 = 4;
constexpr int RING = 4;            // phase-2 TMEM regions
constexpr int EPI_WARPS = 16;
constexpr int THREADS = 64 + 32 * EPI_WARPS;  // 576
constexpr uint32_t TMEM_COLS1 = 512;         // two 128-column accumulators + the FWHT exchange
constexpr uint32_t XCOL1 = 2 * BN;           // phase-1 exchange columns [XCOL1, XCOL1 + 64)
constexpr uint32_t TMEM_COLS2 = RING * BN;   // 512
constexpr int YSTR = BN + 4;       // phase-2 output staging row stride (floats)
constexpr int ERR_TIMEOUT = 1;

struct Smem1 {
  uint8_t stage[STAGES1][STAGE_BYTES];  // first member: 1024-byte aligned
  float amax[BM][4];
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
  // dense: the bf16 output rows staged as float [BM][YSTR]; MoE: 16 boxes of
  // 32 x 32 f32 (one per epilogue warp, 128-byte swizzled) for TMA stores
  union {
    float ystage[BM][YSTR];
    uint8_t ybox[EPI_WARPS][32 * 128];
  };
  uint64_t full[STAGES2];
  uint64_t empty[STAGES2];
  uint64_t reg_full[RING];
  uint64_t reg_empty[RING];
  uint32_t tmem_base;
  int failed;
  TileTable tt;
};

// kind::i8, D = s32, A = B = signed int8, both K-major, N = 128, M = 128.
constexpr uint32_t IDESC_I8 = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                              ((uint32_t)(BM >> 4) << 24);

__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t da, uint64_t db, uint32_t accumulate) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %5, %5, %5}, p; }"
      ::"r"(d_tmem), "l"(da), "l"(db), "r"(IDESC_I8), "r"(accumulate), "r"(0u)
      : "memory");
}

// DENSE: the dense MLP's gate/up product (dense_bq.cu's mathematics, gate and
// up rounded to bf16 before GeGLU) over dense_rows token rows in order, as one
// "expert" with 2112 intermediate columns: B rows [0, 2112) gate, [2112, 4224) up.
template <bool DENSE>
__global__ void __launch_bounds__(THREADS, 1)
tc_phase1_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                 const int32_t* __restrict__ expert_offset, int epr, int dense_rows,
                 const float* __restrict__ xg_sa, const float* __restrict__ gu_scale,
                 int8_t* __restrict__ bucket_i8, float* __restrict__ bucket_sa,
                 uint16_t* __restrict__ bucket_bf16, int* __restrict__ err, int max_rows,
                 int max_tiles) {
  constexpr int IW = DENSE ? DENSE_I : I;  // intermediate columns per expert
  constexpr int GUW = 2 * IW;               // gate + up rows per expert
  constexpr int NJ = IW / 64;               // column tiles
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  Smem1& s = *reinterpret_cast<Smem1*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  pdl_wait();
  pdl_trigger();
  if (tid == 0) {
    for (int i = 0; i < STAGES1; ++i) {
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
  if (warp == 2) {
    if constexpr (DENSE) {
      if (lane == 0) {
        s.tt.eoff[0] = 0;
        s.tt.eoff[1] = dense_rows;
        s.tt.moff[0] = 0;
        s.tt.moff[1] = (dense_rows + TILE_M - 1) / TILE_M;
      }
    } else {
      build_tile_table(s.tt, expert_offset, epr, lane);
    }
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&s.tmem_base)),
                 "r"(TMEM_COLS1));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  const uint32_t tmem = s.tmem_base;
  int total = s.tt.moff[epr] * NJ;
  // Defensive bound: never more tiles than the route buffers can hold.
  if (total < 0 || total > max_tiles || s.tt.eoff[epr] > max_rows) {
    if (tid == 0) atomicExch(err, 2);
    total = 0;
  }

  if (warp == 0) {
    // ---------------- TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int t = blockIdx.x; t < total; t += gridDim.x) {
        const TileInfo ti = tile_info(s.tt, epr, NJ, t);
        const int brow_g = ti.e * GUW + ti.col * 64;
        const int brow_u = ti.e * GUW + IW + ti.col * 64;
        for (int kb = 0; kb < KB1; ++kb) {
          if (!mbar_wait(&s.empty[stage], phase ^ 1, &s.failed)) goto producer_done;
          uint8_t* st = s.stage[stage];
          mbar_expect_tx(&s.full[stage], STAGE_BYTES);
          tma_load_2d(st, &map_a, kb * BK, ti.row0, &s.full[stage]);
          tma_load_2d(st + A_BYTES, &map_b, kb * BK, brow_g, &s.full[stage]);
          tma_load_2d(st + A_BYTES + B_BYTES / 2, &map_b, kb * BK, brow_u, &s.full[stage]);
          if (++stage == STAGES1) { stage = 0; phase ^= 1; }
        }
      }
    producer_done:;
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int t = blockIdx.x; t < total; t += gridDim.x) {
        if (!mbar_wait(&s.acc_empty[acc], acc_phase ^ 1, &s.failed)) break;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(acc * BN);
        bool ok = true;
        for (int kb = 0; kb < KB1; ++kb) {
          if (!mbar_wait(&s.full[stage], phase, &s.failed)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a0 = smem_u32(s.stage[stage]);
          const uint32_t b0 = a0 + A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 32; ++kk)
            mma_i8(d, kmajor_sw128_desc(a0 + kk * 32), kmajor_sw128_desc(b0 + kk * 32),
                   (kb | kk) != 0);
          mma_commit(&s.empty[stage]);
          if (++stage == STAGES1) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        mma_commit(&s.acc_full[acc]);
        if (++acc == 2) { acc = 0; acc_phase ^= 1; }
      }
    }
  } else {
    // ---------------- epilogue: warp (q, cb) owns TMEM lanes 32q..32q+31 and
    // bucket columns 16cb..16cb+15 of the tile's 64
    const int q = warp & 3;
    const int cb = (warp - 2) >> 2;
    const int r = q * 32 + lane;
    const float inv127 = 1.0f / 127.0f;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x) {
      const TileInfo ti = tile_info(s.tt, epr, NJ, t);
      // per-tile operands are loaded before the accumulator wait
      const bool valid = r < ti.nvalid;
      const int row = ti.row0 + r;
      const float ad = valid ? __fmul_rn(xg_sa[row], inv127) : 0.0f;
      const float* wsg = gu_scale + (size_t)ti.e * GUW + ti.col * 64 + 16 * cb;
      float sg[16], su[16];
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        sg[c] = __ldg(wsg + c);
        su[c] = __ldg(wsg + IW + c);
      }
      // On a failed (timed-out) wait the epilogue keeps walking the tiles
      // without waiting (the CTA's failed flag makes every later wait return at
      // once) so that the named barriers below are always met; the results are
      // then discarded through *err.  The vote keeps the warp converged for the
      // .sync.aligned tcgen05.ld.
      (void)__all_sync(0xffffffffu, mbar_wait(&s.acc_full[acc], acc_phase, &s.failed));
      tc_fence_after();
      const uint32_t base = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN);
      int gd[16], ud[16];
      tmem_ld16(base + 16 * cb, gd);
      tmem_ld16(base + 64 + 16 * cb, ud);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.acc_empty[acc]);  // the warp's share drained: MMA may reuse it
      if (++acc == 2) { acc = 0; acc_phase ^= 1; }

      float hv[16];
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        float gv = __fmul_rn(__fmul_rn((float)gd[c], ad), sg[c]);
        float uv = __fmul_rn(__fmul_rn((float)ud[c], ad), su[c]);
        if constexpr (DENSE) {  // bq_linear stores gate and up as bf16 before GeGLU
          gv = bf2f(f2bf(gv));
          uv = bf2f(f2bf(uv));
        }
        hv[c] = bf2f(f2bf(__fmul_rn(gelu_tanh_f32(gv), uv)));
      }
      if (bucket_bf16 && valid) {
        uint4* dst = reinterpret_cast<uint4*>(bucket_bf16 + (size_t)row * IW + ti.col * 64 + 16 * cb);
#pragma unroll
        for (int v = 0; v < 2; ++v) {
          uint32_t w[4];
#pragma unroll
          for (int u = 0; u < 4; ++u)
            w[u] = (uint32_t)f2bf(hv[v * 8 + 2 * u]) | ((uint32_t)f2bf(hv[v * 8 + 2 * u + 1]) << 16);
          dst[v] = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
      // FWHT-64 stages of stride 1..8 stay inside this thread's 16 columns
#pragma unroll
      for (int st = 1; st < 16; st <<= 1)
#pragma unroll
        for (int i = 0; i < 16; ++i)
          if (!(i & st)) {
            const float a = hv[i], b = hv[i + st];
            hv[i] = __fadd_rn(a, b);
            hv[i + st] = __fsub_rn(a, b);
          }
      // strides 16 and 32 pair this block with block cb^1, then cb^2 (the lower
      // block keeps a+b, the upper a-b with a from the lower block)
      // (exchanged through TMEM columns [XCOL1, XCOL1 + 64) of the quarter's
      // lanes: each of its 4 warps writes its 16 columns, then reads its partner's)
      const uint32_t xq = tmem + ((uint32_t)(q * 32) << 16) + XCOL1;
#pragma unroll
      for (int sx = 1; sx <= 2; sx <<= 1) {
        uint32_t mine[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) mine[i] = __float_as_uint(hv[i]);
        tmem_st16(xq + 16 * cb, mine);
        tmem_st_wait();
        tc_fence_before();
        quarter_sync(q);
        tc_fence_after();
        int other[16];
        tmem_ld16(xq + 16 * (cb ^ sx), other);
        tmem_ld_wait();
        const bool upper = (cb & sx) != 0;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float pv = __int_as_float(other[i]);
          hv[i] = upper ? __fsub_rn(pv, hv[i]) : __fadd_rn(hv[i], pv);
        }
        tc_fence_before();
        quarter_sync(q);  // partners have read before the columns are rewritten
        tc_fence_after();
      }
      float amax = 0.0f;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        hv[i] = __fmul_rn(hv[i], fwht_scale_64());
        amax = fmaxf(amax, fabsf(hv[i]));
      }
      s.amax[r][cb] = amax;
      quarter_sync(q);
      amax = fmaxf(fmaxf(s.amax[r][0], s.amax[r][1]), fmaxf(s.amax[r][2], s.amax[r][3]));
      if (valid) {
        const float qinv = amax > 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
        uint32_t w[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          uint32_t p = 0;
#pragma unroll
          for (int b = 0; b < 4; ++b)
            p |= (uint32_t)(quantize_i8(hv[u * 4 + b], qinv) & 0xFF) << (8 * b);
          w[u] = p;
        }
        *reinterpret_cast<uint4*>(bucket_i8 + (size_t)row * IW + ti.col * 64 + 16 * cb) =
            make_uint4(w[0], w[1], w[2], w[3]);
        if (cb == 0) bucket_sa[(size_t)row * NJ + ti.col] = amax;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS1));
  }
  if (tid == 0 && s.failed) atomicExch(err, ERR_TIMEOUT);
}

// DENSE: the dense MLP's down product (K = 2112, 33 blocks) over dense_rows
// token rows in order, out = bf16(facc * sw) into a bf16 [rows][2816] `yout`.
template <bool DENSE>
__global__ void __launch_bounds__(THREADS, 1)
tc_phase2_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                 const __grid_constant__ CUtensorMap map_y,
                 const int32_t* __restrict__ expert_offset, int epr, int dense_rows,
                 const float* __restrict__ bsa, const SparseRoute* __restrict__ routes,
                 const float* __restrict__ dn_scale, void* __restrict__ yout,
                 int* __restrict__ err, int max_rows, int max_tiles) {
  constexpr int KW = DENSE ? DENSE_I : I;   // K bytes per row
  constexpr int NB = KW / 64;               // dequantisation blocks
  constexpr int KC = (KW + BK - 1) / BK;    // K stages (last half zero-filled)
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  Smem2& s = *reinterpret_cast<Smem2*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  pdl_wait();
  pdl_trigger();
  if (tid == 0) {
    for (int i = 0; i < STAGES2; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
    }
    for (int i = 0; i < RING; ++i) {
      mbar_init(&s.reg_full[i], 1);
      mbar_init(&s.reg_empty[i], EPI_WARPS);  // one arrival per epilogue warp
    }
    s.failed = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 2) {
    if constexpr (DENSE) {
      if (lane == 0) {
        s.tt.eoff[0] = 0;
        s.tt.eoff[1] = dense_rows;
        s.tt.moff[0] = 0;
        s.tt.moff[1] = (dense_rows + TILE_M - 1) / TILE_M;
      }
    } else {
      build_tile_table(s.tt, expert_offset, epr, lane);
    }
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&s.tmem_base)),
                 "r"(TMEM_COLS2));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

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
        for (int c = 0; c < KC; ++c) {
          if (!mbar_wait<false>(&s.empty[stage], phase ^ 1, &s.failed)) goto producer_done2;
          uint8_t* st = s.stage[stage];
          mbar_expect_tx(&s.full[stage], STAGE_BYTES);
          tma_load_2d(st, &map_a, c * BK, ti.row0, &s.full[stage]);
          tma_load_2d(st + A_BYTES, &map_b, c * BK, ti.e * H + ti.col * BN, &s.full[stage]);
          if (++stage == STAGES2) { stage = 0; phase ^= 1; }
        }
      }
    producer_done2:;
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int stage = 0, reg = 0;
      uint32_t phase = 0, rphase = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < total; t += gridDim.x) {
        for (int c = 0; ok && c < KC; ++c) {
          if (!mbar_wait<false>(&s.full[stage], phase, &s.failed)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a0 = smem_u32(s.stage[stage]);
          const uint32_t b0 = a0 + A_BYTES;
          for (int h = 0; h < 2; ++h) {
            if (2 * c + h >= NB) break;  // K bytes beyond KW are padding
            if (!mbar_wait<false>(&s.reg_empty[reg], rphase ^ 1, &s.failed)) { ok = false; break; }
            tc_fence_after();
            const uint32_t d = tmem + (uint32_t)(reg * BN);
#pragma unroll
            for (int kk = 0; kk < 2; ++kk) {
              const uint32_t off = (uint32_t)((2 * h + kk) * 32);
              mma_i8(d, kmajor_sw128_desc(a0 + off), kmajor_sw128_desc(b0 + off), kk);
            }
            mma_commit(&s.reg_full[reg]);
            if (++reg == RING) { reg = 0; rphase ^= 1; }
          }
          if (!ok) break;
          mma_commit(&s.empty[stage]);
          if (++stage == STAGES2) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else {
    // epilogue warp (q, cb): TMEM lanes 32q..32q+31, hidden columns 32cb..32cb+31
    const int q = warp & 3;
    const int cb = (warp - 2) >> 2;
    const int r = q * 32 + lane;
    const float inv127 = 1.0f / 127.0f;
    int reg = 0;
    uint32_t rphase = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x) {
      const TileInfo ti = tile_info(s.tt, epr, NT2, t);
      const bool valid = r < ti.nvalid;
      const bool quarter_live = q * 32 < ti.nvalid;  // warp-uniform
      const int row = ti.row0 + r;
      // per-tile operands are loaded before the first accumulator wait
      // the 11 expert block scales are held in registers; the dense MLP's 33
      // are read per block (issued before that block's accumulator wait)
      float adv[DENSE ? 1 : NB];
      if constexpr (!DENSE) {
#pragma unroll
        for (int b = 0; b < NB; ++b)
          adv[b] = valid ? __fmul_rn(bsa[(size_t)row * NB + b], inv127) : 0.0f;
      }
      const float wr = (!DENSE && valid) ? routes[row].weight : 0.0f;
      const float* wsc = dn_scale + (size_t)ti.e * H + ti.col * BN + 32 * cb;
      float2 facc[16];
#pragma unroll
      for (int n = 0; n < 16; ++n) facc[n] = make_float2(0.0f, 0.0f);
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        float adv_b;
        if constexpr (DENSE)
          adv_b = valid ? __fmul_rn(__ldg(bsa + (size_t)row * NB + b), inv127) : 0.0f;
        else
          adv_b = adv[b];
        // as in phase 1: after a failed wait keep going without waiting, so the
        // quarter's named barriers are always met
        (void)__all_sync(0xffffffffu, mbar_wait<false>(&s.reg_full[reg], rphase, &s.failed));
        tc_fence_after();
        int d[32];
        if (quarter_live)  // a quarter with no valid route rows only releases the region
          tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(reg * BN + 32 * cb), d);
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.reg_empty[reg]);  // the warp's columns read
        if (++reg == RING) { reg = 0; rphase ^= 1; }
        if (quarter_live) {
          const float2 a2 = make_float2(adv_b, adv_b);
#pragma unroll
          for (int i = 0; i < 16; ++i)
            facc[i] = fma2(small_ints_to_float2(d[2 * i], d[2 * i + 1]), a2, facc[i]);
        }
      }
      if constexpr (!DENSE) {
        // y = facc * sw * w_route for this warp's 32 rows x 32 columns: a fully
        // valid quarter goes out as one TMA store of the warp's swizzled box
        // (issued by lane 0, no barrier with the other warps); a partial one
        // is stored row by row from registers
        const float2 wr2 = make_float2(wr, wr);
        const bool full = q * 32 + 32 <= ti.nvalid;  // warp-uniform
        uint8_t* box = s.ybox[warp - 2];
        if (full) {
          if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");  // box free again
          __syncwarp();
        }
        float4* dst = reinterpret_cast<float4*>(static_cast<float*>(yout) + (size_t)row * H + ti.col * BN + 32 * cb);
#pragma unroll
        for (int v = 0; v < 8; ++v) {
          const float4 sw = __ldg(reinterpret_cast<const float4*>(wsc) + v);
          const float2 lo = mul2(mul2(facc[2 * v], make_float2(sw.x, sw.y)), wr2);
          const float2 hi = mul2(mul2(facc[2 * v + 1], make_float2(sw.z, sw.w)), wr2);
          const float4 yv = make_float4(lo.x, lo.y, hi.x, hi.y);
          if (full)
            *reinterpret_cast<float4*>(box + lane * 128 + ((v ^ (lane & 7)) << 4)) = yv;
          else if (valid)
            dst[v] = yv;
        }
        if (full) {
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          __syncwarp();
          if (lane == 0) {
            asm volatile(
                "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];"
                ::"l"(&map_y), "r"(ti.col * BN + 32 * cb), "r"(ti.row0 + q * 32), "r"(smem_u32(box))
                : "memory");
            asm volatile("cp.async.bulk.commit_group;" ::: "memory");
          }
        }
        continue;
      }
      // dense: y = facc * sw, staged per row then written as whole bf16 rows
      const float2 wr2 = make_float2(wr, wr);
      float4* ys = reinterpret_cast<float4*>(&s.ystage[r][32 * cb]);
#pragma unroll
      for (int v = 0; v < 8; ++v) {
        const float4 sw = __ldg(reinterpret_cast<const float4*>(wsc) + v);
        float2 lo = mul2(facc[2 * v], make_float2(sw.x, sw.y));
        float2 hi = mul2(facc[2 * v + 1], make_float2(sw.z, sw.w));
        if constexpr (!DENSE) {
          lo = mul2(lo, wr2);
          hi = mul2(hi, wr2);
        }
        ys[v] = make_float4(lo.x, lo.y, hi.x, hi.y);
      }
      quarter_sync(q);
      // the 4 warps of quarter q write its 32 rows: 8 rows each, one whole row per warp store
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int rr = q * 32 + cb * 8 + j;
        if (rr < ti.nvalid) {
          const float4 v = reinterpret_cast<const float4*>(&s.ystage[rr][0])[lane];
          if constexpr (DENSE) {
            const uint2 o = make_uint2((uint32_t)f2bf(v.x) | ((uint32_t)f2bf(v.y) << 16),
                                       (uint32_t)f2bf(v.z) | ((uint32_t)f2bf(v.w) << 16));
            reinterpret_cast<uint2*>(static_cast<uint16_t*>(yout) + (size_t)(ti.row0 + rr) * H +
                                     ti.col * BN)[lane] = o;
          } else {
            reinterpret_cast<float4*>(static_cast<float*>(yout) + (size_t)(ti.row0 + rr) * H +
                                      ti.col * BN)[lane] = v;
          }
        }
      }
      quarter_sync(q);  // staging rows read before the next tile overwrites them
    }
    if (!DENSE && lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");  // stores complete
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS2));
  }
  if (tid == 0 && s.failed) atomicExch(err, ERR_TIMEOUT);
}

// xg[pos] = x_i8[routes[pos].token], xg_sa[pos] = x_sa[token]: the routed
// activation rows in schedule order (one warp per route).
__global__ void __launch_bounds__(256)
gather_rows_kernel(const uint8_t* __restrict__ x, int row_bytes, const float* __restrict__ xsa,
                   const SparseRoute* __restrict__ routes, const int32_t* __restrict__ expert_offset,
                   int epr, uint8_t* __restrict__ xg, float* __restrict__ xg_sa) {
  pdl_wait();
  pdl_trigger();
  const int R = expert_offset[epr];
  const int lane = threadIdx.x & 31;
  const int n16 = row_bytes / 16;
  // GATHER_BATCH 16-byte units per lane are loaded before any is stored, so a
  // row (176 units for int8 rows) costs one L2 round trip, not six
  constexpr int GATHER_BATCH = 6;
  for (int pos = blockIdx.x * 8 + (threadIdx.x >> 5); pos < R; pos += gridDim.x * 8) {
    const int tok = routes[pos].token;
    const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)tok * row_bytes);
    uint4* dst = reinterpret_cast<uint4*>(xg + (size_t)pos * row_bytes);
    for (int c0 = 0; c0 < n16; c0 += 32 * GATHER_BATCH) {
      uint4 v[GATHER_BATCH];
#pragma unroll
      for (int i = 0; i < GATHER_BATCH; ++i) {
        const int c = c0 + i * 32 + lane;
        if (c < n16) v[i] = __ldg(src + c);
      }
#pragma unroll
      for (int i = 0; i < GATHER_BATCH; ++i) {
        const int c = c0 + i * 32 + lane;
        if (c < n16) dst[c] = v[i];
      }
    }
    if (lane == 0 && xsa) xg_sa[pos] = xsa[tok];
  }
}

}  // namespace tc

// ------------------------------------------------------------------ host side
namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

int sm_count() {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

}  // namespace

// 2-D int8 tensor map [rows][cols] with a box of box_rows x 128 bytes, 128-byte
// swizzle, zero fill outside the tensor.
bool make_tmap_2d(void* map, const void* base, long rows, int cols, int elem_bytes, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn || (reinterpret_cast<uintptr_t>(base) & 15) || ((long)cols * elem_bytes) % 16) return false;
  // boxes of 128 bytes (one 128-byte swizzle row) by box_rows rows
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * elem_bytes};
  cuuint32_t box[2] = {(cuuint32_t)(128 / elem_bytes), (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  return fn(reinterpret_cast<CUtensorMap*>(map),
            elem_bytes == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
            : elem_bytes == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8, 2,
            const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_tmap_i8(void* map, const void* base, long rows, int cols, int box_rows) {
  return make_tmap_2d(map, base, rows, cols, 1, box_rows);
}

size_t tmap_bytes() { return sizeof(CUtensorMap); }

cudaError_t launch_gather_rows(const void* x, int row_bytes, const float* xsa,
                               const SparseRoute* routes, const int32_t* expert_offset, int epr,
                               int T, void* xg, float* xg_sa, cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  const int rows = T * TOPK;
  const int grid = std::min((rows + 7) / 8, 148 * 8);
  return launch_k(tc::gather_rows_kernel, dim3(grid), dim3(256), 0, s,
                  static_cast<const uint8_t*>(x), row_bytes, xsa, routes, expert_offset, epr,
                  static_cast<uint8_t*>(xg), xg_sa);
}

cudaError_t launch_tc_phase1(const void* map_a, const void* map_b, const int32_t* expert_offset,
                             int epr, int T, const float* xg_sa, const float* gu_scale,
                             int8_t* bucket_i8, float* bucket_sa, uint16_t* bucket_bf16, int* err,
                             cudaStream_t s) {
  const int max_rows = T * TOPK;
  const int max_tiles = (max_rows / tc::BM + epr) * tc::NJ1;
  const size_t smem = sizeof(tc::Smem1) + 1024;
  auto k = tc::tc_phase1_kernel<false>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  return launch_k(k, dim3(sm_count()), dim3(tc::THREADS), smem, s,
                  *reinterpret_cast<const CUtensorMap*>(map_a),
                  *reinterpret_cast<const CUtensorMap*>(map_b), expert_offset, epr, 0, xg_sa, gu_scale,
                  bucket_i8, bucket_sa, bucket_bf16, err, max_rows, max_tiles);
}

cudaError_t launch_tc_dense_gate_up(const void* map_x, const void* map_w, int T, const float* xsa,
                                    const float* gu_scale, int8_t* h_i8, float* h_sa,
                                    uint16_t* h_bf16, int* err, cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  const int tiles = (T + tc::BM - 1) / tc::BM * (DENSE_I / 64);
  const size_t smem = sizeof(tc::Smem1) + 1024;
  auto k = tc::tc_phase1_kernel<true>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  return launch_k(k, dim3(std::min(sm_count(), tiles)), dim3(tc::THREADS), smem, s,
                  *reinterpret_cast<const CUtensorMap*>(map_x),
                  *reinterpret_cast<const CUtensorMap*>(map_w), nullptr, 1, T, xsa, gu_scale, h_i8,
                  h_sa, h_bf16, err, T, tiles);
}

cudaError_t launch_tc_phase2(const void* map_a, const void* map_b, const void* map_y, const int32_t* expert_offset,
                             int epr, int T, const float* bsa, const SparseRoute* routes,
                             const float* dn_scale, float* ybuf, int* err, cudaStream_t s) {
  const int max_rows = T * TOPK;
  const int max_tiles = (max_rows / tc::BM + epr) * tc::NT2;
  const size_t smem = sizeof(tc::Smem2) + 1024;
  auto k = tc::tc_phase2_kernel<false>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  return launch_k(k, dim3(sm_count()), dim3(tc::THREADS), smem, s,
                  *reinterpret_cast<const CUtensorMap*>(map_a),
                  *reinterpret_cast<const CUtensorMap*>(map_b), *reinterpret_cast<const CUtensorMap*>(map_y),
                  expert_offset, epr, 0, bsa, routes, dn_scale, static_cast<void*>(ybuf), err, max_rows,
                  max_tiles);
}

cudaError_t launch_tc_dense_down(const void* map_h, const void* map_w, int T, const float* hsa,
                                 const float* dn_scale, uint16_t* out, int* err, cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  const int tiles = (T + tc::BM - 1) / tc::BM * tc::NT2;
  const size_t smem = sizeof(tc::Smem2) + 1024;
  auto k = tc::tc_phase2_kernel<true>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  return launch_k(k, dim3(std::min(sm_count(), tiles)), dim3(tc::THREADS), smem, s,
                  *reinterpret_cast<const CUtensorMap*>(map_h),
                  *reinterpret_cast<const CUtensorMap*>(map_w), *reinterpret_cast<const CUtensorMap*>(map_w),
                  nullptr, 1, T, hsa, nullptr, dn_scale, static_cast<void*>(out), err, T, tiles);
}

}  // namespace gm
