// gm_common.cuh -- shared device helpers for the sm_100a Gemma-4 MoE block.
//
// The reference engine (CoffeeVampir3/Mojo-Gemma4-CPU) defines its own float
// approximations (exp, tanh, gelu, softmax exp); they are restated here with
// the same operation order.  Every multiply/add that the reference writes as
// separate operations is written with __fmul_rn/__fadd_rn so nvcc cannot
// contract it into an FMA; __fmaf_rn appears only where the reference calls
// SIMD.fma().
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_bf16.h>

namespace gm {

constexpr int H = 2816;          // hidden (modeling/gemma4_common.mojo:5)
constexpr int E = 128;           // experts (:26)
constexpr int TOPK = 8;          // (:27)
constexpr int I = 704;           // expert intermediate (:24)
constexpr int GU = 1408;         // fused gate|up rows (:23)
constexpr int DOWN_BLOCK = 64;   // DOWN_FWHT_BLOCK (:25)
constexpr int NB_DOWN = I / DOWN_BLOCK;  // 11
constexpr int NORM_BLOCK = 128;  // FWHT block of the gate/up activation
constexpr int DENSE_I = 2112;    // dense MLP intermediate (modeling/gemma4_common.mojo:22)
constexpr int NB_DENSE = DENSE_I / DOWN_BLOCK;  // 33
constexpr int VNNI_N = 32;       // rows per packed N-tile (butterquant/vnni.mojo:13)
constexpr int VNNI_K = 64;       // cols per packed K-step (vnni.mojo:14)

// kernels/moe_router.mojo:33-36 SparseRoute{token, weight}: 8 bytes.
struct SparseRoute {
  int32_t token;
  float weight;
};

__device__ __forceinline__ float bf2f(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }

// butterquant/convert.mojo:13-17 round-to-nearest-even bf16 store.
__device__ __forceinline__ uint16_t f2bf(float f) {
  uint32_t bits = __float_as_uint(f);
  uint32_t rne = bits + ((bits >> 16) & 1u) + 0x7FFFu;
  return (uint16_t)(rne >> 16);
}

// simd_math/ops.mojo:25-31 quantize_i8: clamp(roundeven(v*inv), -128, 127)
// Clamping before rounding gives the same integer for every input (NaN and
// +-inf included); 1.5*2^23 + t for |t| <= 128 rounds to the nearest even
// integer in the low mantissa bits, so no float-to-int conversion is needed.
__device__ __forceinline__ int quantize_i8(float v, float inv) {
  const float t = fminf(fmaxf(__fmul_rn(v, inv), -128.0f), 127.0f);
  return __float_as_int(__fadd_rn(t, 12582912.0f)) - 0x4B400000;
}

// simd_math/ops.mojo:72-96 exp_f32_fast (~0.3% rel. error, x <= 0)
__device__ __forceinline__ float exp_f32_fast(float x) {
  const float LN2 = 0.6931471805599453f;
  const float INV_LN2 = 1.4426950408889634f;
  float xc = fmaxf(x, -87.0f);
  float xn = __fmul_rn(xc, INV_LN2);
  int n = __float2int_rn(xn);
  float r = __fsub_rn(xc, __fmul_rn((float)n, LN2));
  float p = __fadd_rn(1.0f, __fmul_rn(r, __fadd_rn(0.9999f,
                __fmul_rn(r, __fadd_rn(0.4985f, __fmul_rn(r, 0.1681f))))));
  int nc = max(n, -126);
  float pow2n = __uint_as_float((uint32_t)(nc + 127) << 23);
  return __fmul_rn(p, pow2n);
}

// simd_math/ops.mojo:127-141 tanh_f32
__device__ __forceinline__ float tanh_f32(float x) {
  uint32_t sign = __float_as_uint(x) & 0x80000000u;
  float ax = __uint_as_float(__float_as_uint(x) & 0x7FFFFFFFu);
  float e = exp_f32_fast(__fmul_rn(-2.0f, ax));
  float t = __fdiv_rn(__fsub_rn(1.0f, e), __fadd_rn(1.0f, e));
  return __uint_as_float(__float_as_uint(t) ^ sign);
}

// simd_math/ops.mojo:144-156 gelu_tanh_f32
__device__ __forceinline__ float gelu_tanh_f32(float x) {
  const float s2pi = 0.7978845608028654f;
  const float a = 0.044715f;
  float x3 = __fmul_rn(__fmul_rn(x, x), x);
  float inner = __fmul_rn(s2pi, __fadd_rn(x, __fmul_rn(a, x3)));
  float t = tanh_f32(inner);
  return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, t));
}

// simd_math/exponential.mojo:177-194 fast_exp_softmax_biased
__device__ __forceinline__ float fast_exp_softmax_biased(float x) {
  const float A_MAGIC = 12102203.16156148f;
  const float BIAS_F = 1059208216.0f;
  const float INV_TWO23 = 1.0f / (float)(1 << 23);
  const float QC_A = 1.6501418352127075f;
  const float QC_B = -0.37554836273193359f;
  const float QC_C = 0.38696467876434326f;
  int32_t i = __float2int_rz(__fadd_rn(__fmul_rn(A_MAGIC, x), BIAS_F));
  uint32_t u = (uint32_t)i;
  float k = __uint_as_float(u);
  float f = __fmul_rn((float)(u & 0x7FFFFFu), INV_TWO23);
  return __fmul_rn(k, __fadd_rn(QC_A, __fmul_rn(f, __fadd_rn(QC_B, __fmul_rn(f, QC_C)))));
}

// FWHT scale of butterquant/fwht.mojo:55: f32(1 / f64(sqrt_f32(block)))
__host__ __device__ constexpr float fwht_scale_128() { return 0.08838834764831845f; }
__host__ __device__ constexpr float fwht_scale_64() { return 0.125f; }

// Butterfly stage across lanes: lane with bit `m` clear keeps a+b, the lane
// with the bit set keeps a-b, where a is the lower lane's value (fwht.mojo:31-53).
// p - v and v + p as one fma with v scaled by -1 or +1 (both products exact).
__device__ __forceinline__ float fwht_xor_stage(float v, int lane, int m) {
  float p = __shfl_xor_sync(0xffffffffu, v, m);
  return __fmaf_rn(v, (lane & m) ? -1.0f : 1.0f, p);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, m));
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, m));
  return v;
}

// kernels/rmsnorm.mojo:45-46: inv_rms = sqrt(H) / sqrt(sum_sq + H*eps)
__device__ __forceinline__ float inv_rms_from_sumsq(float ss) {
  const float sqrt_n = __uint_as_float(0x42544395u);  // sqrt_f32(2816)
  const float n_eps = __uint_as_float(0x3b388ca4u);   // f32(2816) * f32(1e-6)
  return __fdiv_rn(sqrt_n, __fsqrt_rn(__fadd_rn(ss, n_eps)));
}

// 128-bit streaming load that bypasses L1 (weights are read once per call).
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}

// 16-byte global -> shared asynchronous copy (bypasses registers and L1).
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
  const uint32_t d = (uint32_t)__cvta_generic_to_shared(smem_dst);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
}
// 4-byte global -> shared asynchronous copy (through L1).
__device__ __forceinline__ void cp_async4(void* smem_dst, const void* gmem_src) {
  const uint32_t d = (uint32_t)__cvta_generic_to_shared(smem_dst);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(d), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// Waits until at most N committed groups of this thread are still in flight.
template <int N>
__device__ __forceinline__ void cp_async_wait_group() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// mma.sync m16n8k32 s8 x s8 -> s32 (fragment layout: PTX ISA, "Matrix
// Fragments for mma.m16n8k32").
__device__ __forceinline__ void mma_s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                       uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// mma.sync m16n8k16 bf16 x bf16 -> f32
__device__ __forceinline__ void mma_bf16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Programmatic dependent launch.  The forward's kernels are launched with
// programmatic stream serialisation, so kernel N+1 may start while kernel N is
// finishing; pdl_wait() blocks until the predecessor grid has completed and its
// writes are visible (a no-op for launches without the attribute), and
// pdl_trigger() lets the successor grid launch early.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;"); }

// Locate the expert owning global route-chunk `cg` given the per-expert chunk
// prefix `chunk_off[0..n]` (binary search; chunk_off is non-decreasing).
__device__ __forceinline__ int find_segment(const int* chunk_off, int n, int cg) {
  int lo = 0, hi = n;  // invariant: chunk_off[lo] <= cg < chunk_off[hi]
  while (hi - lo > 1) {
    int mid = (lo + hi) >> 1;
    if (__ldg(chunk_off + mid) <= cg) lo = mid; else hi = mid;
  }
  return lo;
}

}  // namespace gm
