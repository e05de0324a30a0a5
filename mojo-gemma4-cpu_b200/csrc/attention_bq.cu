// attention_bq.cu -- butterquant attention for decode: head prep into the
// int8 FWHT-rotated paged KV cache, split-KV flash decode over it, and the
// log-sum merge of the splits.
//
// Reference:
//  * prep (butterquant_kernels/attention.mojo:474-560 BqAttnPrepKernel with
//    butterquant/head_prep.mojo:9-97): per head, RMSNorm (sqrt(d)/sqrt(ssq +
//    d*eps)) times the q/k gain, RoPE over rope_half lanes pairing e with
//    e + pair_stride, FWHT over the head, absmax int8.  q: q_i8, qi_bias =
//    128*sum(q_i8), f_q = absmax; k and v (v: no gain, no rope) into cache row
//    kv.slot(pos / cache_degree) with their absmax as the row scale.
//  * decode (attention.mojo:33-146 bq_process_kv_tile, kernels/attention_ops.
//    mojo:196-212 online softmax, kernels/logsum_merge.mojo:29-117): score =
//    f32(q.k) * f_q * ks / 127^2 (the reference's shifted VNNI dot minus
//    qi_bias is this signed dot exactly), running max / sum with the
//    reference's fast_exp_softmax_biased, acc += v * (w * vs / 127) in the
//    rotated domain, partials merged with max-rescaled sums, bf16 output.
//
// B200 shape.  Prep: a half-warp per head, element e in lane e % 16 of
// register e / 16 -- the reference's 16-lane SIMD layout, so the
// sum-of-squares chains and their lane tree are the reference's and the prep
// is bit-exact.  Decode: CTA = (token, KV head, KV split), 4 warps; a warp
// owns two query heads of the GQA group and a stripe of 32-position tiles:
// lane j scores position j of the tile from its own K row (dp4a against the
// query in shared memory), then all lanes stream each V row once (coalesced)
// into per-lane accumulators of head_dim/32 columns.  Warps that share heads
// merge in shared memory; the CTA writes one partial (m, l, acc) per head.
#include "gm_kernels.h"

namespace gm {

namespace {

constexpr int AW = 16;                 // reference SIMD lanes (AVX-512 f32)
constexpr int DEC_WARPS = 4;
constexpr int QW = 2;                  // query heads per warp
constexpr float NEG_BIG = -1e30f;      // the reference's initial running max

struct KvRun {
  int32_t buf_start, base_pos, rows_off, page_count;
};

// The 16 lanes of this half-warp (shuffles never leave it, so the two halves
// of a warp may work on different kinds of heads).
__device__ __forceinline__ unsigned half_mask() {
  return (threadIdx.x & 16) ? 0xFFFF0000u : 0x0000FFFFu;
}

__device__ __forceinline__ float half_tree_sum(float v, unsigned hm) {
  // SIMD.reduce_add of 16 lanes: v[i] + v[i + 8], then +4, +2, +1
#pragma unroll
  for (int m = 8; m >= 1; m >>= 1) v = __fadd_rn(v, __shfl_xor_sync(hm, v, m));
  return v;
}

__device__ __forceinline__ float half_max(float v, unsigned hm) {
#pragma unroll
  for (int m = 8; m >= 1; m >>= 1) v = fmaxf(v, __shfl_xor_sync(hm, v, m));
  return v;
}

__device__ __forceinline__ int find_run(const KvRun* runs, int num_runs, int t) {
  int lo = 0, hi = num_runs;  // runs[lo].buf_start <= t < runs[hi].buf_start
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (__ldg(&runs[mid].buf_start) <= t) lo = mid; else hi = mid;
  }
  return lo;
}

// kernels/attention_ops.mojo:41-52 PagedKV.slot
__device__ __forceinline__ long kv_slot(const int32_t* base_rows, int shift, int row_mask, int page_mask,
                                        int p) {
  return (long)__ldg(base_rows + ((p >> shift) & page_mask)) + (p & row_mask);
}

// One head on a half-warp (butterquant/head_prep.mojo:40-97): returns the
// absmax; the int8 values go to dst (element ri*16 + lt from register ri) when
// dst is non-NULL, their sum to *qsum when qsum is non-NULL.  ROPE: gain and
// rotary (q, k) or neither (v).
template <int HD, int RH, int PS, bool ROPE>
__device__ __forceinline__ float prep_head(const uint16_t* __restrict__ src, const uint16_t* __restrict__ gamma,
                                           const float* __restrict__ cosr, const float* __restrict__ sinr,
                                           int lt, unsigned hm, int8_t* __restrict__ dst, int* qsum) {
  constexpr int REGS = HD / AW;
  constexpr int RR = RH / AW, PR = PS / AW;
  static_assert(PR + RR <= REGS, "rotary pairs inside the head");
  float r[REGS];
#pragma unroll
  for (int ri = 0; ri < REGS; ++ri) r[ri] = bf2f(src[ri * AW + lt]);
  float ssq = __fmul_rn(r[0], r[0]);
#pragma unroll
  for (int ri = 1; ri < REGS; ++ri) ssq = __fmaf_rn(r[ri], r[ri], ssq);
  const float sqrt_n = __fsqrt_rn((float)HD);
  const float n_eps = __fmul_rn((float)HD, 1e-6f);
  const float inv = __fdiv_rn(sqrt_n, __fsqrt_rn(__fadd_rn(half_tree_sum(ssq, hm), n_eps)));
#pragma unroll
  for (int ri = 0; ri < REGS; ++ri) {
    r[ri] = __fmul_rn(r[ri], inv);
    if (ROPE) r[ri] = __fmul_rn(r[ri], bf2f(gamma[ri * AW + lt]));
  }
  if (ROPE) {
#pragma unroll
    for (int ri = 0; ri < RR; ++ri) {
      const float lo = r[ri], hi = r[PR + ri];
      const float cv = cosr[ri * AW + lt], sv = sinr[ri * AW + lt];
      r[ri] = __fsub_rn(__fmul_rn(lo, cv), __fmul_rn(hi, sv));
      r[PR + ri] = __fadd_rn(__fmul_rn(hi, cv), __fmul_rn(lo, sv));
    }
  }
  // FWHT over the head (butterquant/fwht.mojo:20-57): strides 1..8 across the
  // half-warp, then 16, 32, .. across registers; then the 1/sqrt(HD) scale
#pragma unroll
  for (int m = 1; m < AW; m <<= 1)
#pragma unroll
    for (int ri = 0; ri < REGS; ++ri) {
      const float p = __shfl_xor_sync(hm, r[ri], m);
      r[ri] = (lt & m) ? __fsub_rn(p, r[ri]) : __fadd_rn(r[ri], p);
    }
#pragma unroll
  for (int rs = 1; rs < REGS; rs <<= 1)
#pragma unroll
    for (int ri = 0; ri < REGS; ++ri)
      if (!(ri & rs)) {
        const float a = r[ri], b = r[ri + rs];
        r[ri] = __fadd_rn(a, b);
        r[ri + rs] = __fsub_rn(a, b);
      }
  // f32(1 / f64(sqrt_f32(HD)))
  const float sc = (float)(1.0 / (double)(HD == 256 ? 16.0f : 22.627416997969522f));
  float vmax = 0.0f;
#pragma unroll
  for (int ri = 0; ri < REGS; ++ri) {
    r[ri] = __fmul_rn(r[ri], sc);
    vmax = fmaxf(vmax, fabsf(r[ri]));
  }
  float amax = half_max(vmax, hm);
  if (amax < 1e-10f) amax = 1e-10f;
  const float qinv = __fdiv_rn(127.0f, amax);
  int s = 0;
#pragma unroll
  for (int ri = 0; ri < REGS; ++ri) {
    const int q = quantize_i8(r[ri], qinv);
    if (dst) dst[ri * AW + lt] = (int8_t)q;
    s += q;
  }
  if (qsum) {
#pragma unroll
    for (int m = 8; m >= 1; m >>= 1) s += __shfl_xor_sync(hm, s, m);
    *qsum = s;
  }
  return amax;
}

template <int HD, int RH, int PS>
__global__ void __launch_bounds__(256)
attn_prep_kernel(const uint16_t* __restrict__ q_src, const uint16_t* __restrict__ k_src,
                 const uint16_t* __restrict__ v_src, const uint16_t* __restrict__ q_norm,
                 const uint16_t* __restrict__ k_norm, int8_t* __restrict__ q_i8,
                 float* __restrict__ qi_bias, float* __restrict__ f_q, int8_t* __restrict__ k_cache,
                 float* __restrict__ k_scale, int8_t* __restrict__ v_cache, float* __restrict__ v_scale,
                 const float* __restrict__ cos_table, const float* __restrict__ sin_table,
                 const KvRun* __restrict__ runs, int num_runs, const int32_t* __restrict__ base_rows,
                 int T, int num_q, int num_kv, int cache_degree, int rank, int shift, int row_mask,
                 int page_mask) {
  pdl_wait();
  pdl_trigger();
  const int per_tok = num_q + 2 * num_kv;
  const int task = (blockIdx.x * blockDim.x + threadIdx.x) >> 4;  // one head per half-warp
  if (task >= T * per_tok) return;  // whole half-warps leave together
  const int lt = threadIdx.x & 15;
  const unsigned hm = half_mask();
  const int t = task / per_tok, k = task % per_tok;
  const KvRun run = runs[find_run(runs, num_runs, t)];
  const int pos = run.base_pos + (t - run.buf_start);
  const float* cosr = cos_table + (size_t)pos * RH;
  const float* sinr = sin_table + (size_t)pos * RH;
  const size_t qs = (size_t)num_q * HD, kvs = (size_t)num_kv * HD;
  if (k < num_q) {
    int qsum = 0;
    const float amax = prep_head<HD, RH, PS, true>(q_src + t * qs + (size_t)k * HD, q_norm, cosr, sinr, lt,
                                                   hm, q_i8 + t * qs + (size_t)k * HD, &qsum);
    if (lt == 0) {
      qi_bias[(size_t)t * num_q + k] = __fmul_rn((float)qsum, 128.0f);
      f_q[(size_t)t * num_q + k] = amax;
    }
    return;
  }
  if (pos % cache_degree != rank) return;  // another rank's cache row
  const bool is_k = k < num_q + num_kv;
  const int h = is_k ? k - num_q : k - num_q - num_kv;
  const long slot = kv_slot(base_rows + run.rows_off, shift, row_mask, page_mask, pos / cache_degree);
  float amax;
  if (is_k)
    amax = prep_head<HD, RH, PS, true>(k_src + t * kvs + (size_t)h * HD, k_norm, cosr, sinr, lt, hm,
                                       k_cache + slot * kvs + (size_t)h * HD, nullptr);
  else
    amax = prep_head<HD, RH, PS, false>(v_src + t * kvs + (size_t)h * HD, nullptr, cosr, sinr, lt, hm,
                                        v_cache + slot * kvs + (size_t)h * HD, nullptr);
  if (lt == 0) (is_k ? k_scale : v_scale)[slot * num_kv + h] = amax;
}

// kernels/helpers.mojo:182-190 worker_range
__device__ __forceinline__ void split_range(int total, int n, int s, int& b, int& e) {
  const int per = (total + n - 1) / n;
  b = s * per;
  e = min(b + per, total);
  if (b >= total) b = e = total;
}

template <int HD>
__global__ void __launch_bounds__(32 * DEC_WARPS)
attn_decode_kernel(const int8_t* __restrict__ q_i8, const float* __restrict__ f_q,
                   const int8_t* __restrict__ k_cache, const float* __restrict__ k_scale,
                   const int8_t* __restrict__ v_cache, const float* __restrict__ v_scale,
                   const KvRun* __restrict__ runs, const int32_t* __restrict__ base_rows, int num_q,
                   int num_kv, int window, int cache_degree, int rank, int shift, int row_mask,
                   int page_mask, int n_splits, float* __restrict__ partials) {
  constexpr int VPL = HD / 32;       // V columns per lane
  constexpr int QWORDS = HD / 4;     // int32 words per query head
  const int s = blockIdx.x, g = blockIdx.y, t = blockIdx.z;
  const int G = num_q / num_kv;      // query heads per KV head (even)
  const int n_hs = G / QW, wph = DEC_WARPS / n_hs;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hs = warp % n_hs, stripe = warp / n_hs;
  const int h0 = g * G + hs * QW;
  extern __shared__ __align__(16) uint8_t smem[];
  int* qs = reinterpret_cast<int*>(smem);                               // [G][QWORDS]
  float* red = reinterpret_cast<float*>(qs + G * QWORDS);               // [DEC_WARPS][QW][HD + 2]

  pdl_wait();
  pdl_trigger();
  for (int i = threadIdx.x; i < G * QWORDS; i += blockDim.x)
    qs[i] = __ldg(reinterpret_cast<const int*>(q_i8 + ((size_t)t * num_q + g * G) * HD) + i);
  __syncthreads();

  const KvRun run = runs[t];
  const int pos = run.base_pos;
  int valid, start;
  if (window > 0) {  // sliding: the last min(pos + 1, window) positions
    valid = pos + 1 >= window ? window : pos + 1;
    start = pos - valid + 1;
  } else {           // full: this rank's positions (kernels/attention_ops.mojo:167-173)
    valid = rank <= pos % cache_degree ? pos / cache_degree + 1 : pos / cache_degree;
    start = 0;
  }
  const int32_t* rows = base_rows + run.rows_off;
  int b, e;
  split_range(valid, n_splits, s, b, e);
  const float inv127 = 1.0f / 127.0f;
  const float inv127sq = __fmul_rn(inv127, inv127);
  const float fq0 = __ldg(f_q + (size_t)t * num_q + h0), fq1 = __ldg(f_q + (size_t)t * num_q + h0 + 1);
  const size_t kvs = (size_t)num_kv * HD;

  float m[QW] = {NEG_BIG, NEG_BIG}, l[QW] = {0.0f, 0.0f};
  float acc[QW][VPL];
#pragma unroll
  for (int a = 0; a < QW; ++a)
#pragma unroll
    for (int c = 0; c < VPL; ++c) acc[a][c] = 0.0f;
  const int* q0 = qs + (hs * QW) * QWORDS;
  const int* q1 = q0 + QWORDS;

  for (int p0 = b + stripe * 32; p0 < e; p0 += wph * 32) {
    const int i = p0 + lane;
    const bool ok = i < e;
    const long slot = ok ? kv_slot(rows, shift, row_mask, page_mask, start + i) : 0;
    float sc0 = NEG_BIG, sc1 = NEG_BIG, vs = 0.0f;
    if (ok) {
      const int4* kr = reinterpret_cast<const int4*>(k_cache + slot * kvs + (size_t)g * HD);
      int d0 = 0, d1 = 0;
#pragma unroll 4
      for (int c = 0; c < HD / 16; ++c) {
        const int4 kw = __ldg(kr + c);
        d0 = __dp4a(kw.x, q0[4 * c], d0);
        d0 = __dp4a(kw.y, q0[4 * c + 1], d0);
        d0 = __dp4a(kw.z, q0[4 * c + 2], d0);
        d0 = __dp4a(kw.w, q0[4 * c + 3], d0);
        d1 = __dp4a(kw.x, q1[4 * c], d1);
        d1 = __dp4a(kw.y, q1[4 * c + 1], d1);
        d1 = __dp4a(kw.z, q1[4 * c + 2], d1);
        d1 = __dp4a(kw.w, q1[4 * c + 3], d1);
      }
      const float ks = __ldg(k_scale + slot * num_kv + g);
      sc0 = __fmul_rn(__fmul_rn(__fmul_rn((float)d0, fq0), ks), inv127sq);
      sc1 = __fmul_rn(__fmul_rn(__fmul_rn((float)d1, fq1), ks), inv127sq);
      vs = __ldg(v_scale + slot * num_kv + g);
    }
    float w0, w1;
    {
      const float mn0 = fmaxf(m[0], warp_max(sc0)), mn1 = fmaxf(m[1], warp_max(sc1));
      const float c0 = fast_exp_softmax_biased(fmaxf(-87.0f, __fsub_rn(m[0], mn0)));
      const float c1 = fast_exp_softmax_biased(fmaxf(-87.0f, __fsub_rn(m[1], mn1)));
      w0 = ok ? fast_exp_softmax_biased(fmaxf(-87.0f, __fsub_rn(sc0, mn0))) : 0.0f;
      w1 = ok ? fast_exp_softmax_biased(fmaxf(-87.0f, __fsub_rn(sc1, mn1))) : 0.0f;
      l[0] = __fadd_rn(__fmul_rn(l[0], c0), warp_sum(w0));
      l[1] = __fadd_rn(__fmul_rn(l[1], c1), warp_sum(w1));
      m[0] = mn0;
      m[1] = mn1;
#pragma unroll
      for (int c = 0; c < VPL; ++c) {
        acc[0][c] = __fmul_rn(acc[0][c], c0);
        acc[1][c] = __fmul_rn(acc[1][c], c1);
      }
    }
    const float wv0 = __fmul_rn(__fmul_rn(w0, vs), inv127), wv1 = __fmul_rn(__fmul_rn(w1, vs), inv127);
    const int n = min(32, e - p0);
    for (int j = 0; j < n; ++j) {
      const long sj = (long)__shfl_sync(0xffffffffu, (int)slot, j);
      const float a0 = __shfl_sync(0xffffffffu, wv0, j), a1 = __shfl_sync(0xffffffffu, wv1, j);
      const int8_t* vr = v_cache + sj * kvs + (size_t)g * HD + lane * VPL;
      uint32_t vw[VPL / 4];
      if constexpr (VPL == 8) {
        const int2 x = __ldg(reinterpret_cast<const int2*>(vr));
        vw[0] = (uint32_t)x.x;
        vw[1] = (uint32_t)x.y;
      } else {
        const int4 x = __ldg(reinterpret_cast<const int4*>(vr));
        vw[0] = (uint32_t)x.x;
        vw[1] = (uint32_t)x.y;
        vw[2] = (uint32_t)x.z;
        vw[3] = (uint32_t)x.w;
      }
#pragma unroll
      for (int c = 0; c < VPL; ++c) {
        const float v = (float)(int8_t)((vw[c >> 2] >> (8 * (c & 3))) & 0xFFu);
        acc[0][c] = __fmaf_rn(v, a0, acc[0][c]);
        acc[1][c] = __fmaf_rn(v, a1, acc[1][c]);
      }
    }
  }

  // merge the stripes of each head set in shared memory, then one partial per head
  float* mine = red + (size_t)warp * QW * (HD + 2);
#pragma unroll
  for (int a = 0; a < QW; ++a) {
#pragma unroll
    for (int c = 0; c < VPL; ++c) mine[a * (HD + 2) + 2 + lane * VPL + c] = acc[a][c];
    if (lane == 0) {
      mine[a * (HD + 2)] = m[a];
      mine[a * (HD + 2) + 1] = l[a];
    }
  }
  __syncthreads();
  if (stripe == 0) {
    for (int a = 0; a < QW; ++a) {
      float M = NEG_BIG;
      for (int w = hs; w < DEC_WARPS; w += n_hs) M = fmaxf(M, red[((size_t)w * QW + a) * (HD + 2)]);
      float L = 0.0f;
      float o[VPL];
#pragma unroll
      for (int c = 0; c < VPL; ++c) o[c] = 0.0f;
      for (int w = hs; w < DEC_WARPS; w += n_hs) {
        const float* src = red + ((size_t)w * QW + a) * (HD + 2);
        const float cw = src[1] > 0.0f ? fast_exp_softmax_biased(fmaxf(-87.0f, __fsub_rn(src[0], M))) : 0.0f;
        L = __fmaf_rn(src[1], cw, L);
#pragma unroll
        for (int c = 0; c < VPL; ++c) o[c] = __fmaf_rn(src[2 + lane * VPL + c], cw, o[c]);
      }
      float* dst = partials + (((size_t)t * num_q + h0 + a) * n_splits + s) * (HD + 2);
#pragma unroll
      for (int c = 0; c < VPL; ++c) dst[2 + lane * VPL + c] = o[c];
      if (lane == 0) {
        dst[0] = M;
        dst[1] = L;
      }
    }
  }
}

// kernels/logsum_merge.mojo:29-117: one CTA per (token, head), a thread per column
template <int HD>
__global__ void __launch_bounds__(HD)
attn_merge_kernel(const float* __restrict__ partials, int n_splits, uint16_t* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const size_t th = blockIdx.x;  // token * num_q + head
  const float* p = partials + th * n_splits * (HD + 2);
  float M = NEG_BIG;
  for (int s = 0; s < n_splits; ++s) M = fmaxf(M, p[(size_t)s * (HD + 2)]);
  float L = 0.0f, o = 0.0f;
  for (int s = 0; s < n_splits; ++s) {
    const float* ps = p + (size_t)s * (HD + 2);
    const float ls = ps[1];
    if (!(ls > 0.0f)) continue;
    const float c = fast_exp_softmax_biased(fmaxf(-87.0f, __fsub_rn(ps[0], M)));
    L = __fmaf_rn(ls, c, L);
    o = __fmaf_rn(ps[2 + threadIdx.x], c, o);
  }
  out[th * HD + threadIdx.x] = L > 0.0f ? f2bf(__fmul_rn(o, __fdiv_rn(1.0f, L))) : (uint16_t)0;
}

}  // namespace

int attention_splits(int T, int num_kv, int max_kv_len) {
  const int want = (148 * 8 + T * num_kv - 1) / (T * num_kv);
  const int cap = std::max(1, (max_kv_len + 63) / 64);
  return std::max(1, std::min({want, cap, 32}));
}

size_t attention_workspace_floats(int T, int head_dim, int num_q, int num_kv, int max_kv_len) {
  return (size_t)T * num_q * attention_splits(T, num_kv, max_kv_len) * (head_dim + 2);
}

cudaError_t launch_attn_prep(const uint16_t* q_src, const uint16_t* k_src, const uint16_t* v_src,
                             const uint16_t* q_norm, const uint16_t* k_norm, int8_t* q_i8, float* qi_bias,
                             float* f_q, int8_t* k_cache, float* k_scale, int8_t* v_cache, float* v_scale,
                             const float* cos_table, const float* sin_table, const void* runs, int num_runs,
                             const int32_t* base_rows, int T, int head_dim, int num_q, int num_kv,
                             int rope_half, int pair_stride, int cache_degree, int rank, int shift,
                             int row_mask, int page_mask, cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  const long halves = (long)T * (num_q + 2 * num_kv);
  const int grid = (int)((halves * 16 + 255) / 256);
  const KvRun* r = static_cast<const KvRun*>(runs);
  // the two head geometries of Gemma-4 (modeling/gemma4_common.mojo:9-20 and
  // the pair strides of modeling/gemma_4_moe_bq.mojo:488-490, 565-589)
  if (head_dim == 256 && rope_half == 128 && pair_stride == 128)
    return launch_k(attn_prep_kernel<256, 128, 128>, dim3(grid), dim3(256), 0, s, q_src, k_src, v_src, q_norm,
                    k_norm, q_i8, qi_bias, f_q, k_cache, k_scale, v_cache, v_scale, cos_table, sin_table, r,
                    num_runs, base_rows, T, num_q, num_kv, cache_degree, rank, shift, row_mask, page_mask);
  if (head_dim == 512 && rope_half == 64 && pair_stride == 256)
    return launch_k(attn_prep_kernel<512, 64, 256>, dim3(grid), dim3(256), 0, s, q_src, k_src, v_src, q_norm,
                    k_norm, q_i8, qi_bias, f_q, k_cache, k_scale, v_cache, v_scale, cos_table, sin_table, r,
                    num_runs, base_rows, T, num_q, num_kv, cache_degree, rank, shift, row_mask, page_mask);
  return cudaErrorInvalidValue;
}

cudaError_t launch_attn_decode(const int8_t* q_i8, const float* f_q, const int8_t* k_cache,
                               const float* k_scale, const int8_t* v_cache, const float* v_scale,
                               const void* runs, const int32_t* base_rows, int T, int head_dim, int num_q,
                               int num_kv, int window, int cache_degree, int rank, int shift, int row_mask,
                               int page_mask, int max_kv_len, float* partials, uint16_t* out, cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  const int n_splits = attention_splits(T, num_kv, max_kv_len);
  const int G = num_q / num_kv;
  const size_t smem = (size_t)G * head_dim + (size_t)DEC_WARPS * QW * (head_dim + 2) * 4;
  const KvRun* r = static_cast<const KvRun*>(runs);
  const dim3 grid(n_splits, num_kv, T);
  cudaError_t e;
  if (head_dim == 256) {
    e = launch_k(attn_decode_kernel<256>, grid, dim3(32 * DEC_WARPS), smem, s, q_i8, f_q, k_cache, k_scale,
                 v_cache, v_scale, r, base_rows, num_q, num_kv, window, cache_degree, rank, shift, row_mask,
                 page_mask, n_splits, partials);
    if (e != cudaSuccess) return e;
    return launch_k(attn_merge_kernel<256>, dim3(T * num_q), dim3(256), 0, s, (const float*)partials,
                    n_splits, out);
  }
  e = launch_k(attn_decode_kernel<512>, grid, dim3(32 * DEC_WARPS), smem, s, q_i8, f_q, k_cache, k_scale,
               v_cache, v_scale, r, base_rows, num_q, num_kv, window, cache_degree, rank, shift, row_mask,
               page_mask, n_splits, partials);
  if (e != cudaSuccess) return e;
  return launch_k(attn_merge_kernel<512>, dim3(T * num_q), dim3(512), 0, s, (const float*)partials, n_splits,
                  out);
}

}  // namespace gm
