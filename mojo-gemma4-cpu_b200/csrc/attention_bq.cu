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
// is bit-exact.  Decode: CTA = (token, KV head, KV split), 256 threads,
// tiles of 16 positions; each K and V row of the split is read once and
// serves every query head of the GQA group (see attn_decode_kernel); the CTA
// writes one partial (m, l, acc) per head and a merge kernel combines the
// splits.
#include "gm_kernels.h"

namespace gm {

namespace {

constexpr int AW = 16;                 // reference SIMD lanes (AVX-512 f32)
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

// CTA = (split, KV head g, token t), 256 threads, tiles of DEC_TP positions.  The
// K and V rows of a tile (and their scales) are copied into shared memory
// with cp.async one tile ahead (double buffer), then:
//  A. scores: mma.m16n8k32 s8 with the tile's positions as M and the
//     group's heads as N; the eight warps split K and their integer
//     partials are summed exactly;
//  B. softmax: the warp owning head h (h % 8) keeps its running max / sum and
//     turns the tile's scores into weights w*vs/127;
//  C. V: thread i owns columns [i*CPT, (i+1)*CPT) of every head: each V row is
//     converted once and used for all G heads.
constexpr int DEC_TP = 16;  // positions per tile

template <int HD>
struct DecodeSmem {
  static constexpr int TP = DEC_TP;
  static constexpr int RS = HD + 16;  // padded row: the 32 lanes of phase A hit distinct banks
  int8_t k[2][TP][RS];  // RS padding: lanes reading rows at one column hit distinct banks
  int8_t v[2][TP][RS];
  float ks[2][TP];
  float vs[2][TP];
};

constexpr int DEC_THREADS = 256;
constexpr int DEC_WARPS = DEC_THREADS / 32;

template <int HD, int G>
__global__ void __launch_bounds__(DEC_THREADS)
attn_decode_kernel(const int8_t* __restrict__ q_i8, const float* __restrict__ f_q,
                   const int8_t* __restrict__ k_cache, const float* __restrict__ k_scale,
                   const int8_t* __restrict__ v_cache, const float* __restrict__ v_scale,
                   const KvRun* __restrict__ runs, const int32_t* __restrict__ base_rows, int num_q,
                   int num_kv, int window, int cache_degree, int rank, int shift, int row_mask,
                   int page_mask, int n_splits, float* __restrict__ partials) {
  using Sm = DecodeSmem<HD>;
  constexpr int TP = Sm::TP;
  constexpr int NW = DEC_WARPS;
  constexpr int CPT = HD / DEC_THREADS;           // V columns per thread (the partial's layout)
  // Phase C: a thread accumulates PVC adjacent columns (one shared load of
  // PVC int8) over every PG-th position of the tile; with PG > 1 the PG
  // position groups' sums are added in group order at the end of the split.
  // Head 256 with 2 heads per group (the sliding layers): 4 columns x 4
  // groups, fewer loads and conversions per FMA than one column per thread;
  // otherwise CPT columns, one group.
  constexpr int PVC = (HD == 256 && G == 2) ? 4 : CPT;
  constexpr int PG = DEC_THREADS * PVC / HD;
  static_assert(PG == 1 || HD == DEC_THREADS, "the group sum maps one column to a thread");
  constexpr int HPW = (G + NW - 1) / NW;          // heads whose softmax state a warp keeps
  constexpr int TPR = DEC_THREADS / TP;           // copying threads per row
  constexpr int CHUNKS = HD / (16 * TPR);         // 16-byte chunks per copying thread
  constexpr int KSW = HD / 32 / NW;               // 32-wide K steps per warp
  static_assert(KSW >= 1 && CPT >= 1 && CHUNKS >= 1, "tile geometry");
  static_assert(G <= 8, "heads of a group fit the N = 8 tile");
  const int s = blockIdx.x, g = blockIdx.y, t = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int grp = lane >> 2, tig = lane & 3;
  extern __shared__ __align__(16) uint8_t dsm[];
  Sm& sm = *reinterpret_cast<Sm*>(dsm);
  __shared__ __align__(16) int8_t qs[G * HD];
  __shared__ int part[DEC_WARPS][G][TP];
  __shared__ __align__(16) float wv[TP][G];
  __shared__ float corr_s[G];

  pdl_wait();
  pdl_trigger();
  for (int i = tid; i < G * HD / 16; i += DEC_THREADS)
    reinterpret_cast<int4*>(qs)[i] =
        __ldg(reinterpret_cast<const int4*>(q_i8 + ((size_t)t * num_q + g * G) * HD) + i);
  __syncthreads();
  // B fragments of the query (k = 4*tig.., head = grp; heads past G are zero),
  // held for the whole split
  uint32_t bq[KSW][2];
#pragma unroll
  for (int ks = 0; ks < KSW; ++ks) {
    const int k0 = (warp * KSW + ks) * 32 + 4 * tig;
    bq[ks][0] = grp < G ? *reinterpret_cast<const uint32_t*>(qs + grp * HD + k0) : 0u;
    bq[ks][1] = grp < G ? *reinterpret_cast<const uint32_t*>(qs + grp * HD + k0 + 16) : 0u;
  }

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
  const size_t kvs = (size_t)num_kv * HD;
  // copy rows [p0, p0 + TP) of the split into buffer `buf`: thread tid copies
  // part tid % TPR of row tid / TPR (and one of its two scales)
  const int crow = tid / TPR, cpart = tid % TPR;
  auto issue = [&](int p0, int buf) {
    const int p = p0 + crow;
    if (p < e) {
      const long slot = kv_slot(rows, shift, row_mask, page_mask, start + p);
      const int8_t* kr = k_cache + slot * kvs + (size_t)g * HD + cpart * (HD / TPR);
      const int8_t* vr = v_cache + slot * kvs + (size_t)g * HD + cpart * (HD / TPR);
#pragma unroll
      for (int c = 0; c < CHUNKS; ++c) {
        cp_async16(&sm.k[buf][crow][cpart * (HD / TPR) + 16 * c], kr + 16 * c);
        cp_async16(&sm.v[buf][crow][cpart * (HD / TPR) + 16 * c], vr + 16 * c);
      }
      if (cpart == 0) cp_async4(&sm.ks[buf][crow], k_scale + slot * num_kv + g);
      if (cpart == 1) cp_async4(&sm.vs[buf][crow], v_scale + slot * num_kv + g);
    }
    cp_async_commit();
  };

  const float inv127 = 1.0f / 127.0f;
  const float inv127sq = __fmul_rn(inv127, inv127);
  float fq[HPW], m[HPW], l[HPW];
#pragma unroll
  for (int j = 0; j < HPW; ++j) {
    const int h = warp + NW * j;
    fq[j] = h < G ? __ldg(f_q + (size_t)t * num_q + g * G + h) : 0.0f;
    m[j] = NEG_BIG;
    l[j] = 0.0f;
  }
  const int cg = tid % (HD / PVC), pg = tid / (HD / PVC);
  float acc[G][PVC];
#pragma unroll
  for (int h = 0; h < G; ++h)
#pragma unroll
    for (int c = 0; c < PVC; ++c) acc[h][c] = 0.0f;

  if (b < e) issue(b, 0);
  int buf = 0;
  for (int p0 = b; p0 < e; p0 += TP, buf ^= 1) {
    const int n = min(TP, e - p0);
    if (p0 + TP < e) {
      issue(p0 + TP, buf ^ 1);  // next tile in flight during this one
      cp_async_wait_group<1>();
    } else {
      cp_async_wait_group<0>();
    }
    __syncthreads();
    // ---- A: QK on the tensor cores (mma.m16n8k32 s8): positions are M (TP/16
    // 16-row tiles), the group's heads N (8, zero-padded), K split over the warps
    constexpr int MT = TP / 16;
    const bool ok = lane < n;  // n <= TP
    {
      int c[MT][4];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int i = 0; i < 4; ++i) c[mt][i] = 0;
#pragma unroll
      for (int ks = 0; ks < KSW; ++ks) {
        const int k0 = (warp * KSW + ks) * 32 + 4 * tig;
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          const int8_t* r0 = &sm.k[buf][mt * 16 + grp][k0];
          const int8_t* r1 = &sm.k[buf][mt * 16 + grp + 8][k0];
          mma_s8(c[mt], *reinterpret_cast<const uint32_t*>(r0), *reinterpret_cast<const uint32_t*>(r1),
                 *reinterpret_cast<const uint32_t*>(r0 + 16), *reinterpret_cast<const uint32_t*>(r1 + 16),
                 bq[ks][0], bq[ks][1]);
        }
      }
      // c[mt][0..1]: position mt*16 + grp, heads 2*tig, 2*tig+1; [2..3]: position + 8
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int h = 2 * tig + (i & 1);
          if (h < G) part[warp][h][mt * 16 + grp + 8 * (i >> 1)] = c[mt][i];
        }
    }
    __syncthreads();
    // ---- B: online softmax of the heads this warp owns
    {
      const float ks = ok ? sm.ks[buf][lane] : 0.0f;
      const float vs = ok ? sm.vs[buf][lane] : 0.0f;
      const int pl = ok ? lane : 0;  // lanes past the tile read row 0 and are masked
#pragma unroll
      for (int j = 0; j < HPW; ++j) {
        const int h = warp + NW * j;
        if (h < G) {
          int dot = 0;
#pragma unroll
          for (int w = 0; w < NW; ++w) dot += part[w][h][pl];
          const float sc = ok ? __fmul_rn(__fmul_rn(__fmul_rn((float)dot, fq[j]), ks), inv127sq) : NEG_BIG;
          const float mn = fmaxf(m[j], warp_max(sc));
          const float cr = fast_exp_softmax_biased(fmaxf(-87.0f, __fsub_rn(m[j], mn)));
          const float w = ok ? fast_exp_softmax_biased(fmaxf(-87.0f, __fsub_rn(sc, mn))) : 0.0f;
          l[j] = __fadd_rn(__fmul_rn(l[j], cr), warp_sum(w));
          m[j] = mn;
          if (lane < TP) wv[lane][h] = __fmul_rn(__fmul_rn(w, vs), inv127);
          if (lane == 0) corr_s[h] = cr;
        }
      }
    }
    __syncthreads();
    // ---- C: acc = acc*corr + sum_p v[p] * wv[p]
#pragma unroll
    for (int h = 0; h < G; ++h) {
      const float cr = corr_s[h];
#pragma unroll
      for (int c = 0; c < PVC; ++c) acc[h][c] = __fmul_rn(acc[h][c], cr);
    }
#pragma unroll 4
    for (int p = pg; p < n; p += PG) {
      uint32_t vw;
      if constexpr (PVC == 4) vw = *reinterpret_cast<const uint32_t*>(&sm.v[buf][p][cg * PVC]);
      else if constexpr (PVC == 2) vw = *reinterpret_cast<const uint16_t*>(&sm.v[buf][p][cg * PVC]);
      else vw = (uint32_t)(uint8_t)sm.v[buf][p][cg * PVC];
      float v[PVC];
#pragma unroll
      for (int c = 0; c < PVC; ++c) v[c] = (float)(int8_t)((vw >> (8 * c)) & 0xFFu);
      float a[G];
      if constexpr (G == 2) {
        const float2 w2 = *reinterpret_cast<const float2*>(&wv[p][0]);
        a[0] = w2.x;
        a[1] = w2.y;
      } else if constexpr (G % 4 == 0) {
#pragma unroll
        for (int h4 = 0; h4 < G / 4; ++h4) {
          const float4 w4 = reinterpret_cast<const float4*>(&wv[p][0])[h4];
          a[4 * h4] = w4.x;
          a[4 * h4 + 1] = w4.y;
          a[4 * h4 + 2] = w4.z;
          a[4 * h4 + 3] = w4.w;
        }
      } else {
#pragma unroll
        for (int h = 0; h < G; ++h) a[h] = wv[p][h];
      }
#pragma unroll
      for (int h = 0; h < G; ++h)
#pragma unroll
        for (int c = 0; c < PVC; ++c) acc[h][c] = __fmaf_rn(v[c], a[h], acc[h][c]);
    }
    __syncthreads();  // this buffer and part / wv / corr_s are reused
  }

  // one partial (m, l, acc) per head of the group
  if constexpr (PG > 1) {
    // the position groups' sums meet in the K buffers (free after the loop's
    // last barrier), then thread tid adds column tid's groups in order
    static_assert(PVC == 4 && sizeof(sm.k) >= sizeof(float) * PG * G * HD, "group sum fits the K buffers");
    float* red = reinterpret_cast<float*>(&sm.k[0][0][0]);
#pragma unroll
    for (int h = 0; h < G; ++h)
      reinterpret_cast<float4*>(red + (size_t)(pg * G + h) * HD)[cg] =
          make_float4(acc[h][0], acc[h][1], acc[h][2], acc[h][3]);
    __syncthreads();
#pragma unroll
    for (int h = 0; h < G; ++h) {
      float sum = red[(size_t)h * HD + tid];
#pragma unroll
      for (int q = 1; q < PG; ++q) sum = __fadd_rn(sum, red[(size_t)(q * G + h) * HD + tid]);
      partials[(((size_t)t * num_q + g * G + h) * n_splits + s) * (HD + 2) + 2 + tid] = sum;
    }
  } else {
#pragma unroll
    for (int h = 0; h < G; ++h) {
      float* dst = partials + (((size_t)t * num_q + g * G + h) * n_splits + s) * (HD + 2);
#pragma unroll
      for (int c = 0; c < PVC; ++c) dst[2 + cg * PVC + c] = acc[h][c];
    }
  }
  if (lane == 0) {
#pragma unroll
    for (int j = 0; j < HPW; ++j) {
      const int h = warp + NW * j;
      if (h < G) {
        float* dst = partials + (((size_t)t * num_q + g * G + h) * n_splits + s) * (HD + 2);
        dst[0] = m[j];
        dst[1] = l[j];
      }
    }
  }
}

// Prefill (butterquant_kernels/attention.mojo:150-332 BqFlashPrefillSliding /
// BqFlashPrefillFull at degree 1): every token of a chunk attends to its own
// causal range of its run -- sliding: [max(0, p - window + 1), p], full:
// [0, p] -- over the cache the prep has just written.  CTA = (QT consecutive
// tokens, KV head g): its C = QT * G = 32 (token, head) columns share every
// K/V tile, so each cache row is read once per QT tokens instead of once per
// token.  Per tile of PF_TP positions (cp.async double buffer):
//  A. scores on the tensor cores (mma.m16n8k32 s8): positions are M, the
//     columns N (C / 8 N-tiles), K split over the 8 warps, exact int32 sums;
//  B. online softmax per column (warp w owns columns w, w + 8, ...), with the
//     positions outside a column's range (causal / window / other run)
//     masked; the weights p = w * vs / 127 are stored as two bf16 parts,
//     hi = bf16(p) and lo = bf16(p - hi) (p to about 2^-17 relative); the V
//     tile is converted once into a transposed bf16 tile (int8 is exact in
//     bf16);
//  C. PV on the tensor cores (mma.m16n8k16 bf16, f32 accumulate): the columns
//     are M (2 M-tiles), the positions K, the head dimension N (warp w owns
//     HD/8 of it); acc = acc * corr + P_hi V + P_lo V.
// The tile's tokens may span runs (sequences): the runs are visited in turn,
// each over the union of its tokens' ranges.  Output bf16(acc / l).
constexpr int PF_TP = 16;
constexpr int PF_STR = PF_TP + 8;  // bf16 row stride of the transposed tiles: conflict-free fragment loads

constexpr int PF_STAGES = 2;       // K/V tiles in the cp.async ring (one ahead of the one in use)

template <int HD>
struct PrefillRing {
  static constexpr int TP = PF_TP;
  static constexpr int RS = HD + 16;  // padded row, as DecodeSmem
  int8_t k[PF_STAGES][TP][RS];
  int8_t v[PF_STAGES][TP][RS];
  float ks[PF_STAGES][TP];
  float vs[PF_STAGES][TP];
};

template <int HD, int C>
struct PrefillSmem {
  PrefillRing<HD> kv;
  uint16_t vt[HD][PF_STR];   // V tile transposed: [head column][position]
  uint16_t phi[C][PF_STR];   // weights, high bf16 part: [column][position]
  uint16_t plo[C][PF_STR];   // low bf16 part
};

template <int HD, int G, int QT>
__global__ void __launch_bounds__(DEC_THREADS, 2)
attn_prefill_kernel(const int8_t* __restrict__ q_i8, const float* __restrict__ f_q,
                    const int8_t* __restrict__ k_cache, const float* __restrict__ k_scale,
                    const int8_t* __restrict__ v_cache, const float* __restrict__ v_scale,
                    const KvRun* __restrict__ runs, int num_runs, const int32_t* __restrict__ base_rows,
                    int T, int num_q, int num_kv, int window, int shift, int row_mask, int page_mask,
                    uint16_t* __restrict__ out) {
  constexpr int C = QT * G;                       // (token, head) columns
  using Sm = PrefillSmem<HD, C>;
  static_assert(C == 32, "two 16-row M-tiles of columns");
  constexpr int NT = C / 8;                       // QK mma N-tiles
  constexpr int NW = DEC_WARPS;
  constexpr int CPW = C / NW;                     // softmax columns per warp
  constexpr int KS2 = HD / 32 / 2;                // QK: warp pair (2nt, 2nt+1) = one N-tile, K in halves
  constexpr int TPR = DEC_THREADS / PF_TP;        // copying threads per row
  constexpr int CHUNKS = HD / (16 * TPR);
  constexpr int NPW = HD / NW;                    // head columns per warp in PV
  constexpr int NTW = NPW / 8;                    // PV mma N-tiles per warp
  constexpr int VPT = HD / DEC_THREADS;           // V columns each thread transposes
  static_assert(NT * 2 == NW && CPW == 4 && KS2 >= 1 && CHUNKS >= 1 && NTW >= 1 && (VPT == 1 || VPT == 2),
                "tile geometry");
  const int t0 = blockIdx.x * QT, g = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int grp = lane >> 2, tig = lane & 3;
  extern __shared__ __align__(16) uint8_t dsm[];
  Sm& sm = *reinterpret_cast<Sm*>(dsm);
  __shared__ __align__(16) int8_t qs[C * HD];
  __shared__ int part[2][C][PF_TP];  // the two K halves of every score
  __shared__ float corr_s[C];
  __shared__ float l_s[C];

  pdl_wait();
  pdl_trigger();
  // the tile's queries: column col = tq * G + h is token t0 + tq, head g*G + h
  for (int i = tid; i < C * HD / 16; i += DEC_THREADS) {
    const int col = i / (HD / 16), u = i % (HD / 16);
    const int t = t0 + col / G;
    int4 v = make_int4(0, 0, 0, 0);
    if (t < T) v = __ldg(reinterpret_cast<const int4*>(q_i8 + ((size_t)t * num_q + g * G + col % G) * HD) + u);
    reinterpret_cast<int4*>(qs)[i] = v;
  }
  __syncthreads();
  // QK: warp w computes N-tile w/2 (8 columns) over K half w%2
  const int qnt = warp >> 1, qkh = warp & 1;
  uint32_t bq[KS2][2];
#pragma unroll
  for (int ks = 0; ks < KS2; ++ks) {
    const int k0 = (qkh * KS2 + ks) * 32 + 4 * tig;
    const int8_t* qc = qs + (qnt * 8 + grp) * HD + k0;
    bq[ks][0] = *reinterpret_cast<const uint32_t*>(qc);
    bq[ks][1] = *reinterpret_cast<const uint32_t*>(qc + 16);
  }
  // softmax: half-warp hf = lane / 16 of warp w owns columns w + 8*(2*pp + hf),
  // pp = 0, 1; lane % 16 is the position in the tile
  const int hf = lane >> 4, l16 = lane & 15;

  const float inv127 = 1.0f / 127.0f;
  const float inv127sq = __fmul_rn(inv127, inv127);
  float fq[CPW], m[CPW], l[CPW];
#pragma unroll
  for (int j = 0; j < CPW; ++j) {
    const int col = warp + NW * j, t = t0 + col / G;
    fq[j] = t < T ? __ldg(f_q + (size_t)t * num_q + g * G + col % G) : 0.0f;
    m[j] = NEG_BIG;
    l[j] = 0.0f;
  }
  // acc[mt][nt]: columns mt*16 + grp (+8 for [2..3]), head columns
  // warp*NPW + nt*8 + 2*tig (+1)
  float acc[2][NTW][4];
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int nt = 0; nt < NTW; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[mt][nt][i] = 0.0f;

  const size_t kvs = (size_t)num_kv * HD;
  const int t_end = min(t0 + QT, T);
  const int r_first = find_run(runs, num_runs, t0), r_last = find_run(runs, num_runs, t_end - 1);
  for (int r = r_first; r <= r_last; ++r) {
    const KvRun run = runs[r];
    const int run_end = r + 1 < num_runs ? __ldg(&runs[r + 1].buf_start) : T;
    const int tb = max(t0, run.buf_start), te = min(t_end, run_end);
    if (tb >= te) continue;
    // positions of the run's tokens in this tile; the union of their ranges
    const int pos_b = run.base_pos + (tb - run.buf_start), pos_e = run.base_pos + (te - 1 - run.buf_start);
    const int p_first = window > 0 ? max(0, pos_b - window + 1) : 0;
    const int p_last = pos_e;
    // the owned columns' ranges (empty for tokens outside this run)
    int c_lo[CPW], c_hi[CPW];
#pragma unroll
    for (int j = 0; j < CPW; ++j) {
      const int t = t0 + (warp + NW * j) / G;
      if (t >= tb && t < te) {
        const int p = run.base_pos + (t - run.buf_start);
        c_lo[j] = window > 0 ? max(0, p - window + 1) : 0;
        c_hi[j] = p;
      } else {
        c_lo[j] = 1;
        c_hi[j] = 0;
      }
    }
    const int32_t* rows = base_rows + run.rows_off;
    const int crow = tid / TPR, cpart = tid % TPR;
    auto issue = [&](int p0, int buf) {  // one commit group per call, empty past the range
      const int p = p0 + crow;
      if (p <= p_last) {
        const long slot = kv_slot(rows, shift, row_mask, page_mask, p);
        const int8_t* kr = k_cache + slot * kvs + (size_t)g * HD + cpart * (HD / TPR);
        const int8_t* vr = v_cache + slot * kvs + (size_t)g * HD + cpart * (HD / TPR);
#pragma unroll
        for (int cc = 0; cc < CHUNKS; ++cc) {
          cp_async16(&sm.kv.k[buf][crow][cpart * (HD / TPR) + 16 * cc], kr + 16 * cc);
          cp_async16(&sm.kv.v[buf][crow][cpart * (HD / TPR) + 16 * cc], vr + 16 * cc);
        }
        if (cpart == 0) cp_async4(&sm.kv.ks[buf][crow], k_scale + slot * num_kv + g);
        if (cpart == 1) cp_async4(&sm.kv.vs[buf][crow], v_scale + slot * num_kv + g);
      }
      cp_async_commit();
    };
#pragma unroll
    for (int i = 0; i < PF_STAGES - 1; ++i) issue(p_first + i * PF_TP, i);
    int buf = 0;
    for (int p0 = p_first; p0 <= p_last; p0 += PF_TP, buf = (buf + 1) % PF_STAGES) {
      const int n = min(PF_TP, p_last + 1 - p0);
      // tile p0 + (PF_STAGES-1)*PF_TP into the stage the previous tile used (all threads
      // are past it: the barrier that ends each tile)
      issue(p0 + (PF_STAGES - 1) * PF_TP, (buf + PF_STAGES - 1) % PF_STAGES);
      cp_async_wait_group<PF_STAGES - 1>();  // this tile's group has landed
      __syncthreads();
      // ---- A: scores (exact int32 partials of the two K halves)
      {
        int cacc[4] = {0, 0, 0, 0};
#pragma unroll
        for (int ks = 0; ks < KS2; ++ks) {
          const int k0 = (qkh * KS2 + ks) * 32 + 4 * tig;
          const int8_t* r0 = &sm.kv.k[buf][grp][k0];
          const int8_t* r1 = &sm.kv.k[buf][grp + 8][k0];
          const uint32_t a0 = *reinterpret_cast<const uint32_t*>(r0), a1 = *reinterpret_cast<const uint32_t*>(r1);
          const uint32_t a2 = *reinterpret_cast<const uint32_t*>(r0 + 16),
                         a3 = *reinterpret_cast<const uint32_t*>(r1 + 16);
          mma_s8(cacc, a0, a1, a2, a3, bq[ks][0], bq[ks][1]);
        }
        // cacc[0..1]: position grp, columns qnt*8 + 2*tig (+1); [2..3]: position grp + 8
#pragma unroll
        for (int i = 0; i < 4; ++i) part[qkh][qnt * 8 + 2 * tig + (i & 1)][grp + 8 * (i >> 1)] = cacc[i];
      }
      // V tile -> transposed bf16 (every position of the buffer: rows past n
      // hold finite stale bytes and meet zero weights)
      {
        uint32_t pk[VPT][PF_TP / 2];
#pragma unroll
        for (int pp = 0; pp < PF_TP; pp += 2) {
          uint32_t w0, w1;
          if constexpr (VPT == 2) {
            w0 = *reinterpret_cast<const uint16_t*>(&sm.kv.v[buf][pp][2 * tid]);
            w1 = *reinterpret_cast<const uint16_t*>(&sm.kv.v[buf][pp + 1][2 * tid]);
          } else {
            w0 = (uint8_t)sm.kv.v[buf][pp][tid];
            w1 = (uint8_t)sm.kv.v[buf][pp + 1][tid];
          }
#pragma unroll
          for (int x = 0; x < VPT; ++x) {
            const float v0 = (float)(int8_t)((w0 >> (8 * x)) & 0xFFu);
            const float v1 = (float)(int8_t)((w1 >> (8 * x)) & 0xFFu);
            pk[x][pp / 2] = (uint32_t)f2bf(v0) | ((uint32_t)f2bf(v1) << 16);
          }
        }
#pragma unroll
        for (int x = 0; x < VPT; ++x) {
          uint4* dst = reinterpret_cast<uint4*>(&sm.vt[VPT * tid + x][0]);
          dst[0] = make_uint4(pk[x][0], pk[x][1], pk[x][2], pk[x][3]);
          dst[1] = make_uint4(pk[x][4], pk[x][5], pk[x][6], pk[x][7]);
        }
      }
      __syncthreads();
      // ---- B: online softmax, two columns per warp at a time (one per
      // half-warp; the 16-lane trees give the 32-lane trees' results, as the
      // upper lanes only ever added -inf maxima and zero weights)
      {
        const bool in_tile = l16 < n;
        const float ksc = in_tile ? sm.kv.ks[buf][l16] : 0.0f;
        const float vsc = in_tile ? sm.kv.vs[buf][l16] : 0.0f;
        const int p = p0 + l16;
#pragma unroll
        for (int pp = 0; pp < 2; ++pp) {
          const int j0 = 2 * pp;  // this half's column index is j0 + hf
          const int col = warp + NW * (j0 + hf);
          const float fqj = hf ? fq[j0 + 1] : fq[j0];
          const float mj = hf ? m[j0 + 1] : m[j0];
          const float lj = hf ? l[j0 + 1] : l[j0];
          const int lo = hf ? c_lo[j0 + 1] : c_lo[j0], hi_p = hf ? c_hi[j0 + 1] : c_hi[j0];
          const bool ok = in_tile && p >= lo && p <= hi_p;
          const int dot = part[0][col][l16] + part[1][col][l16];
          const float sc = ok ? __fmul_rn(__fmul_rn(__fmul_rn((float)dot, fqj), ksc), inv127sq) : NEG_BIG;
          float mx = sc;
#pragma unroll
          for (int o = 8; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
          const float mn = fmaxf(mj, mx);
          const float cr = fast_exp_softmax_biased(fmaxf(-87.0f, __fsub_rn(mj, mn)));
          const float w = ok ? fast_exp_softmax_biased(fmaxf(-87.0f, __fsub_rn(sc, mn))) : 0.0f;
          float ws = w;
#pragma unroll
          for (int o = 8; o >= 1; o >>= 1) ws = __fadd_rn(ws, __shfl_xor_sync(0xffffffffu, ws, o));
          const float ln = __fadd_rn(__fmul_rn(lj, cr), ws);
          if (hf) { m[j0 + 1] = mn; l[j0 + 1] = ln; } else { m[j0] = mn; l[j0] = ln; }
          const float pw = __fmul_rn(__fmul_rn(w, vsc), inv127);
          const uint16_t hb = f2bf(pw);
          sm.phi[col][l16] = hb;
          sm.plo[col][l16] = f2bf(__fsub_rn(pw, bf2f(hb)));
          if (l16 == 0) corr_s[col] = cr;
        }
      }
      __syncthreads();
      // ---- C: acc = acc*corr + P V on the tensor cores
      {
        float cr[2][2];
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
          for (int h = 0; h < 2; ++h) cr[mt][h] = corr_s[mt * 16 + grp + 8 * h];
        uint32_t ah[2][4], al[2][4];
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
          const int c0 = mt * 16 + grp;
          ah[mt][0] = *reinterpret_cast<const uint32_t*>(&sm.phi[c0][2 * tig]);
          ah[mt][1] = *reinterpret_cast<const uint32_t*>(&sm.phi[c0 + 8][2 * tig]);
          ah[mt][2] = *reinterpret_cast<const uint32_t*>(&sm.phi[c0][2 * tig + 8]);
          ah[mt][3] = *reinterpret_cast<const uint32_t*>(&sm.phi[c0 + 8][2 * tig + 8]);
          al[mt][0] = *reinterpret_cast<const uint32_t*>(&sm.plo[c0][2 * tig]);
          al[mt][1] = *reinterpret_cast<const uint32_t*>(&sm.plo[c0 + 8][2 * tig]);
          al[mt][2] = *reinterpret_cast<const uint32_t*>(&sm.plo[c0][2 * tig + 8]);
          al[mt][3] = *reinterpret_cast<const uint32_t*>(&sm.plo[c0 + 8][2 * tig + 8]);
        }
#pragma unroll
        for (int nt = 0; nt < NTW; ++nt) {
          const int hc = warp * NPW + nt * 8 + grp;
          const uint32_t b0 = *reinterpret_cast<const uint32_t*>(&sm.vt[hc][2 * tig]);
          const uint32_t b1 = *reinterpret_cast<const uint32_t*>(&sm.vt[hc][2 * tig + 8]);
#pragma unroll
          for (int mt = 0; mt < 2; ++mt) {
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[mt][nt][i] = __fmul_rn(acc[mt][nt][i], cr[mt][i >> 1]);
            mma_bf16(acc[mt][nt], ah[mt][0], ah[mt][1], ah[mt][2], ah[mt][3], b0, b1);
            mma_bf16(acc[mt][nt], al[mt][0], al[mt][1], al[mt][2], al[mt][3], b0, b1);
          }
        }
      }
      __syncthreads();  // this buffer and part / vt / phi / plo / corr_s are reused
    }
  }
  if (l16 == 0) {
    l_s[warp + NW * hf] = hf ? l[1] : l[0];
    l_s[warp + NW * (2 + hf)] = hf ? l[3] : l[2];
  }
  __syncthreads();
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int c = mt * 16 + grp + 8 * h;
      const int t = t0 + c / G;
      if (t >= T) continue;
      const float lc = l_s[c];
      const float il = lc > 0.0f ? __fdiv_rn(1.0f, lc) : 0.0f;
      uint16_t* dst = out + ((size_t)t * num_q + g * G + c % G) * HD + warp * NPW + 2 * tig;
#pragma unroll
      for (int nt = 0; nt < NTW; ++nt) {
        const uint32_t o = lc > 0.0f ? (uint32_t)f2bf(__fmul_rn(acc[mt][nt][2 * h], il)) |
                                           ((uint32_t)f2bf(__fmul_rn(acc[mt][nt][2 * h + 1], il)) << 16)
                                     : 0u;
        *reinterpret_cast<uint32_t*>(dst + nt * 8) = o;
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

// The splits of one (token, head) reduced to ONE unnormalised partial
// (m, l, acc) over this rank's positions -- the value each rank of a
// position-sharded full-layer cache contributes to the cross-rank merge
// (kernels/logsum_merge.mojo:29-96): m = max_s m_s, c_s =
// exp(m_s - m) (0 when l_s = 0), l = sum l_s c_s, acc = sum acc_s c_s.
template <int HD>
__global__ void __launch_bounds__(HD)
attn_rank_partial_kernel(const float* __restrict__ partials, int n_splits, float* __restrict__ part) {
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
  float* dst = part + th * (HD + 2);
  if (threadIdx.x == 0) {
    dst[0] = M;
    dst[1] = L;
  }
  dst[2 + threadIdx.x] = o;
}

// The ranks' partials (each [T * num_q][HD + 2], rank order) merged and
// normalised: the same log-sum merge, then bf16(acc / l) (0 when l = 0).
struct PartList {
  const float* p[8];
  int n;
};
template <int HD>
__global__ void __launch_bounds__(HD)
attn_merge_parts_kernel(const __grid_constant__ PartList parts, uint16_t* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const size_t th = blockIdx.x;
  float M = NEG_BIG;
  for (int r = 0; r < parts.n; ++r) M = fmaxf(M, parts.p[r][th * (HD + 2)]);
  float L = 0.0f, o = 0.0f;
  for (int r = 0; r < parts.n; ++r) {
    const float* ps = parts.p[r] + th * (HD + 2);
    const float ls = ps[1];
    if (!(ls > 0.0f)) continue;
    const float c = fast_exp_softmax_biased(fmaxf(-87.0f, __fsub_rn(ps[0], M)));
    L = __fmaf_rn(ls, c, L);
    o = __fmaf_rn(ps[2 + threadIdx.x], c, o);
  }
  out[th * HD + threadIdx.x] = L > 0.0f ? f2bf(__fmul_rn(o, __fdiv_rn(1.0f, L))) : (uint16_t)0;
}

}  // namespace

cudaError_t launch_attn_prefill(const int8_t* q_i8, const float* f_q, const int8_t* k_cache, const float* k_scale,
                                const int8_t* v_cache, const float* v_scale, const void* runs, int num_runs,
                                const int32_t* base_rows, int T, int head_dim, int num_q, int num_kv, int window,
                                int shift, int row_mask, int page_mask, uint16_t* out, cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  const int G = num_q / num_kv;
  const KvRun* r = static_cast<const KvRun*>(runs);
  // 32 (token, head) columns per CTA: the GQA group's heads times the tokens
  if (head_dim == 256 && G == 2) {
    constexpr int QT = 16;
    auto k = attn_prefill_kernel<256, 2, QT>;
    const size_t smem = sizeof(PrefillSmem<256, QT * 2>);
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    return launch_k(k, dim3((T + QT - 1) / QT, num_kv), dim3(DEC_THREADS), smem, s, q_i8, f_q, k_cache, k_scale,
                    v_cache, v_scale, r, num_runs, base_rows, T, num_q, num_kv, window, shift, row_mask, page_mask,
                    out);
  }
  if (head_dim == 512 && G == 8) {
    constexpr int QT = 4;
    auto k = attn_prefill_kernel<512, 8, QT>;
    const size_t smem = sizeof(PrefillSmem<512, QT * 8>);
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    return launch_k(k, dim3((T + QT - 1) / QT, num_kv), dim3(DEC_THREADS), smem, s, q_i8, f_q, k_cache, k_scale,
                    v_cache, v_scale, r, num_runs, base_rows, T, num_q, num_kv, window, shift, row_mask, page_mask,
                    out);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_attn_rank_partial(const float* partials, int T, int num_q, int head_dim, int n_splits,
                                     float* part, cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  if (head_dim == 256)
    return launch_k(attn_rank_partial_kernel<256>, dim3(T * num_q), dim3(256), 0, s, partials, n_splits, part);
  return launch_k(attn_rank_partial_kernel<512>, dim3(T * num_q), dim3(512), 0, s, partials, n_splits, part);
}

cudaError_t launch_attn_merge_parts(const float* const* parts, int n, int T, int num_q, int head_dim,
                                    uint16_t* out, cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  if (n < 1 || n > 8) return cudaErrorInvalidValue;
  PartList pl = {};
  for (int r = 0; r < n; ++r) pl.p[r] = parts[r];
  pl.n = n;
  if (head_dim == 256)
    return launch_k(attn_merge_parts_kernel<256>, dim3(T * num_q), dim3(256), 0, s, pl, out);
  return launch_k(attn_merge_parts_kernel<512>, dim3(T * num_q), dim3(512), 0, s, pl, out);
}

using DecodeKernel = void (*)(const int8_t*, const float*, const int8_t*, const float*, const int8_t*,
                              const float*, const KvRun*, const int32_t*, int, int, int, int, int, int, int,
                              int, int, float*);

DecodeKernel decode_kernel_for(int head_dim, int G) {
  if (head_dim == 256) {
    if (G == 2) return attn_decode_kernel<256, 2>;
    if (G == 4) return attn_decode_kernel<256, 4>;
    if (G == 8) return attn_decode_kernel<256, 8>;
  } else if (head_dim == 512) {
    if (G == 2) return attn_decode_kernel<512, 2>;
    if (G == 4) return attn_decode_kernel<512, 4>;
    if (G == 8) return attn_decode_kernel<512, 8>;
  }
  return nullptr;
}

size_t decode_smem(int head_dim) {
  return head_dim == 256 ? sizeof(DecodeSmem<256>) : sizeof(DecodeSmem<512>);
}

// KV splits per (token, KV head).  Every split is one CTA; the decode kernel
// is latency-bound per CTA, so the time of a call is about (waves of resident
// CTAs) x (positions per split + a fixed per-CTA cost of ~48 positions).  The
// split count minimises that over 1..min(64, max_kv_len / 64) (at least 64
// positions per split), the resident CTAs per SM from the occupancy of the
// kernel that runs; the smallest count wins a tie (fewer partials to merge).
int attention_splits(int T, int head_dim, int num_q, int num_kv, int max_kv_len) {
  if (T <= 0 || num_kv <= 0 || max_kv_len <= 0) return 1;
  int per_sm = 0;
  const DecodeKernel k = decode_kernel_for(head_dim, num_q / num_kv);
  if (!k || cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, DEC_THREADS, decode_smem(head_dim)) !=
                cudaSuccess || per_sm <= 0) {
    cudaGetLastError();
    per_sm = 2048 / DEC_THREADS;
  }
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) {
    cudaGetLastError();
    sms = 148;
  }
  const long slots = (long)sms * per_sm, units = (long)T * num_kv;
  const int cap = std::max(1, std::min(64, (max_kv_len + 63) / 64));
  int best = 1;
  long best_cost = -1;
  for (int s = 1; s <= cap; ++s) {
    const long waves = (units * s + slots - 1) / slots;
    const long cost = waves * ((max_kv_len + s - 1) / s + 48);
    if (best_cost < 0 || cost < best_cost) {
      best = s;
      best_cost = cost;
    }
  }
  return best;
}

size_t attention_workspace_floats(int T, int head_dim, int num_q, int num_kv, int max_kv_len) {
  return (size_t)T * num_q * attention_splits(T, head_dim, num_q, num_kv, max_kv_len) * (head_dim + 2);
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
  const int n_splits = attention_splits(T, head_dim, num_q, num_kv, max_kv_len);
  const KvRun* r = static_cast<const KvRun*>(runs);
  const dim3 grid(n_splits, num_kv, T);
  const DecodeKernel k = decode_kernel_for(head_dim, num_q / num_kv);
  if (!k) return cudaErrorInvalidValue;
  const size_t smem = decode_smem(head_dim);
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  e = launch_k(k, grid, dim3(DEC_THREADS), smem, s, q_i8, f_q, k_cache, k_scale, v_cache, v_scale, r, base_rows,
                           num_q, num_kv, window, cache_degree, rank, shift, row_mask, page_mask, n_splits,
                           partials);
  if (e != cudaSuccess) return e;
  if (!out) return cudaSuccess;  // the caller reduces the splits (launch_attn_rank_partial)
  if (head_dim == 256)
    return launch_k(attn_merge_kernel<256>, dim3(T * num_q), dim3(256), 0, s, (const float*)partials,
                    n_splits, out);
  return launch_k(attn_merge_kernel<512>, dim3(T * num_q), dim3(512), 0, s, (const float*)partials, n_splits,
                  out);
}

}  // namespace gm
