// moe_oracle.cpp -- CPU restatement of the Gemma-4 MoE block exactly as the
// Mojo reference engine (CoffeeVampir3/Mojo-Gemma4-CPU) computes it.
//
// TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the B200
// product library (libgmoe) and the timed CPU baseline of bench.py.  Nothing
// in the product path links, loads or calls it.
//
// PARITY UNPINNED: the reference is Mojo and no Mojo toolchain exists here or
// on the GPU hosts, and the reference ships no golden vectors / known-answer
// tests for its MoE path.  The restatement follows the reference source line
// by line (citations below are paths inside the reference project); the only
// pins are mathematical self-checks (FWHT orthonormality, quantizer spec
// identities, the router-merge softmax invariant of
// benchmarks/benchmark_router_merge.mojo:120-135) exercised in tests/.
//
// Floating point: built with -ffp-contract=off so every a*b+c below rounds
// twice exactly as written; explicit fmaf() appears only where the reference
// calls SIMD.fma().
#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>
#include <algorithm>
#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

constexpr int H = 2816;          // modeling/gemma4_common.mojo:5
constexpr int E = 128;           // :26
constexpr int TOPK = 8;          // :27
constexpr int I = 704;           // :24
constexpr int GU = 1408;         // :23
constexpr int DOWN_BLOCK = 64;   // :25
constexpr int NB_DOWN = I / DOWN_BLOCK;

inline float bf2f(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}
inline uint32_t f2bits(float f) { uint32_t u; std::memcpy(&u, &f, 4); return u; }
inline float bits2f(uint32_t u) { float f; std::memcpy(&f, &u, 4); return f; }

// butterquant/convert.mojo:13-17 (explicit RNE store, also what cast[bf16] does)
inline uint16_t f2bf(float f) {
  uint32_t bits = f2bits(f);
  uint32_t rne = bits + ((bits >> 16) & 1u) + 0x7FFFu;
  return (uint16_t)(rne >> 16);
}

// simd_math/ops.mojo:14-31  roundeven + clamp to [-128,127]
inline int8_t quantize_i8(float v, float inv) {
  float r = std::nearbyint(v * inv);  // default rounding mode = nearest-even
  r = std::max(r, -128.0f);
  r = std::min(r, 127.0f);
  return (int8_t)(int)r;
}

// simd_math/ops.mojo:72-96 exp_f32_fast
inline float exp_f32_fast(float x) {
  const float LN2 = 0.6931471805599453f;
  const float INV_LN2 = 1.4426950408889634f;
  float xc = std::max(x, -87.0f);
  float xn = xc * INV_LN2;
  int n = (int)std::nearbyint(xn);
  float r = xc - (float)n * LN2;
  float p = 1.0f + r * (0.9999f + r * (0.4985f + r * 0.1681f));
  int nc = std::max(n, -126);
  float pow2n = bits2f((uint32_t)(nc + 127) << 23);
  return p * pow2n;
}

// simd_math/ops.mojo:127-141 tanh_f32
inline float tanh_f32(float x) {
  uint32_t sign = f2bits(x) & 0x80000000u;
  float ax = bits2f(f2bits(x) & 0x7FFFFFFFu);
  float e = exp_f32_fast(-2.0f * ax);
  float t = (1.0f - e) / (1.0f + e);
  return bits2f(f2bits(t) ^ sign);
}

// simd_math/ops.mojo:144-156 gelu_tanh_f32
inline float gelu_tanh_f32(float x) {
  const float s2pi = 0.7978845608028654f;
  const float a = 0.044715f;
  float x3 = x * x * x;
  float inner = s2pi * (x + a * x3);
  float t = tanh_f32(inner);
  return 0.5f * x * (1.0f + t);
}

// simd_math/exponential.mojo:177-194 fast_exp_softmax_biased
inline float fast_exp_softmax_biased(float x) {
  const float A_MAGIC = 12102203.16156148f;
  const float BIAS_F = 1059208216.0f;
  const float INV_TWO23 = 1.0f / (float)(1 << 23);
  const float QC_A = 1.6501418352127075f;
  const float QC_B = -0.37554836273193359f;
  const float QC_C = 0.38696467876434326f;
  int32_t i = (int32_t)(A_MAGIC * x + BIAS_F);
  uint32_t u = (uint32_t)i;
  float k = bits2f(u);
  uint32_t fb = u & 0x7FFFFFu;
  float f = (float)fb * INV_TWO23;
  return k * (QC_A + f * (QC_B + f * QC_C));
}

// butterquant/fwht.mojo:20-57: stages stride=1,2,4..; (a+b, a-b); then scale
// by f32(1 / f64(sqrt_f32(block))).
inline float fwht_scale(int block) {
  float s = std::sqrt((float)block);
  return (float)(1.0 / (double)s);
}
inline void fwht_block(float* v, int block) {
  for (int stride = 1; stride < block; stride <<= 1) {
    for (int i = 0; i < block; ++i) {
      if (i & stride) continue;
      float a = v[i], b = v[i + stride];
      v[i] = a + b;
      v[i + stride] = a - b;
    }
  }
  float sc = fwht_scale(block);
  for (int i = 0; i < block; ++i) v[i] = v[i] * sc;
}

// kernels/dot_products.mojo:144-159 with AVX-512 widths (W=16, BW=32):
// vdpbf16ps per f32 lane adds the odd pair product then the even one; the
// port-unrolled accumulators are summed in order then reduced as a tree.
float bf16_dot(const uint16_t* a, const uint16_t* b, int cols, int pu) {
  float acc[8][16];
  std::memset(acc, 0, sizeof(acc));
  const int stride = pu * 32;
  for (int i = 0; i < cols / stride; ++i)
    for (int p = 0; p < pu; ++p) {
      int off = i * stride + p * 32;
      for (int l = 0; l < 16; ++l) {
        float t = acc[p][l];
        t = t + bf2f(a[off + 2 * l + 1]) * bf2f(b[off + 2 * l + 1]);
        t = t + bf2f(a[off + 2 * l]) * bf2f(b[off + 2 * l]);
        acc[p][l] = t;
      }
    }
  float s[16] = {0};
  for (int p = 0; p < pu; ++p)
    for (int l = 0; l < 16; ++l) s[l] = s[l] + acc[p][l];
  for (int w = 8; w >= 1; w >>= 1)
    for (int l = 0; l < w; ++l) s[l] = s[l] + s[l + w];
  return s[0];
}

// kernels/dot_products.mojo:182-203 dot_to_scalar(f32 x, bf16 w): PU=8 banks of
// 16 lanes with fma, tree-merged (simd_math/matrixops.mojo:265-288).
float f32_bf16_dot(const float* x, const uint16_t* w, int cols) {
  float acc[8][16];
  std::memset(acc, 0, sizeof(acc));
  const int pu = 8, stride = pu * 16;
  for (int i = 0; i < cols / stride; ++i)
    for (int p = 0; p < pu; ++p)
      for (int l = 0; l < 16; ++l) {
        int off = i * stride + p * 16 + l;
        acc[p][l] = std::fmaf(x[off], bf2f(w[off]), acc[p][l]);
      }
  for (int st = 1; st < pu; st <<= 1)
    for (int i = 0; i < pu; i += 2 * st)
      for (int l = 0; l < 16; ++l) acc[i][l] = acc[i][l] + acc[i + st][l];
  float s[16];
  for (int l = 0; l < 16; ++l) s[l] = acc[0][l];
  for (int w = 8; w >= 1; w >>= 1)
    for (int l = 0; l < w; ++l) s[l] = s[l] + s[l + w];
  return s[0];
}

inline float sqrt_n() { return std::sqrt((float)H); }
inline float n_eps() { return (float)H * 1e-6f; }

// kernels/rmsnorm.mojo:16-17,45-46: inv_rms = sqrt(H)/sqrt(sum_sq + H*eps)
inline float inv_rms_row(const uint16_t* x) {
  float ss = bf16_dot(x, x, H, 8);
  return sqrt_n() / std::sqrt(ss + n_eps());
}

struct Cand { int32_t e; float l; };

// kernels/moe_router.mojo:44-57 insert_candidate
inline void insert_candidate(Cand* c, int32_t e, float l) {
  for (int k = 0; k < TOPK; ++k) {
    if (l > c[k].l || (l == c[k].l && e < c[k].e)) {
      for (int j = TOPK - 1; j > k; --j) c[j] = c[j - 1];
      c[k] = Cand{e, l};
      return;
    }
  }
}

}  // namespace

extern "C" {

struct OrcSparseRoute { int32_t token; float weight; };

int orc_dims(int* out) {
  out[0] = H; out[1] = E; out[2] = TOPK; out[3] = I; out[4] = GU; out[5] = DOWN_BLOCK;
  return 0;
}

float orc_fast_exp_softmax_biased(float x) { return fast_exp_softmax_biased(x); }
float orc_gelu_tanh(float x) { return gelu_tanh_f32(x); }
float orc_exp_f32_fast(float x) { return exp_f32_fast(x); }
uint16_t orc_f2bf(float x) { return f2bf(x); }

void orc_fwht_rows(float* v, long rows, int cols, int block) {
  for (long r = 0; r < rows; ++r)
    for (int b = 0; b < cols / block; ++b) fwht_block(v + r * cols + b * block, block);
}

// butterquant/kernels.mojo:37-45 bake_split_gain_in_place (model_init,
// modeling/gemma_4_moe_bq.mojo:909-915): g -> bf16(sign(g)*sqrt(max(|g|,1e-12)))
void orc_bake_split_gain(const uint16_t* g, uint16_t* out, int n) {
  for (int k = 0; k < n; ++k) {
    float v = bf2f(g[k]);
    float s = std::sqrt(std::max(std::fabs(v), 1e-12f));
    out[k] = f2bf(v < 0.0f ? -s : s);
  }
}

// modeling/gemma4_topology.mojo:362-388: router.scale *= 1/sqrt_f32(H), to bf16
void orc_bake_router_scale(const uint16_t* s, uint16_t* out, int n) {
  const float inv = 1.0f / std::sqrt((float)H);
  for (int k = 0; k < n; ++k) out[k] = f2bf(bf2f(s[k]) * inv);
}

// butterquant/kernels.mojo:171-224 router_center_softmax: W - mean over rows.
void orc_router_center(const uint16_t* w, int rows, int cols, uint16_t* centered) {
  std::vector<float> gauge(cols, 0.0f);
  for (int r = 0; r < rows; ++r)
    for (int k = 0; k < cols; ++k) gauge[k] = gauge[k] + bf2f(w[(long)r * cols + k]);
  const float inv_rows = 1.0f / (float)rows;
  for (int k = 0; k < cols; ++k) gauge[k] = gauge[k] * inv_rows;
  for (int r = 0; r < rows; ++r)
    for (int k = 0; k < cols; ++k)
      centered[(long)r * cols + k] = f2bf(bf2f(w[(long)r * cols + k]) - gauge[k]);
}

// quant/quantizer.mojo:963-1051 do_quant (PerRowQuant, SingleSided):
//   work = f32(W); if gamma: work *= sqrt|gamma| (quantizer.mojo:923-943,
//   butterquant/kernels.mojo:28-33); FWHT along K in `block` chunks
//   (kernels.mojo:81-85); per-row absmax quant, scale = amax/127
//   (kernels.mojo:58-78,105-107).  Output int8 row-major [rows][cols].
void orc_quantize_rows(const uint16_t* w, long rows, int cols, const uint16_t* gamma,
                       int block, int8_t* q, float* scale) {
  std::vector<float> g;
  if (gamma) {
    g.resize(cols);
    for (int k = 0; k < cols; ++k) g[k] = std::sqrt(std::fabs(bf2f(gamma[k])));
  }
#pragma omp parallel
  {
    std::vector<float> work(cols);
#pragma omp for schedule(static)
    for (long r = 0; r < rows; ++r) {
      const uint16_t* src = w + r * cols;
      for (int k = 0; k < cols; ++k) work[k] = bf2f(src[k]);
      if (gamma)
        for (int k = 0; k < cols; ++k) work[k] = work[k] * g[k];
      for (int b = 0; b < cols / block; ++b) fwht_block(work.data() + b * block, block);
      float amax = 0.0f;
      for (int k = 0; k < cols; ++k) amax = std::max(amax, std::fabs(work[k]));
      scale[r] = amax / 127.0f;
      float inv = amax > 0.0f ? 127.0f / amax : 0.0f;
      for (int k = 0; k < cols; ++k) q[r * cols + k] = quantize_i8(work[k], inv);
    }
  }
}

// butterquant/vnni.mojo:31-83 pack: per 32-row N-tile t and 64-col K-step ks,
// a 2048-byte tile at t*32*cols + ks*2048; two 16-row halves of 1024 B; within
// a half byte (k/4)*64 + n*4 + k%4.
void orc_vnni_pack(const int8_t* q, long rows, int cols, int8_t* packed) {
#pragma omp parallel for schedule(static)
  for (long r = 0; r < rows; ++r) {
    long t = r / 32;
    int n = (int)(r % 32);
    int half = n / 16, nn = n % 16;
    for (int k = 0; k < cols; ++k) {
      int ks = k / 64, kk = k % 64;
      long off = t * 32L * cols + (long)ks * 2048 + half * 1024 + (kk / 4) * 64 + nn * 4 + (kk % 4);
      packed[off] = q[r * cols + k];
    }
  }
}

void orc_vnni_unpack(const int8_t* packed, long rows, int cols, int8_t* q) {
#pragma omp parallel for schedule(static)
  for (long r = 0; r < rows; ++r) {
    long t = r / 32;
    int n = (int)(r % 32);
    int half = n / 16, nn = n % 16;
    for (int k = 0; k < cols; ++k) {
      int ks = k / 64, kk = k % 64;
      long off = t * 32L * cols + (long)ks * 2048 + half * 1024 + (kk / 4) * 64 + nn * 4 + (kk % 4);
      q[r * cols + k] = packed[off];
    }
  }
}

// butterquant/vnni.mojo:272-288 colsum: per row and per block_cols block of
// int8 sums as f32; row-major [rows][nb] or block-major [nb][rows].
void orc_colsum(const int8_t* q, long rows, int cols, int block_cols, float* cs, int row_major) {
  int nb = cols / block_cols;
#pragma omp parallel for schedule(static)
  for (long r = 0; r < rows; ++r)
    for (int b = 0; b < nb; ++b) {
      int32_t s = 0;
      for (int k = 0; k < block_cols; ++k) s += q[r * cols + b * block_cols + k];
      if (row_major) cs[r * nb + b] = (float)s; else cs[(long)b * rows + r] = (float)s;
    }
}

// kernels/moe_router.mojo:164-191 (RouterExpertKernel) + :259-293
// (RouterMergeKernel).  Per-worker top-8 lists merged with insert_candidate
// give the same list as inserting all E logits in ascending expert order.
// logits_out (optional) receives the [T][E] f32 logits.
void orc_router(const uint16_t* x, int T, const uint16_t* wr, const uint16_t* rscale,
                const uint16_t* pes, int32_t* route_idx, float* route_w, float* logits_out) {
#pragma omp parallel
  {
    std::vector<float> s(H);
    std::vector<float> lg(E);
#pragma omp for schedule(static)
    for (int t = 0; t < T; ++t) {
      const uint16_t* xr = x + (long)t * H;
      float inv = inv_rms_row(xr);
      for (int k = 0; k < H; ++k) s[k] = bf2f(xr[k]) * bf2f(rscale[k]) * inv;
      Cand c[TOPK];
      for (int k = 0; k < TOPK; ++k) c[k] = Cand{0, -1.0e30f};
      for (int e = 0; e < E; ++e) {
        lg[e] = f32_bf16_dot(s.data(), wr + (long)e * H, H);
        insert_candidate(c, e, lg[e]);
      }
      if (logits_out) std::memcpy(logits_out + (long)t * E, lg.data(), E * sizeof(float));
      float maxl = c[0].l;
      float ev[TOPK];
      float sum = 0.0f;
      for (int k = 0; k < TOPK; ++k) { ev[k] = fast_exp_softmax_biased(c[k].l - maxl); sum = sum + ev[k]; }
      float inv_sum = 1.0f / sum;
      for (int k = 0; k < TOPK; ++k) {
        route_idx[t * TOPK + k] = c[k].e;
        route_w[t * TOPK + k] = ev[k] * inv_sum * bf2f(pes[c[k].e]);
      }
    }
  }
}

// kernels/moe_router.mojo:72-101 BuildScheduleKernel: histogram over the
// local expert range, exclusive prefix, stable (token-major, then k) permute.
void orc_build_schedules(const int32_t* route_idx, const float* route_w, int T, int expert_base,
                         int epr, int32_t* expert_offset, OrcSparseRoute* routes) {
  std::vector<int32_t> counts(epr, 0), wo(epr);
  for (int t = 0; t < T; ++t)
    for (int k = 0; k < TOPK; ++k) {
      int e = route_idx[t * TOPK + k];
      if (e >= expert_base && e < expert_base + epr) counts[e - expert_base]++;
    }
  int32_t run = 0;
  for (int e = 0; e < epr; ++e) { expert_offset[e] = run; wo[e] = run; run += counts[e]; }
  expert_offset[epr] = run;
  for (int t = 0; t < T; ++t)
    for (int k = 0; k < TOPK; ++k) {
      int slot = t * TOPK + k;
      int e = route_idx[slot];
      if (e >= expert_base && e < expert_base + epr) {
        int pos = wo[e - expert_base]++;
        routes[pos].token = t;
        routes[pos].weight = route_w[slot];
      }
    }
}

// ---------------------------------------------------------------- bf16 path
// kernels/rmsnorm.mojo:21-47 rms_norm_row (scaled): bf16(x*inv_rms*gamma)
void orc_rms_norm(const uint16_t* x, const uint16_t* gamma, int T, uint16_t* out) {
#pragma omp parallel for schedule(static)
  for (int t = 0; t < T; ++t) {
    const uint16_t* xr = x + (long)t * H;
    float inv = inv_rms_row(xr);
    for (int k = 0; k < H; ++k) out[(long)t * H + k] = f2bf(bf2f(xr[k]) * inv * bf2f(gamma[k]));
  }
}

// kernels/rmsnorm.mojo:48-64 norm_residual_add_row, the decoder layer's step
// after the attention block (modeling/gemma_4_moe_bq.mojo:1098-1102):
// out = bf16(r + (s*inv_rms(s))*w).  out may alias r.
void orc_norm_residual_add(const uint16_t* src, const uint16_t* r, const uint16_t* w, int T, uint16_t* out) {
#pragma omp parallel for schedule(static)
  for (int t = 0; t < T; ++t) {
    const uint16_t* s = src + (long)t * H;
    const float inv = inv_rms_row(s);
    for (int k = 0; k < H; ++k)
      out[(long)t * H + k] = f2bf(bf2f(r[(long)t * H + k]) + bf2f(s[k]) * inv * bf2f(w[k]));
  }
}

// The tail of dispatch_bq_ffn after the MoE (modeling/gemma_4_moe_bq.mojo:
// 785-805), per token:
//   dense = rms_norm(dense, post_ffn_norm_1)                 (kernels/rmsnorm.mojo:21-47)
//   dense = norm_residual_add(src=moe, residual=dense, w=post_ffn_norm_2)
//   x     = norm_residual_add(src=dense, residual=x,  w=post_ffn_norm)
//   x     = x * layer_scalar                              (kernels/elementwise.mojo:75-83)
// norm_residual_add_row (kernels/rmsnorm.mojo:51-67): bf16(r + (s*inv_rms(s))*w).
void orc_post_moe(const uint16_t* moe, const uint16_t* dense, const uint16_t* x_main,
                  const uint16_t* w1, const uint16_t* w2, const uint16_t* w, float layer_scalar,
                  int T, uint16_t* out) {
#pragma omp parallel for schedule(static)
  for (int t = 0; t < T; ++t) {
    const uint16_t* m = moe + (long)t * H;
    const uint16_t* d = dense + (long)t * H;
    const uint16_t* x = x_main + (long)t * H;
    std::vector<uint16_t> d1(H), d2(H), xm(H);
    const float inv_d = inv_rms_row(d);
    for (int k = 0; k < H; ++k) d1[k] = f2bf(bf2f(d[k]) * inv_d * bf2f(w1[k]));
    const float inv_m = inv_rms_row(m);
    for (int k = 0; k < H; ++k) d2[k] = f2bf(bf2f(d1[k]) + bf2f(m[k]) * inv_m * bf2f(w2[k]));
    const float inv_2 = inv_rms_row(d2.data());
    for (int k = 0; k < H; ++k) xm[k] = f2bf(bf2f(x[k]) + bf2f(d2[k]) * inv_2 * bf2f(w[k]));
    for (int k = 0; k < H; ++k) out[(long)t * H + k] = f2bf(bf2f(xm[k]) * layer_scalar);
  }
}

// kernels/moe_experts.mojo:16-54,82-154 Phase1GateUpKernel: per routed record
// g = x.Wgu[e][j], u = x.Wgu[e][I+j] (bf16 dots, PU=4), bucket = bf16(gelu(g)*u)
void orc_phase1_bf16(const uint16_t* x_normed, const int32_t* expert_offset,
                     const OrcSparseRoute* routes, const uint16_t* w_gu, int epr,
                     uint16_t* bucket) {
  int nrec = expert_offset[epr];
#pragma omp parallel for schedule(dynamic, 4)
  for (int r = 0; r < nrec; ++r) {
    int e = 0;
    while (expert_offset[e + 1] <= r) ++e;
    const uint16_t* xr = x_normed + (long)routes[r].token * H;
    const uint16_t* we = w_gu + (long)e * GU * H;
    for (int j = 0; j < I; ++j) {
      float g = bf16_dot(we + (long)j * H, xr, H, 4);
      float u = bf16_dot(we + (long)(I + j) * H, xr, H, 4);
      bucket[(long)r * I + j] = f2bf(gelu_tanh_f32(g) * u);
    }
  }
}

// kernels/moe_experts.mojo:201-319 Phase2DownKernel: acc[tok] = 0; for e
// ascending, for each record acc[tok][m] += (bucket.Wd[e][m]) * w; out = bf16(acc)
void orc_phase2_bf16(const int32_t* expert_offset, const OrcSparseRoute* routes,
                     const uint16_t* bucket, const uint16_t* w_dn, int epr, int T,
                     uint16_t* out) {
  std::vector<float> acc((size_t)T * H, 0.0f);
#pragma omp parallel for schedule(static)
  for (int m = 0; m < H; ++m) {
    for (int e = 0; e < epr; ++e) {
      const uint16_t* wrow = w_dn + ((long)e * H + m) * I;
      for (int r = expert_offset[e]; r < expert_offset[e + 1]; ++r) {
        float v = bf16_dot(wrow, bucket + (long)r * I, I, 2);
        float* a = &acc[(size_t)routes[r].token * H + m];
        *a = *a + v * routes[r].weight;
      }
    }
  }
  for (size_t i = 0; i < (size_t)T * H; ++i) out[i] = f2bf(acc[i]);
}

// ---------------------------------------------------------- butterquant path
// butterquant/runtime.mojo:11-37 prepare_norm_activation[per_block=False,
// block=128]: v = x*inv_rms*gamma'; FWHT-128 blocks; per-row absmax int8,
// sa = raw amax (quantize.mojo:5-9, kernels.mojo:69-78 store_divided=False).
void orc_bq_norm_quant(const uint16_t* x, const uint16_t* gamma, int T, int8_t* xi8, float* sa) {
#pragma omp parallel
  {
    std::vector<float> v(H);
#pragma omp for schedule(static)
    for (int t = 0; t < T; ++t) {
      const uint16_t* xr = x + (long)t * H;
      float inv = inv_rms_row(xr);
      for (int k = 0; k < H; ++k) v[k] = bf2f(xr[k]) * inv * bf2f(gamma[k]);
      for (int b = 0; b < H / 128; ++b) fwht_block(v.data() + b * 128, 128);
      float amax = 0.0f;
      for (int k = 0; k < H; ++k) amax = std::max(amax, std::fabs(v[k]));
      sa[t] = amax;
      float qi = amax > 0.0f ? 127.0f / amax : 0.0f;
      for (int k = 0; k < H; ++k) xi8[(long)t * H + k] = quantize_i8(v[k], qi);
    }
  }
}

// butterquant_kernels/moe.mojo:26-74,100-124 BqPhase1GateUpKernel with
// butterquant/gemm.mojo:36-75 (u8 x s8 vpdpbusd accumulation) and
// dot_products.mojo:70-73 (f32(iacc) - 128*colsum).
// w_gu: row-major int8 [epr*GU][H] (the VNNI pack is a pure permutation).
void orc_bq_phase1(const int8_t* xi8, const float* xsa, const int32_t* expert_offset,
                   const OrcSparseRoute* routes, const int8_t* w_gu, const float* gu_scale,
                   const float* gu_cs, int epr, uint16_t* bucket) {
  const float inv127 = 1.0f / 127.0f;
  int nrec = expert_offset[epr];
#pragma omp parallel for schedule(dynamic, 2)
  for (int r = 0; r < nrec; ++r) {
    int e = 0;
    while (expert_offset[e + 1] <= r) ++e;
    int tok = routes[r].token;
    const uint8_t* xr = reinterpret_cast<const uint8_t*>(xi8 + (long)tok * H);
    float ad = xsa[tok] * inv127;
    const int8_t* we = w_gu + (long)e * GU * H;
    const float* ws = gu_scale + (long)e * GU;
    const float* cs = gu_cs + (long)e * GU;
    for (int j = 0; j < I; ++j) {
      int32_t ig = 0, iu = 0;
      const int8_t* wg = we + (long)j * H;
      const int8_t* wu = we + (long)(I + j) * H;
      for (int k = 0; k < H; ++k) {
        int32_t a = (int32_t)(uint8_t)(xr[k] ^ 0x80u);
        ig += a * (int32_t)wg[k];
        iu += a * (int32_t)wu[k];
      }
      float gv = ((float)ig - 128.0f * cs[j]) * ad * ws[j];
      float uv = ((float)iu - 128.0f * cs[I + j]) * ad * ws[I + j];
      bucket[(long)r * I + j] = f2bf(gelu_tanh_f32(gv) * uv);
    }
  }
}

// butterquant/runtime.mojo:62-79 prepare_block_activation[64, fwht=True]:
// f32(bucket) -> FWHT-64 per block -> per-block absmax int8, sa raw amax.
void orc_bq_block_quant(const uint16_t* bucket, long R, int cols, int block, int8_t* qi8, float* sa) {
  int nb = cols / block;
#pragma omp parallel
  {
    std::vector<float> v(cols);
#pragma omp for schedule(static)
    for (long r = 0; r < R; ++r) {
      for (int k = 0; k < cols; ++k) v[k] = bf2f(bucket[r * cols + k]);
      for (int b = 0; b < nb; ++b) {
        float* vb = v.data() + b * block;
        fwht_block(vb, block);
        float amax = 0.0f;
        for (int k = 0; k < block; ++k) amax = std::max(amax, std::fabs(vb[k]));
        sa[r * nb + b] = amax;
        float inv = amax > 0.0f ? 127.0f / amax : 0.0f;
        for (int k = 0; k < block; ++k) qi8[r * cols + b * block + k] = quantize_i8(vb[k], inv);
      }
    }
  }
}

// prepare_block_activation[block, apply_fwht] (butterquant/runtime.mojo:62-79)
// with the FWHT optional: the attention output is quantised per head (block =
// head_dim) without one (modeling/gemma_4_moe_bq.mojo:516-518).
void orc_bq_block_quant_ex(const uint16_t* src, long R, int cols, int block, int apply_fwht, int8_t* qi8,
                           float* sa) {
  int nb = cols / block;
#pragma omp parallel
  {
    std::vector<float> v(cols);
#pragma omp for schedule(static)
    for (long r = 0; r < R; ++r) {
      for (int k = 0; k < cols; ++k) v[k] = bf2f(src[r * cols + k]);
      for (int b = 0; b < nb; ++b) {
        float* vb = v.data() + b * block;
        if (apply_fwht) fwht_block(vb, block);
        float amax = 0.0f;
        for (int k = 0; k < block; ++k) amax = std::max(amax, std::fabs(vb[k]));
        sa[r * nb + b] = amax;
        float inv = amax > 0.0f ? 127.0f / amax : 0.0f;
        for (int k = 0; k < block; ++k) qi8[r * cols + b * block + k] = quantize_i8(vb[k], inv);
      }
    }
  }
}

// gemm_i8_per_block_panel (butterquant/gemm.mojo:174-216) for any block: the
// attention output projection uses block = head_dim.  cs block-major
// [k/block][n_rows].
void orc_bq_block_linear_ex(const int8_t* hi8, const float* hsa, int T, int k, int block, const int8_t* w,
                            const float* ws, const float* cs, int n_rows, uint16_t* out) {
  const float inv127 = 1.0f / 127.0f;
  const int nb = k / block;
#pragma omp parallel for schedule(static)
  for (int t = 0; t < T; ++t) {
    const uint8_t* ar = reinterpret_cast<const uint8_t*>(hi8 + (long)t * k);
    for (int n = 0; n < n_rows; ++n) {
      const int8_t* wr = w + (long)n * k;
      float facc = 0.0f;
      for (int b = 0; b < nb; ++b) {
        int32_t ia = 0;
        for (int j = b * block; j < (b + 1) * block; ++j)
          ia += (int32_t)(uint8_t)(ar[j] ^ 0x80u) * (int32_t)wr[j];
        const float corr = (float)ia - 128.0f * cs[(long)b * n_rows + n];
        facc = std::fmaf(corr, hsa[(long)t * nb + b] * inv127, facc);
      }
      out[(long)t * n_rows + n] = f2bf(facc * ws[n]);
    }
  }
}

// butterquant_kernels/moe.mojo:168-295 BqPhase2DownKernel: for each record,
// facc = fma(f32(iacc_b) - 128*cs[b][n], sa[r][b]/127, facc) over the 11 K
// blocks; acc[tok][n] += facc*sw[n]*w (experts ascending); out = bf16(acc).
// w_dn row-major int8 [epr*H][I]; dn_cs block-major [NB][cs_stride] indexed at
// b*cs_stride + e*H + n (cs_stride = epr*H for a rank-local array).
void orc_bq_phase2(const int8_t* bi8, const float* bsa, const int32_t* expert_offset,
                   const OrcSparseRoute* routes, const int8_t* w_dn, const float* dn_scale,
                   const float* dn_cs, long cs_stride, int epr, int T, uint16_t* out) {
  const float inv127 = 1.0f / 127.0f;
  std::vector<float> acc((size_t)T * H, 0.0f);
#pragma omp parallel for schedule(static)
  for (int n = 0; n < H; ++n) {
    for (int e = 0; e < epr; ++e) {
      const int8_t* wrow = w_dn + ((long)e * H + n) * I;
      float sw = dn_scale[(long)e * H + n];
      for (int r = expert_offset[e]; r < expert_offset[e + 1]; ++r) {
        const uint8_t* ar = reinterpret_cast<const uint8_t*>(bi8 + (long)r * I);
        float facc = 0.0f;
        for (int b = 0; b < NB_DOWN; ++b) {
          int32_t ia = 0;
          for (int k = b * DOWN_BLOCK; k < (b + 1) * DOWN_BLOCK; ++k)
            ia += (int32_t)(uint8_t)(ar[k] ^ 0x80u) * (int32_t)wrow[k];
          float corr = (float)ia - 128.0f * dn_cs[(long)b * cs_stride + (long)e * H + n];
          float adv = bsa[(long)r * NB_DOWN + b] * inv127;
          facc = std::fmaf(corr, adv, facc);
        }
        float res = facc * sw * routes[r].weight;
        float* a = &acc[(size_t)routes[r].token * H + n];
        *a = *a + res;
      }
    }
  }
  for (size_t i = 0; i < (size_t)T * H; ++i) out[i] = f2bf(acc[i]);
}

// ------------------------------------------------------------ dense MLP
// butterquant/gemm.mojo:115-143 gemm_i8_per_row_panel (u8 x s8 vpdpbusd,
// dot_products.mojo:70-73 correction), stored as bf16 (convert.mojo:8-28):
// out[t][n] = bf16((f32(iacc) - 128*cs[n]) * (sa[t]*(1/127)) * ws[n]).
// w row-major int8 [n_rows][k] (the VNNI pack is a pure permutation).
void orc_bq_linear(const int8_t* xi8, const float* xsa, int T, const int8_t* w, const float* ws,
                   const float* cs, int n_rows, int k, uint16_t* out) {
  const float inv127 = 1.0f / 127.0f;
#pragma omp parallel for schedule(static)
  for (int t = 0; t < T; ++t) {
    const uint8_t* xr = reinterpret_cast<const uint8_t*>(xi8 + (long)t * k);
    const float ad = xsa[t] * inv127;
    for (int n = 0; n < n_rows; ++n) {
      const int8_t* wr = w + (long)n * k;
      int32_t ia = 0;
      for (int j = 0; j < k; ++j) ia += (int32_t)(uint8_t)(xr[j] ^ 0x80u) * (int32_t)wr[j];
      const float corr = (float)ia - 128.0f * cs[n];
      out[(long)t * n_rows + n] = f2bf(corr * ad * ws[n]);
    }
  }
}

// kernels/elementwise.mojo:17-24 gelu_gate_up_row: bf16(gelu_tanh(g) * u).
void orc_gelu_gate_up(const uint16_t* gate, const uint16_t* up, long n, uint16_t* out) {
  for (long i = 0; i < n; ++i) out[i] = f2bf(gelu_tanh_f32(bf2f(gate[i])) * bf2f(up[i]));
}

// butterquant/gemm.mojo:174-216 gemm_i8_per_block_panel: per output row n,
// facc = fma(f32(iacc_b) - 128*cs[b][n], sa[t][b]*(1/127), facc) over the k/64
// blocks in order, out = bf16(facc * ws[n]).  cs block-major [nb][n_rows].
void orc_bq_block_linear(const int8_t* hi8, const float* hsa, int T, int k, const int8_t* w,
                         const float* ws, const float* cs, int n_rows, uint16_t* out) {
  const float inv127 = 1.0f / 127.0f;
  const int nb = k / DOWN_BLOCK;
#pragma omp parallel for schedule(static)
  for (int t = 0; t < T; ++t) {
    const uint8_t* ar = reinterpret_cast<const uint8_t*>(hi8 + (long)t * k);
    for (int n = 0; n < n_rows; ++n) {
      const int8_t* wr = w + (long)n * k;
      float facc = 0.0f;
      for (int b = 0; b < nb; ++b) {
        int32_t ia = 0;
        for (int j = b * DOWN_BLOCK; j < (b + 1) * DOWN_BLOCK; ++j)
          ia += (int32_t)(uint8_t)(ar[j] ^ 0x80u) * (int32_t)wr[j];
        const float corr = (float)ia - 128.0f * cs[(long)b * n_rows + n];
        facc = std::fmaf(corr, hsa[(long)t * nb + b] * inv127, facc);
      }
      out[(long)t * n_rows + n] = f2bf(facc * ws[n]);
    }
  }
}

// modeling/gemma_4_moe_bq.mojo:749-783 the dense half of dispatch_bq_ffn:
// norm+quant (pre_feedforward_layernorm, split-gain baked), gate and up
// bq_linear, GeGLU, FWHT-64 block quant of h, bq_block_linear with down.
// h_bf16/h_i8/h_sa (optional) receive the intermediates.
void orc_dense_mlp(const uint16_t* x, int T, const uint16_t* gamma, int inter,
                   const int8_t* wg, const float* wgs, const float* wgcs,
                   const int8_t* wu, const float* wus, const float* wucs,
                   const int8_t* wd, const float* wds, const float* wdcs, uint16_t* out,
                   uint16_t* h_bf16, int8_t* h_i8, float* h_sa) {
  std::vector<int8_t> xi8((size_t)T * H);
  std::vector<float> xsa(T);
  orc_bq_norm_quant(x, gamma, T, xi8.data(), xsa.data());
  std::vector<uint16_t> g((size_t)T * inter), u((size_t)T * inter), hh((size_t)T * inter);
  orc_bq_linear(xi8.data(), xsa.data(), T, wg, wgs, wgcs, inter, H, g.data());
  orc_bq_linear(xi8.data(), xsa.data(), T, wu, wus, wucs, inter, H, u.data());
  orc_gelu_gate_up(g.data(), u.data(), (long)T * inter, hh.data());
  const int nb = inter / DOWN_BLOCK;
  std::vector<int8_t> qi((size_t)T * inter);
  std::vector<float> qs((size_t)T * nb);
  orc_bq_block_quant(hh.data(), T, inter, DOWN_BLOCK, qi.data(), qs.data());
  orc_bq_block_linear(qi.data(), qs.data(), T, inter, wd, wds, wdcs, H, out);
  if (h_bf16) std::memcpy(h_bf16, hh.data(), hh.size() * 2);
  if (h_i8) std::memcpy(h_i8, qi.data(), qi.size());
  if (h_sa) std::memcpy(h_sa, qs.data(), qs.size() * 4);
}

// ------------------------------------------------------------ bq attention
// The reference's SIMD width on its AVX-512 hosts (W = 16 f32 lanes) fixes
// the order of its per-head reductions; the restatement keeps it: element e
// lives in lane e % 16 of register e / 16.
constexpr int ATT_W = 16;

// SIMD.reduce_add / reduce_max of 16 lanes: halving tree v[i] op v[i + w/2].
inline float lane_tree_sum(float* v) {
  for (int w = ATT_W / 2; w >= 1; w >>= 1)
    for (int i = 0; i < w; ++i) v[i] = v[i] + v[i + w];
  return v[0];
}

// butterquant/head_prep.mojo:9-37 head_inv_rms (sqrt_n = sqrt_f32(head_dim),
// n_eps = f32(head_dim) * f32(1e-6)) and absmax_quantize_head.
inline float head_inv_rms(const float* r, int head_dim) {
  float lanes[ATT_W];
  const int regs = head_dim / ATT_W;
  for (int l = 0; l < ATT_W; ++l) {
    float s = r[l] * r[l];
    for (int ri = 1; ri < regs; ++ri) s = std::fmaf(r[ri * ATT_W + l], r[ri * ATT_W + l], s);
    lanes[l] = s;
  }
  const float sqrt_n = std::sqrt((float)head_dim);
  const float n_eps = (float)head_dim * 1e-6f;
  return sqrt_n / std::sqrt(lane_tree_sum(lanes) + n_eps);
}

inline float absmax_quantize_head(const float* r, int head_dim, int8_t* q, int32_t* qsum) {
  float amax = 0.0f;
  for (int e = 0; e < head_dim; ++e) amax = std::max(amax, std::fabs(r[e]));
  if (amax < 1e-10f) amax = 1e-10f;
  const float inv = 127.0f / amax;
  int32_t s = 0;
  for (int e = 0; e < head_dim; ++e) {
    q[e] = quantize_i8(r[e], inv);
    s += q[e];
  }
  if (qsum) *qsum = s;
  return amax;
}

// butterquant/head_prep.mojo:40-75 prep_head_qk_i8 (gamma != NULL, rope over
// rope_half lanes pairing e with e + pair_stride) and :78-97 prep_head_v_i8
// (gamma == NULL: no gain, no rope): RMSNorm, RoPE, FWHT over the head, int8.
float orc_prep_head(const uint16_t* src, const uint16_t* gamma, const float* cos, const float* sin,
                    int head_dim, int rope_half, int pair_stride, int8_t* q_out, int32_t* qsum) {
  std::vector<float> r(head_dim);
  for (int e = 0; e < head_dim; ++e) r[e] = bf2f(src[e]);
  const float inv = head_inv_rms(r.data(), head_dim);
  for (int e = 0; e < head_dim; ++e) r[e] = gamma ? (r[e] * inv) * bf2f(gamma[e]) : r[e] * inv;
  if (gamma) {
    for (int e = 0; e < rope_half; ++e) {
      const float lo = r[e], hi = r[pair_stride + e];
      r[e] = lo * cos[e] - hi * sin[e];
      r[pair_stride + e] = hi * cos[e] + lo * sin[e];
    }
  }
  fwht_block(r.data(), head_dim);
  return absmax_quantize_head(r.data(), head_dim, q_out, qsum);
}

// butterquant_kernels/attention.mojo:474-560 BqAttnPrepKernel for tokens at
// positions pos[t]: q heads -> q_i8, qi_bias = 128*sum(q), f_q = amax; k and
// v heads into cache row slot[t] (skipped when slot[t] < 0).  v_src may equal
// k_src (the full layers' shared K/V projection).
void orc_bq_attn_prep(const uint16_t* q_src, const uint16_t* k_src, const uint16_t* v_src,
                      const uint16_t* q_norm, const uint16_t* k_norm, int T, const int32_t* pos,
                      const int32_t* slot, int head_dim, int num_q, int num_kv, int rope_half,
                      int pair_stride, const float* cos_table, const float* sin_table, int8_t* q_i8,
                      float* qi_bias, float* f_q, int8_t* k_cache, float* k_scale, int8_t* v_cache,
                      float* v_scale) {
  const long qs = (long)num_q * head_dim, kvs = (long)num_kv * head_dim;
#pragma omp parallel for schedule(static)
  for (int t = 0; t < T; ++t) {
    const float* c = cos_table + (long)pos[t] * rope_half;
    const float* sn = sin_table + (long)pos[t] * rope_half;
    for (int h = 0; h < num_q; ++h) {
      int32_t qsum = 0;
      f_q[(long)t * num_q + h] = orc_prep_head(q_src + t * qs + (long)h * head_dim, q_norm, c, sn,
                                               head_dim, rope_half, pair_stride,
                                               q_i8 + t * qs + (long)h * head_dim, &qsum);
      qi_bias[(long)t * num_q + h] = (float)qsum * 128.0f;
    }
    if (slot[t] < 0) continue;
    const long row = slot[t];
    for (int h = 0; h < num_kv; ++h) {
      k_scale[row * num_kv + h] = orc_prep_head(k_src + t * kvs + (long)h * head_dim, k_norm, c, sn,
                                                head_dim, rope_half, pair_stride,
                                                k_cache + row * kvs + (long)h * head_dim, nullptr);
      v_scale[row * num_kv + h] = orc_prep_head(v_src + t * kvs + (long)h * head_dim, nullptr, c, sn,
                                                head_dim, 0, 0, v_cache + row * kvs + (long)h * head_dim,
                                                nullptr);
    }
  }
}

// Flash decode over int8 K/V (butterquant_kernels/attention.mojo:33-146
// bq_process_kv_tile + BqFlashAttentionKernel, kernels/attention_ops.mojo:
// 196-212 online_softmax_tile with TILE = 16), the KV range of each token
// split into n_splits worker ranges (kernels/helpers.mojo:182-190
// worker_range), then kernels/logsum_merge.mojo:29-117 merge_segments /
// write_finalized_head.  slots: per token, kv_len[t] cache rows in position
// order (row-major [T][max_kv]).  out bf16 [T][num_q*head_dim].
void orc_bq_flash_decode(const int8_t* q_i8, const float* qi_bias, const float* f_q,
                         const int8_t* k_cache, const float* k_scale, const int8_t* v_cache,
                         const float* v_scale, int T, const int32_t* slots, const int32_t* kv_len,
                         int max_kv, int head_dim, int num_q, int num_kv, int n_splits, uint16_t* out) {
  const float inv127 = 1.0f / 127.0f;
  const float inv127sq = inv127 * inv127;
  const int gqa = num_q / num_kv;
  const long kvs = (long)num_kv * head_dim;
#pragma omp parallel for collapse(2) schedule(dynamic, 1)
  for (int t = 0; t < T; ++t) {
    for (int h = 0; h < num_q; ++h) {
      const int g = h / gqa;
      const int8_t* q = q_i8 + ((long)t * num_q + h) * head_dim;
      const float qb = qi_bias[(long)t * num_q + h], fq = f_q[(long)t * num_q + h];
      const int32_t* sl = slots + (long)t * max_kv;
      std::vector<float> pm(n_splits), pl(n_splits), pacc((size_t)n_splits * head_dim);
      for (int s = 0; s < n_splits; ++s) {
        const int per = (kv_len[t] + n_splits - 1) / n_splits;
        int b = s * per, e = std::min(b + per, kv_len[t]);
        if (b >= kv_len[t]) b = e = kv_len[t];
        float m = -1e30f, l = 0.0f;
        float* acc = pacc.data() + (size_t)s * head_dim;
        for (int i = 0; i < head_dim; ++i) acc[i] = 0.0f;
        for (int p = b; p < e; p += ATT_W) {
          const int tl = std::min(ATT_W, e - p);
          float sc[ATT_W];
          for (int j = 0; j < ATT_W; ++j) sc[j] = -1e30f;
          for (int j = 0; j < tl; ++j) {
            const long row = sl[p + j];
            const int8_t* k = k_cache + row * kvs + (long)g * head_dim;
            int32_t r = 0;  // u8(k ^ 0x80) x s8(q): the shifted VNNI dot
            for (int i = 0; i < head_dim; ++i) r += (int32_t)(uint8_t)(k[i] ^ 0x80u) * (int32_t)q[i];
            const float ks = k_scale[row * num_kv + g];
            sc[j] = ((((float)r - qb) * fq) * ks) * inv127sq;
          }
          float tmax = sc[0];
          for (int j = 1; j < ATT_W; ++j) tmax = std::max(tmax, sc[j]);
          const float m_new = tmax > m ? tmax : m;
          const float corr = fast_exp_softmax_biased(std::max(-87.0f, m - m_new));
          float w[ATT_W], wsum[ATT_W];
          for (int j = 0; j < ATT_W; ++j) {
            w[j] = fast_exp_softmax_biased(std::max(-87.0f, sc[j] - m_new));
            wsum[j] = w[j];
          }
          for (int i = 0; i < head_dim; ++i) acc[i] = acc[i] * corr;
          l = l * corr + lane_tree_sum(wsum);
          m = m_new;
          for (int j = 0; j < tl; ++j) {
            const long row = sl[p + j];
            const int8_t* v = v_cache + row * kvs + (long)g * head_dim;
            const float wv = (w[j] * v_scale[row * num_kv + g]) * inv127;
            for (int i = 0; i < head_dim; ++i) acc[i] = std::fmaf((float)v[i], wv, acc[i]);
          }
        }
        pm[s] = m;
        pl[s] = l;
      }
      // merge (batches of 16 partials)
      float gm = -1e30f;
      for (int s = 0; s < n_splits; ++s) gm = pm[s] > gm ? pm[s] : gm;
      float gl = 0.0f;
      bool first = true;
      std::vector<float> acc(head_dim, 0.0f);
      for (int b0 = 0; b0 < n_splits; b0 += ATT_W) {
        const int bl = std::min(ATT_W, n_splits - b0);
        float c[ATT_W], lc[ATT_W];
        for (int j = 0; j < ATT_W; ++j) {
          const float d = j < bl ? pm[b0 + j] - gm : -1e30f;
          const float ls = j < bl ? pl[b0 + j] : 0.0f;
          c[j] = fast_exp_softmax_biased(std::max(-87.0f, d));
          if (!(ls > 0.0f)) c[j] = 0.0f;
          lc[j] = ls * c[j];
        }
        gl += lane_tree_sum(lc);
        for (int j = 0; j < bl; ++j) {
          if (c[j] <= 0.0f) continue;
          const float* src = pacc.data() + (size_t)(b0 + j) * head_dim;
          for (int i = 0; i < head_dim; ++i) acc[i] = first ? src[i] * c[j] : std::fmaf(src[i], c[j], acc[i]);
          first = false;
        }
      }
      uint16_t* o = out + ((long)t * num_q + h) * head_dim;
      if (!(gl > 0.0f)) {
        for (int i = 0; i < head_dim; ++i) o[i] = 0;
      } else {
        const float il = 1.0f / gl;
        for (int i = 0; i < head_dim; ++i) o[i] = f2bf(acc[i] * il);
      }
    }
  }
}

// ------------------------------------------------------------ whole block
struct OrcBqLayer {
  const uint16_t* router_centered;  // [E][H] bf16 (router_center_softmax)
  const uint16_t* router_scale;     // [H] bf16, baked * 1/sqrt(H)
  const uint16_t* pes;              // [E] bf16 per_expert_scale
  const uint16_t* gamma2;           // [H] bf16, split-gain baked
  const int8_t* gu_q;               // [E*GU][H] int8 row-major
  const float* gu_scale;            // [E*GU]
  const float* gu_cs;               // [E*GU]
  const int8_t* dn_q;               // [E*H][I] int8 row-major
  const float* dn_scale;            // [E*H]
  const float* dn_cs;               // [NB][E*H] block-major
};

struct OrcBf16Layer {
  const uint16_t* router_proj;      // [E][H]
  const uint16_t* router_scale;     // [H] baked
  const uint16_t* pes;              // [E]
  const uint16_t* gamma2;           // [H] (not split-baked on the bf16 model)
  const uint16_t* w_gu;             // [E][GU][H]
  const uint16_t* w_dn;             // [E][H][I]
};

// modeling/gemma_4_moe_bq.mojo:630-713 dispatch_bq_moe at `degree` ranks:
// every rank routes all tokens through its experts [r*epr,(r+1)*epr), writes
// a bf16 partial, and dispatch_allreduce_inplace (kernels/reductions.mojo:
// 76-95) sums the partials in f32 in rank order and rounds to bf16.
// Calls above 1024 tokens are processed in 1024-token chunks (the reference's
// per-call cap, modeling/gemma_4_moe_bq.mojo:978-981); results are per-token.
int orc_bq_moe_forward(const uint16_t* x, int T, const OrcBqLayer* L, int degree,
                       uint16_t* out, int32_t* route_idx_out, float* route_w_out,
                       float* logits_out) {
  if (degree < 1 || E % degree) return -1;
  const int epr = E / degree;
  for (int t0 = 0; t0 < T; t0 += 1024) {
    int Tc = std::min(1024, T - t0);
    const uint16_t* xc = x + (long)t0 * H;
    std::vector<int32_t> ridx(Tc * TOPK);
    std::vector<float> rw(Tc * TOPK);
    orc_router(xc, Tc, L->router_centered, L->router_scale, L->pes, ridx.data(), rw.data(),
               logits_out ? logits_out + (long)t0 * E : nullptr);
    if (route_idx_out) std::memcpy(route_idx_out + t0 * TOPK, ridx.data(), Tc * TOPK * 4);
    if (route_w_out) std::memcpy(route_w_out + t0 * TOPK, rw.data(), Tc * TOPK * 4);
    std::vector<int8_t> xi8((size_t)Tc * H);
    std::vector<float> xsa(Tc);
    orc_bq_norm_quant(xc, L->gamma2, Tc, xi8.data(), xsa.data());
    std::vector<float> sum((size_t)Tc * H, 0.0f);
    std::vector<uint16_t> part((size_t)Tc * H);
    for (int r = 0; r < degree; ++r) {
      std::vector<int32_t> off(epr + 1);
      std::vector<OrcSparseRoute> routes(Tc * TOPK);
      orc_build_schedules(ridx.data(), rw.data(), Tc, r * epr, epr, off.data(), routes.data());
      int nrec = off[epr];
      std::vector<uint16_t> bucket((size_t)std::max(nrec, 1) * I);
      orc_bq_phase1(xi8.data(), xsa.data(), off.data(), routes.data(),
                    L->gu_q + (long)r * epr * GU * H, L->gu_scale + (long)r * epr * GU,
                    L->gu_cs + (long)r * epr * GU, epr, bucket.data());
      std::vector<int8_t> bi8((size_t)std::max(nrec, 1) * I);
      std::vector<float> bsa((size_t)std::max(nrec, 1) * NB_DOWN);
      orc_bq_block_quant(bucket.data(), nrec, I, DOWN_BLOCK, bi8.data(), bsa.data());
      orc_bq_phase2(bi8.data(), bsa.data(), off.data(), routes.data(),
                    L->dn_q + (long)r * epr * H * I, L->dn_scale + (long)r * epr * H,
                    L->dn_cs + (long)r * epr * H, (long)E * H, epr, Tc,
                    degree == 1 ? out + (long)t0 * H : part.data());
      if (degree > 1)
        for (size_t i = 0; i < (size_t)Tc * H; ++i) sum[i] = sum[i] + bf2f(part[i]);
    }
    if (degree > 1)
      for (size_t i = 0; i < (size_t)Tc * H; ++i) out[(long)t0 * H + i] = f2bf(sum[i]);
  }
  return 0;
}

// modeling/gemma_4_moe.mojo:493-566 dispatch_moe (bf16) at `degree` ranks.
int orc_bf16_moe_forward(const uint16_t* x, int T, const OrcBf16Layer* L, int degree,
                         uint16_t* out, int32_t* route_idx_out, float* route_w_out,
                         float* logits_out) {
  if (degree < 1 || E % degree) return -1;
  const int epr = E / degree;
  for (int t0 = 0; t0 < T; t0 += 1024) {
    int Tc = std::min(1024, T - t0);
    const uint16_t* xc = x + (long)t0 * H;
    std::vector<int32_t> ridx(Tc * TOPK);
    std::vector<float> rw(Tc * TOPK);
    orc_router(xc, Tc, L->router_proj, L->router_scale, L->pes, ridx.data(), rw.data(),
               logits_out ? logits_out + (long)t0 * E : nullptr);
    if (route_idx_out) std::memcpy(route_idx_out + t0 * TOPK, ridx.data(), Tc * TOPK * 4);
    if (route_w_out) std::memcpy(route_w_out + t0 * TOPK, rw.data(), Tc * TOPK * 4);
    std::vector<uint16_t> xn((size_t)Tc * H);
    orc_rms_norm(xc, L->gamma2, Tc, xn.data());
    std::vector<float> sum((size_t)Tc * H, 0.0f);
    std::vector<uint16_t> part((size_t)Tc * H);
    for (int r = 0; r < degree; ++r) {
      std::vector<int32_t> off(epr + 1);
      std::vector<OrcSparseRoute> routes(Tc * TOPK);
      orc_build_schedules(ridx.data(), rw.data(), Tc, r * epr, epr, off.data(), routes.data());
      int nrec = off[epr];
      std::vector<uint16_t> bucket((size_t)std::max(nrec, 1) * I);
      orc_phase1_bf16(xn.data(), off.data(), routes.data(), L->w_gu + (long)r * epr * GU * H,
                      epr, bucket.data());
      orc_phase2_bf16(off.data(), routes.data(), bucket.data(), L->w_dn + (long)r * epr * H * I,
                      epr, Tc, degree == 1 ? out + (long)t0 * H : part.data());
      if (degree > 1)
        for (size_t i = 0; i < (size_t)Tc * H; ++i) sum[i] = sum[i] + bf2f(part[i]);
    }
    if (degree > 1)
      for (size_t i = 0; i < (size_t)Tc * H; ++i) out[(long)t0 * H + i] = f2bf(sum[i]);
  }
  return 0;
}

int orc_num_threads() {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

void orc_set_num_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

}  // extern "C"
