// gm_kernels.h -- internal launchers of the MoE block kernels (not the C ABI;
// the public boundary is include/gmoe.h).
#pragma once
#include <algorithm>
#include "gm_common.cuh"

struct gm_moe;

namespace gm {

// Kernels launched through launch_k by the calling host thread (the handle
// takes differences around its own launches to count them).
inline thread_local long tls_kernel_launches = 0;
// Programmatic dependent launch for launch_k on the calling thread (the
// handle sets it from GM_OPT_PDL for the duration of a forward).
inline thread_local bool tls_pdl = true;

// Launch with programmatic stream serialisation (see pdl_wait/pdl_trigger):
// every kernel launched this way calls pdl_wait() before touching memory that
// an earlier kernel of the stream writes or reads.
template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                     Args&&... args) {
  ++tls_kernel_launches;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = tls_pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// Records the text returned by gm_last_error(NULL) on the calling thread.
void set_thread_error(const char* msg);
// Shard of a handle (device, first expert held, experts held, layers) and a
// failure recorded on it, for code outside gm_api.cu (the checkpoint loader).
int handle_shard(const ::gm_moe* h, int* device, int* expert_base, int* epr, int* num_layers);
int handle_fail(::gm_moe* h, int code, const char* msg);

int max_route_chunks(int T, int epr, int rc);
// The router writes split-K partial logit slices [slice][T][E];
// router_ksplit(T) is how many the top-8 kernels sum, in slice order: up to 32
// tokens the FMA kernel reduces its ROUTER_SLICES slices itself into slice 0
// (1); from ROUTER_WIDE_MIN_TOKENS the tcgen05 kernel writes
// ROUTER_WIDE_SLICES slices; in between ROUTER_SLICES.
constexpr int ROUTER_SLICES = H / 256;
constexpr int ROUTER_WIDE_SLICES = 4;
constexpr int ROUTER_WIDE_MIN_TOKENS = 3584;
int router_ksplit(int T);
// Up to this many tokens the top-8 and the schedule run as one CTA.
constexpr int TOPK_SCHEDULE_FUSED_MAX = 32;
// Tile counters of the FMA kernel's in-kernel reduction (ints, zero between calls).
int router_tile_counters(int T);
// Router workspace: partials, inv_rms [T], an error word, tile counters.
size_t router_workspace_floats(int T);

// Router dots as split-K partials [ksplit][T][E] over x * router_scale (the
// top-8 step multiplies their sum by inv_rms).  With a device error word and
// T >= ROUTER_TC_MIN_TOKENS the tcgen05 kernel (router_tc.cu) runs, otherwise
// the FMA kernel.  Both read only x and the router weights, so they run beside
// the norm kernel launched just before them (see router.cu).
constexpr int ROUTER_TC_MIN_TOKENS = 512;
// wait_first: the router is the forward's first kernel, so it waits for its
// predecessor before reading x (the tcgen05 prefill path, see gm_api.cu).
cudaError_t launch_router_logits(const uint16_t* x, const uint16_t* wr, const uint16_t* rscale, int T,
                                 float* logits, int* err, int* tile_counters, cudaStream_t s,
                                 bool wait_first = false);
cudaError_t launch_router_logits_tc(const uint16_t* x, const uint16_t* wr, const uint16_t* rscale, int T,
                                    float* logits, int* err, cudaStream_t s, bool wait_first = false);
cudaError_t launch_rms_inv(const uint16_t* x, int T, float* inv_rms, cudaStream_t s);
cudaError_t launch_topk(float* logits, const uint16_t* pes, const float* inv_rms, int T,
                        int32_t* route_idx, float* route_w, cudaStream_t s);
cudaError_t launch_topk_inv(const uint16_t* x, float* logits, const uint16_t* pes, float* inv_rms, int T,
                            int32_t* route_idx, float* route_w, cudaStream_t s);
// top-8 + softmax followed by the expert schedule (one CTA when T <= 1024;
// otherwise a top-8 grid and, given `counts` scratch of schedule_counts_ints(T)
// ints, the two-pass multi-CTA schedule)
cudaError_t launch_topk_schedule(float* logits, const uint16_t* pes, const float* inv_rms, int T,
                                 int32_t* route_idx, float* route_w, int expert_base, int epr,
                                 int route_chunk, int32_t* expert_offset, SparseRoute* routes,
                                 int32_t* route_pos, int32_t* chunk_off, int32_t* counts, cudaStream_t s);
// The same, with each token's inv_rms computed from its x row by the top-8
// warp (rms_inv_kernel's chain and reduction) and written to inv_rms: for the
// tcgen05 prefill path, where the norm runs after the schedule.
cudaError_t launch_topk_inv_schedule(const uint16_t* x, float* logits, const uint16_t* pes, float* inv_rms,
                                     int T, int32_t* route_idx, float* route_w, int expert_base, int epr,
                                     int route_chunk, int32_t* expert_offset, SparseRoute* routes,
                                     int32_t* route_pos, int32_t* chunk_off, int32_t* counts, cudaStream_t s);
int schedule_counts_ints(int T);
cudaError_t launch_schedule_multi(const int32_t* route_idx, const float* route_w, int T,
                                  int expert_base, int epr, int route_chunk, int32_t* counts,
                                  int32_t* expert_offset, SparseRoute* routes, int32_t* route_pos,
                                  int32_t* chunk_off, cudaStream_t s);

cudaError_t launch_router(const uint16_t* x, const uint16_t* wr, const uint16_t* rscale,
                          const uint16_t* pes, int T, float* logits, int32_t* route_idx,
                          float* route_w, cudaStream_t s);
cudaError_t launch_build_schedule(const int32_t* route_idx, const float* route_w, int T,
                                  int expert_base, int epr, int route_chunk,
                                  int32_t* expert_offset, SparseRoute* routes, int32_t* route_pos,
                                  int32_t* chunk_off, cudaStream_t s);
cudaError_t launch_bq_norm_quant(const uint16_t* x, const uint16_t* gamma, int T, int8_t* xi8,
                                 float* xsa, float* inv_rms, cudaStream_t s);
// The norm + FWHT-128 + int8 of bq_norm_quant with the token's inv_rms read
// from inv_rms (the top-8 kernel's) and the row stored once per local route,
// at xg[route_pos[t*8+k]] (schedule order), with its scale at xg_sa[...]: the
// tcgen05 prefill path's routed rows without an x_i8 copy or gather pass.
cudaError_t launch_bq_norm_gather(const uint16_t* x, const uint16_t* gamma, const float* inv_rms, int T,
                                  const int32_t* route_pos, int8_t* xg, float* xg_sa, cudaStream_t s);
// The bf16 layers' counterpart: bf16(x * inv_rms * gamma) rows (rms_norm_bf16)
// stored once per local route at xgb[route_pos[t*8+k]].
cudaError_t launch_rms_norm_gather_bf16(const uint16_t* x, const uint16_t* gamma, const float* inv_rms, int T,
                                        const int32_t* route_pos, uint16_t* xgb, cudaStream_t s);
cudaError_t launch_block_quant(const uint16_t* bucket, long rows, int8_t* qi8, float* sa,
                               cudaStream_t s);
cudaError_t launch_rms_norm_bf16(const uint16_t* x, const uint16_t* gamma, int T, uint16_t* out,
                                 float* inv_rms, cudaStream_t s);
// out = bf16(residual + src * inv_rms(src) * w) per token; out may alias residual.
cudaError_t launch_norm_residual_add(const uint16_t* src, const uint16_t* residual, const uint16_t* w, int T,
                                     uint16_t* out, cudaStream_t s);
cudaError_t launch_bq_phase1(const int8_t* xi8, const float* xsa, const int32_t* expert_offset,
                             const SparseRoute* routes, const int32_t* chunk_off, int epr, int T,
                             const int8_t* w_gu, const float* gu_scale, int8_t* bucket_i8,
                             float* bucket_sa, uint16_t* bucket_bf16, cudaStream_t s);
// dense butterquant MLP (dense_bq.cu): gate/up products + GeGLU + FWHT-64
// block quant of h (h_bf16 optional), then the down product to bf16 [T][H]
cudaError_t launch_dense_gate_up(const int8_t* xi8, const float* xsa, int T, const int8_t* wg,
                                 const float* gsc, const int8_t* wu, const float* usc,
                                 int8_t* h_i8, float* h_sa, uint16_t* h_bf16, cudaStream_t s);
cudaError_t launch_dense_down(const int8_t* hi8, const float* hsa, int T, const int8_t* wd,
                              const float* dsc, uint16_t* out, cudaStream_t s);
// bulk L2 prefetch of [base, base + bytes) (16-byte aligned base)
// L2 prefetch of n_units units of unit_bytes, unit k at (first + stride*k)
cudaError_t launch_l2_prefetch(const void* base, size_t unit_bytes, int n_units, int first, int stride,
                               cudaStream_t s);
cudaError_t launch_bq_phase2(const int8_t* bi8, const float* bsa, const int32_t* expert_offset,
                             const SparseRoute* routes, const int32_t* chunk_off, int epr, int T,
                             const int8_t* w_dn, const float* dn_scale, float* ybuf,
                             bool after_phase1, cudaStream_t s);
cudaError_t launch_bf16_phase1(const uint16_t* xn, const int32_t* expert_offset,
                               const SparseRoute* routes, const int32_t* chunk_off, int epr, int T,
                               const uint16_t* w_gu, uint16_t* bucket, cudaStream_t s);
cudaError_t launch_bf16_phase2(const uint16_t* bucket, const int32_t* expert_offset,
                               const SparseRoute* routes, const int32_t* chunk_off, int epr, int T,
                               const uint16_t* w_dn, float* ybuf, cudaStream_t s);
cudaError_t launch_combine(const int32_t* route_idx, const int32_t* route_pos, const float* ybuf,
                           int T, uint16_t* out, cudaStream_t s);
struct PostParams;
// the combine, then the post-MoE tail updating p.x_main (post_moe.cuh)
cudaError_t launch_combine_post(const int32_t* route_idx, const int32_t* route_pos, const float* ybuf,
                                int T, const PostParams& p, cudaStream_t s);
// tcgen05 prefill path (gemm_tc.cu)
// 2-D TMA descriptor (128-byte swizzle, boxes of 128 bytes x box_rows rows)
// over a row-major [rows][cols] tensor of 1-byte (int8) or 2-byte (bf16) elements
bool make_tmap_2d(void* map, const void* base, long rows, int cols, int elem_bytes, int box_rows);
bool make_tmap_i8(void* map, const void* base, long rows, int cols, int box_rows);
size_t tmap_bytes();
// rows of row_bytes gathered in schedule order (xsa/xg_sa optional)
cudaError_t launch_gather_rows(const void* x, int row_bytes, const float* xsa,
                               const SparseRoute* routes, const int32_t* expert_offset, int epr,
                               int T, void* xg, float* xg_sa, cudaStream_t s);
cudaError_t launch_tc_phase1(const void* map_a, const void* map_b, const int32_t* expert_offset,
                             int epr, int T, const float* xg_sa, const float* gu_scale,
                             int8_t* bucket_i8, float* bucket_sa, uint16_t* bucket_bf16, int* err,
                             cudaStream_t s);
// map_y: make_tmap_2d(f32 route rows ybuf, 4-byte elements, 32-row boxes)
cudaError_t launch_tc_phase2(const void* map_a, const void* map_b, const void* map_y, const int32_t* expert_offset,
                             int epr, int T, const float* bsa, const SparseRoute* routes,
                             const float* dn_scale, float* ybuf, int* err, cudaStream_t s);
// butterquant attention (attention_bq.cu).  runs: device array of
// {buf_start, base_pos, rows_off, page_count} (gm_kv_run_t)
cudaError_t launch_attn_prep(const uint16_t* q_src, const uint16_t* k_src, const uint16_t* v_src,
                             const uint16_t* q_norm, const uint16_t* k_norm, int8_t* q_i8, float* qi_bias,
                             float* f_q, int8_t* k_cache, float* k_scale, int8_t* v_cache, float* v_scale,
                             const float* cos_table, const float* sin_table, const void* runs, int num_runs,
                             const int32_t* base_rows, int T, int head_dim, int num_q, int num_kv,
                             int rope_half, int pair_stride, int cache_degree, int rank, int shift,
                             int row_mask, int page_mask, cudaStream_t s);
cudaError_t launch_attn_decode(const int8_t* q_i8, const float* f_q, const int8_t* k_cache,
                               const float* k_scale, const int8_t* v_cache, const float* v_scale,
                               const void* runs, const int32_t* base_rows, int T, int head_dim, int num_q,
                               int num_kv, int window, int cache_degree, int rank, int shift, int row_mask,
                               int page_mask, int max_kv_len, float* partials, uint16_t* out, cudaStream_t s);
int attention_splits(int T, int head_dim, int num_q, int num_kv, int max_kv_len);
// prefill attention over multi-token runs (Gemma-4 geometries: head 256 with
// 2 query heads per KV head, head 512 with 8)
cudaError_t launch_attn_prefill(const int8_t* q_i8, const float* f_q, const int8_t* k_cache, const float* k_scale,
                                const int8_t* v_cache, const float* v_scale, const void* runs, int num_runs,
                                const int32_t* base_rows, int T, int head_dim, int num_q, int num_kv, int window,
                                int shift, int row_mask, int page_mask, uint16_t* out, cudaStream_t s);
// splits of launch_attn_decode (out == NULL) reduced to one unnormalised
// (m, l, acc) per (token, head) [T*num_q][head_dim + 2]; the ranks' partials
// merged in rank order and normalised into bf16 [T][num_q*head_dim]
cudaError_t launch_attn_rank_partial(const float* partials, int T, int num_q, int head_dim, int n_splits,
                                     float* part, cudaStream_t s);
cudaError_t launch_attn_merge_parts(const float* const* parts, int n, int T, int num_q, int head_dim,
                                    uint16_t* out, cudaStream_t s);
size_t attention_workspace_floats(int T, int head_dim, int num_q, int num_kv, int max_kv_len);
// tcgen05 path of the dense MLP (gemm_tc.cu): maps over the activation rows
// (int8 [rows][2816], 128-row boxes), the row-major gate|up weight ([4224][2816],
// 64-row boxes), h (int8 [rows][2112], 128-row boxes) and the row-major down
// weight ([2816][2112], 128-row boxes); gu_scale is gate scales then up scales
cudaError_t launch_tc_dense_gate_up(const void* map_x, const void* map_w, int T, const float* xsa,
                                    const float* gu_scale, int8_t* h_i8, float* h_sa,
                                    uint16_t* h_bf16, int* err, cudaStream_t s);
cudaError_t launch_tc_dense_down(const void* map_h, const void* map_w, int T, const float* hsa,
                                 const float* dn_scale, uint16_t* out, int* err, cudaStream_t s);
// tcgen05 prefill path for bf16 layers (gemm_tc_bf16.cu)
cudaError_t launch_tcb_phase1(const void* map_a, const void* map_b, const int32_t* expert_offset,
                              int epr, int T, uint16_t* bucket, int* err, cudaStream_t s);
cudaError_t launch_tcb_phase2(const void* map_a, const void* map_b, const int32_t* expert_offset,
                              int epr, int T, const SparseRoute* routes, float* ybuf, int* err,
                              cudaStream_t s);

// attention block products (attn_block.cu): up to 3 bq_linear products over
// one activation (K = 2816), general block quant, general block linear
cudaError_t launch_bq_linear_multi(const int8_t* xi8, const float* xsa, int T, int nseg,
                                   const int8_t* const* w, const float* const* scale, uint16_t* const* out,
                                   const int* n_rows, cudaStream_t s);
cudaError_t launch_block_quant_ex(const uint16_t* src, long rows, int cols, int block, int fwht,
                                  int8_t* qi8, float* sa, cudaStream_t s);
cudaError_t launch_block_linear_ex(const int8_t* hi8, const float* hsa, int T, int k, int block,
                                   const int8_t* w, const float* wsc, int n_rows, uint16_t* out,
                                   cudaStream_t s);

cudaError_t launch_quantize_rows(const uint16_t* w, long rows, int cols, const uint16_t* gamma,
                                 int block, int8_t* q, float* scale, cudaStream_t s);
cudaError_t launch_vnni_permute(const int8_t* src, long rows, int cols, int8_t* dst, int dir,
                                cudaStream_t s);
cudaError_t launch_router_center(const uint16_t* w, int rows, int cols, uint16_t* out,
                                 cudaStream_t s);
cudaError_t launch_bake(const uint16_t* in, uint16_t* out, int n, int kind, cudaStream_t s);

}  // namespace gm
