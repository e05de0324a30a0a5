/* gmoe.h -- C ABI of the B200 (sm_100a) Gemma-4 mixture-of-experts block.
 *
 * Drop-in for the MoE operator of the Mojo CPU engine CoffeeVampir3/Mojo-Gemma4-CPU.
 * Every entry point names the reference interface it replaces (paths are
 * inside that project).  All pointers are plain addresses; bf16 tensors are
 * 16-bit words; no PyTorch or other framework types cross this boundary.
 *
 * Conventions
 *  - Return value: GM_OK (0) or a negative GM_E* status.  Nothing aborts or
 *    traps; the text of the last failure is available from gm_last_error().
 *  - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 *    Entry points taking a stream are asynchronous and stream-ordered.
 *  - Device pointers unless stated otherwise.
 *  - Dimensions are fixed by the model: hidden 2816, 128 experts, top-8,
 *    expert intermediate 704 (gate|up fused 1408), down FWHT block 64
 *    (modeling/gemma4_common.mojo:5,23-28).
 */
#ifndef GMOE_H
#define GMOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GM_OK 0
#define GM_EINVAL (-1)   /* bad argument or shape */
#define GM_ECUDA (-2)    /* CUDA runtime error */
#define GM_ENOMEM (-3)   /* device allocation failed */
#define GM_ENCCL (-4)    /* collective error */
#define GM_ETIMEOUT (-5) /* bounded wait expired */
#define GM_ESTATE (-6)   /* call out of order (e.g. layer not registered) */

#define GM_HIDDEN 2816
#define GM_NUM_EXPERTS 128
#define GM_TOP_K 8
#define GM_INTERMEDIATE 704
#define GM_GATE_UP 1408
#define GM_DOWN_BLOCK 64
#define GM_ROUTE_CHUNK_BQ 16   /* route_chunk the butterquant expert kernels expect */
#define GM_ROUTE_CHUNK_BF16 8  /* route_chunk the bf16 expert kernels expect */

/* kernels/moe_router.mojo:33-36 SparseRoute{token, weight}. */
typedef struct gm_sparse_route {
  int32_t token;
  float weight;
} gm_sparse_route_t;

typedef struct gm_moe gm_moe_t;

const char* gm_version(void);

/* Text of the last failure on this handle; with h == NULL, of the last failed
 * stateless call on the calling thread. */
const char* gm_last_error(const gm_moe_t* h);

/* ---------------------------------------------------------------- handle --
 * Replaces the per-model state the reference keeps for the MoE: expert weights
 * in per-rank arenas (modeling/gemma_4_moe_bq.mojo:872-918 init_state /
 * model_init) and the phase-scoped MoE scratch (Gemma4FfnMoeScratch,
 * modeling/gemma_4_moe_bq.mojo:275-360).  Workspace is allocated once here for
 * `max_tokens` tokens per call; calls never allocate.
 * rank/degree: expert-parallel placement, experts [rank*128/degree,
 * (rank+1)*128/degree) live on this handle (modeling/model_spec.mojo:106-110). */
int gm_moe_create(gm_moe_t** out, int device, int max_tokens, int num_layers, int rank,
                  int degree);
int gm_moe_destroy(gm_moe_t* h);
size_t gm_moe_workspace_bytes(int max_tokens);

/* Butterquant layer weights, exactly in the reference's in-memory layout
 * (host or device pointers; copied to the handle's device memory):
 *   gate_up      int8, VNNI-packed [epr*1408][2816] (butterquant/vnni.mojo:31-83),
 *                rows FWHT-128-rotated and split-gain scaled (quant/quantizer.mojo:963-1051)
 *   gate_up_scale f32 [epr*1408] (amax/127)
 *   down         int8, VNNI-packed [epr*2816][704], FWHT-64 rotated
 *   down_scale   f32 [epr*2816]
 *   router_centered bf16 [128][2816] (butterquant/kernels.mojo:218-224)
 *   router_scale bf16 [2816], baked * 1/sqrt(2816) (modeling/gemma4_topology.mojo:362-388)
 *   per_expert_scale bf16 [128]
 *   pre_ffn_norm_2 bf16 [2816], split-gain baked (butterquant/kernels.mojo:37-45)
 * epr = 128/degree; the expert tensors hold this rank's experts only, as the
 * reference's row-block sharded bindings do (modeling/loader.mojo:113-125).
 * The colsum sidecars of ButterquantWeight (butterquant/weight.mojo:50-64) are
 * not taken: the kernels use signed x signed dots, which need none
 * (quantization_docs/butterquant.md section 2.5). */
int gm_moe_register_layer_bq(gm_moe_t* h, int layer, const void* gate_up,
                             const float* gate_up_scale, const void* down,
                             const float* down_scale, const void* router_centered,
                             const void* router_scale, const void* per_expert_scale,
                             const void* pre_ffn_norm_2);

/* bf16 layer weights (modeling/gemma_4_moe.mojo): gate_up bf16 [epr][1408][2816],
 * down bf16 [epr][2816][704], router_proj bf16 [128][2816], router_scale
 * (baked), per_expert_scale, pre_ffn_norm_2 (raw gain, not split-baked). */
int gm_moe_register_layer_bf16(gm_moe_t* h, int layer, const void* gate_up, const void* down,
                               const void* router_proj, const void* router_scale,
                               const void* per_expert_scale, const void* pre_ffn_norm_2);

/* The MoE operator.  Replaces dispatch_bq_moe (modeling/gemma_4_moe_bq.mojo:
 * 630-713) or, for a bf16 layer, dispatch_moe (modeling/gemma_4_moe.mojo:
 * 493-566): x_input bf16 [T][2816] -> moe_out bf16 [T][2816].  At degree > 1
 * the output is this rank's partial (its experts only, rounded to bf16), i.e.
 * the value the reference holds just before dispatch_allreduce_inplace
 * (kernels/reductions.mojo:186-204); summing the partials across ranks is the
 * caller's exchange step.
 * Asynchronous on `stream`; x and out are device pointers. */
int gm_moe_forward(gm_moe_t* h, int layer, const void* x, void* out, int T, void* stream);

/* Post-MoE tail of dispatch_bq_ffn (modeling/gemma_4_moe_bq.mojo:785-805),
 * fused into the MoE's final kernel so the MoE output never goes to memory:
 *   dense' = rms_norm(dense_out) * post_ffn_norm_1
 *   dense' = dense' + rms_norm(moe_out) * post_ffn_norm_2
 *   x_main = (x_main + rms_norm(dense') * post_ffn_norm) * layer_scalar
 * with the reference's bf16 rounding after each step (kernels/rmsnorm.mojo:
 * 21-67, kernels/elementwise.mojo:75-83).  gm_moe_register_post stores the
 * three bf16 [2816] gains (host or device pointers) and the layer scalar;
 * gm_moe_forward_ffn(h, layer, x_main, dense_out, T, stream) runs the MoE on
 * x_main (its input, as dispatch_bq_ffn passes x_main) and overwrites x_main
 * with the layer's post-FFN value.  dense_out is the dense MLP's output after
 * its all-reduce (bf16 [T][2816], device pointer, read only). */
int gm_moe_register_post(gm_moe_t* h, int layer, const void* post_ffn_norm_1,
                         const void* post_ffn_norm_2, const void* post_ffn_norm, float layer_scalar);
int gm_moe_forward_ffn(gm_moe_t* h, int layer, void* x_main, const void* dense_out, int T,
                       void* stream);

/* The dense butterquant MLP of the same FFN (dispatch_bq_ffn,
 * modeling/gemma_4_moe_bq.mojo:749-783), weights replicated on every handle
 * (17.8 MB per layer; tokens stay on their GPU):
 *   gate_proj, up_proj  int8 VNNI-packed [2112][2816], FWHT-128 rotated,
 *                       split gain of pre_feedforward_layernorm folded in
 *                       (SplitGainPerRowCs, modeling/gemma_4_moe_bq.mojo:113-114)
 *   gate_scale, up_scale f32 [2112]
 *   down_proj           int8 VNNI-packed [2816][2112], FWHT-64 rotated
 *                       (PlainPerRowBlockCs[64]), down_scale f32 [2816]
 *   pre_ffn_norm        bf16 [2816], split-gain baked
 * gm_dense_forward: x [T][2816] -> dense_out [T][2816] (device, async): the
 * reference's dispatch_bq_norm_quant, two dispatch_bq_linear,
 * dispatch_gelu_gate_up, dispatch_bq_block_quant and dispatch_bq_block_linear.
 * gm_ffn_forward: the whole FFN on x_main in place -- the dense MLP on a
 * forked stream beside the MoE, then the MoE's combine with the post-MoE tail
 * (needs gm_moe_register_post; at degree > 1 only with expert parallelism). */
int gm_moe_register_dense_bq(gm_moe_t* h, int layer, const void* gate_proj, const float* gate_scale,
                             const void* up_proj, const float* up_scale, const void* down_proj,
                             const float* down_scale, const void* pre_ffn_norm);
int gm_dense_forward(gm_moe_t* h, int layer, const void* x, void* dense_out, int T, void* stream);
int gm_ffn_forward(gm_moe_t* h, int layer, void* x_main, int T, void* stream);

/* ----------------------------------------------- attention block products --
 * The products of the butterquant attention block around the attention core
 * (modeling/gemma_4_moe_bq.mojo:418-627), weights in the reference's VNNI
 * layout (device pointers, async on `stream`):
 * gm_bq_linear: dispatch_bq_linear (butterquant_kernels/linear.mojo:119-150):
 *   out bf16 [T][n_rows] = (dot(x_i8, w) * (x_sa/127)) * w_scale over K = 2816
 *   (x_i8/x_sa from gm_bq_norm_quant); n_rows a multiple of 32.
 * gm_bq_qkv: dispatch_bq_qkv (linear.mojo:273-328): the q, k and v products of
 *   one attention layer over the same activation in one launch (q [T][qn],
 *   k and v [T][kvn]); v_w == NULL for the full layers, whose V is K.
 * gm_bq_block_quant_ex: dispatch_bq_block_quant[block, apply_fwht]
 *   (linear.mojo:182-205, butterquant/runtime.mojo:62-79): bf16 [rows][cols]
 *   -> int8 + per-block amax [rows][cols/block]; block 64/128/256/512, FWHT
 *   only with block 64.  The attention output uses block = head_dim, no FWHT.
 * gm_bq_block_linear_ex: dispatch_bq_block_linear (linear.mojo:240-270,
 *   butterquant/gemm.mojo:174-216) for any block: out bf16 [T][n_rows], the
 *   per-block fma chain in block order; k/block a multiple of 4 or 3.  The
 *   attention output projection (o_proj, block = head_dim). */
int gm_bq_linear(const int8_t* x_i8, const float* x_sa, int T, const void* w, const float* w_scale,
                 int n_rows, void* out, void* stream);
int gm_bq_qkv(const int8_t* x_i8, const float* x_sa, int T, const void* q_w, const float* q_scale, int qn,
              const void* k_w, const float* k_scale, const void* v_w, const float* v_scale, int kvn,
              void* q_out, void* k_out, void* v_out, void* stream);
int gm_bq_block_quant_ex(const void* x, long rows, int cols, int block, int apply_fwht, int8_t* q, float* sa,
                         void* stream);
int gm_bq_block_linear_ex(const int8_t* h_i8, const float* h_sa, int T, int k, int block, const void* w,
                          const float* w_scale, int n_rows, void* out, void* stream);

/* ------------------------------------------------------------ checkpoints --
 * Safetensors checkpoints as the reference reads and writes them
 * (safetensors/parser.mojo, safetensors/writer.mojo:39-75): an 8-byte
 * little-endian header length, a JSON header {name: {dtype, shape,
 * data_offsets}} ("__metadata__" ignored), then the data.  `path` is one file
 * or a directory whose *.safetensors shards are merged (the reference's
 * source checkpoints are sharded; its butterquant output is one
 * model.safetensors, quant/quantizer.mojo:383-446).  Opening parses and
 * checks every header (offsets inside the file, byte counts equal to the
 * shapes); tensors are read on demand.  These calls need no GPU; failures
 * leave their text in gm_last_error(NULL). */
typedef struct gm_checkpoint gm_checkpoint_t;

#define GM_DTYPE_BOOL 1
#define GM_DTYPE_U8 2
#define GM_DTYPE_I8 3
#define GM_DTYPE_I16 4
#define GM_DTYPE_U16 5
#define GM_DTYPE_F16 6
#define GM_DTYPE_BF16 7
#define GM_DTYPE_I32 8
#define GM_DTYPE_U32 9
#define GM_DTYPE_F32 10
#define GM_DTYPE_I64 11
#define GM_DTYPE_U64 12
#define GM_DTYPE_F64 13
#define GM_DTYPE_F8_E4M3 14
#define GM_DTYPE_F8_E5M2 15
#define GM_CKPT_MAX_DIMS 8

int gm_checkpoint_open(gm_checkpoint_t** out, const char* path);
int gm_checkpoint_close(gm_checkpoint_t* ck);
/* Tensors in name order: count, and the name at `index` (NULL if out of range). */
int gm_checkpoint_tensor_count(const gm_checkpoint_t* ck);
const char* gm_checkpoint_tensor_name(const gm_checkpoint_t* ck, int index);
/* dtype (GM_DTYPE_*), rank and shape[GM_CKPT_MAX_DIMS] of a tensor. */
int gm_checkpoint_tensor_info(const gm_checkpoint_t* ck, const char* name, int* dtype, int* ndim,
                              int64_t* shape);
/* Rows [row0, row0+nrows) of a tensor seen as 2-D (all leading dimensions
 * folded into rows, quant/quantizer.mojo:62-71; a 1-D tensor is a column),
 * into host memory dst of dst_bytes. */
int gm_checkpoint_read_rows(const gm_checkpoint_t* ck, const char* name, int64_t row0,
                            int64_t nrows, void* dst, size_t dst_bytes);

/* One MoE layer from a checkpoint into the handle: replaces the reference's
 * weight load (modeling/loader.mojo:95-150, this rank's row block of the
 * expert tensors) plus its load-time transforms (VNNI packing,
 * modeling/slot.mojo:263-300; router scale bake,
 * modeling/gemma4_topology.mojo:362-388; split-gain bake of
 * pre_feedforward_layernorm_2, modeling/gemma_4_moe_bq.mojo:905-910), then
 * registers the layer as gm_moe_register_layer_bq / _bf16 would.  The format
 * follows the dtype of experts.gate_up_proj: I8 is the butterquant file
 * (members ".scale", quant/manifest.mojo:10-13,93-120), BF16 the original
 * checkpoint ([128][1408][2816] or folded).  Tensor names are `prefix` +
 * modeling/gemma4_topology.mojo:143-158 names; prefix NULL means
 * "model.language_model.layers.%d." with %d = ckpt_layer.  Flags:
 * GM_LOAD_POST also registers the post-MoE gains and layer_scalar
 * (gm_moe_register_post); GM_LOAD_DENSE also registers the dense MLP
 * (mlp.{gate,up,down}_proj.weight + pre_feedforward_layernorm.weight,
 * gm_moe_register_dense_bq); GM_LOAD_QUANTIZE turns a BF16 checkpoint into
 * the butterquant layer on the device, as the reference quantizer would
 * (quant/quantizer.mojo:963-1114: per-row FWHT + int8 with the split gains,
 * router centring), instead of registering bf16 experts.  Synchronous. */
#define GM_LOAD_POST 1
#define GM_LOAD_DENSE 2
#define GM_LOAD_QUANTIZE 4
int gm_moe_load_layer(gm_moe_t* h, int layer, const gm_checkpoint_t* ck, int ckpt_layer,
                      const char* prefix, int flags);

/* Options (no reference counterpart: the reference picks its kernels at
 * compile time).  GM_OPT_TC_MIN_TOKENS: calls with T >= value run the
 * butterquant gate/up product on the tcgen05 grouped GEMM (prefill path),
 * smaller calls on the HBM-streaming decode kernel; both give bit-identical
 * results.  Default 1024.  The prefill path reads a row-major copy of each
 * butterquant layer's expert weights, made at registration only when the
 * handle can reach it (max_tokens times the number of expert shards >=
 * the value at that time); a decode-only handle keeps the VNNI weights
 * alone, and layers registered without the copy run every call on the
 * decode kernels. 
 * GM_OPT_PROFILE: 1 records a CUDA event pair around every stage that
 * gm_moe_forward launches, 0 (default) records none; setting it (either
 * value) clears the stage statistics and the kernel launch count.
 * GM_OPT_PDL: 1 (default) launches the forward's kernels with programmatic
 * dependent launch (each kernel's prologue overlaps its predecessor's tail);
 * 0 launches them with plain stream ordering.
 * GM_OPT_EP_TRANSPORT (expert parallelism): 1 = the dispatch and combine
 * exchanges are stores into the peers' memory (CUDA IPC mappings over
 * NVLink) made by the pack and combine kernels themselves, ordered by flags;
 * the default whenever every rank could map every peer at gm_moe_ep_init.
 * 0 = NCCL send/recv.  Every rank must use the same value.
 * GM_OPT_DENSE_TC_MIN_TOKENS: calls with T >= value run the dense MLP's
 * products on tcgen05 GEMMs, smaller calls on its HBM-streaming kernels;
 * both give bit-identical results.  Default 128.
 * GM_OPT_EP_TIMEOUT_MS (expert parallelism, peer-memory transport): bound in
 * milliseconds of each exchange wait on the GPU, counted from the moment the
 * wait kernel starts.  Default 1000; every rank must enter each forward within
 * that time of its peers (raise it for a first forward that follows slow
 * host-side work on one rank).  On expiry the forward completes with
 * undefined output and gm_moe_device_status reports GM_ETIMEOUT.
 * GM_OPT_EP_INIT_TIMEOUT_MS: bound of gm_moe_ep_init's communicator set-up on
 * the host (default 120000); set it before gm_moe_ep_init. */
#define GM_OPT_TC_MIN_TOKENS 1
#define GM_OPT_PROFILE 2
#define GM_OPT_PDL 3
#define GM_OPT_EP_TRANSPORT 4
#define GM_OPT_DENSE_TC_MIN_TOKENS 5
#define GM_OPT_EP_TIMEOUT_MS 6
#define GM_OPT_EP_INIT_TIMEOUT_MS 7
int gm_moe_set_option(gm_moe_t* h, int option, long value);

/* Per-stage statistics of the handle's forwards.  Replaces the reference's
 * Profiler / DispatchSpan (kernels/profiling.mojo:214-254, 366-413): one
 * record per stage label (the reference's dispatch labels where a stage has
 * one: "bq_norm_quant", "router_expert", "bq_phase1_gate_up",
 * "bq_phase2_down", ...; tcgen05 variants carry a ".tc" suffix), with the
 * device time between the events recorded on the forward's stream before and
 * after the stage's launches. */
typedef struct gm_stage_stat {
  char label[32];
  long calls;       /* stage executions recorded */
  long kernels;     /* kernels the stage launched over those executions */
  double total_ms, min_ms, max_ms;
} gm_stage_stat_t;

/* Waits for the recorded events, folds them into the statistics and copies up
 * to max_stats records (first-seen order) into `stats`; *n_stats = number of
 * records.  *kernel_launches (may be NULL) = kernels gm_moe_forward launched
 * on this handle since creation or the last GM_OPT_PROFILE setting, counted
 * whether or not profiling is on. */
int gm_moe_profile_read(gm_moe_t* h, gm_stage_stat_t* stats, int max_stats, int* n_stats,
                        long* kernel_launches);

/* ------------------------------------------------------ expert parallelism --
 * One process (and one handle) per GPU.  Replaces the reference's expert
 * sharding by rank with replicated activations and the all-reduce of bf16
 * partials (modeling/gemma4_topology.mojo:109-114, modeling/gemma_4_moe_bq.mojo:
 * 711-713, kernels/reductions.mojo:186-204) by token-parallel dispatch and
 * combine over NCCL: each rank passes only its own tokens to gm_moe_forward.
 *
 * gm_ep_unique_id: writes an NCCL unique id (GM_EP_UNIQUE_ID_BYTES bytes) on
 * one rank; the caller distributes it to every rank.
 * gm_moe_ep_init: joins the group (collective: every rank calls it with the
 * same id; world == the handle's degree, rank == its rank).  Afterwards
 * gm_moe_forward(h, layer, x, out, T, stream) takes this rank's T tokens
 * (T <= max_tokens; every rank calls it for every layer, T may differ) and
 * writes their complete MoE output: bf16(sum over ranks in rank order of each
 * rank's bf16 partial), the value the reference's all-reduce produces.
 * The communicator is set up non-blocking and polled against
 * GM_OPT_EP_INIT_TIMEOUT_MS: if a rank never joins, the call aborts the
 * communicator and returns GM_ETIMEOUT instead of blocking.
 * The output of an expert-parallel forward is valid once the stream has
 * reached it AND gm_moe_device_status returns GM_OK: when a peer misses the
 * exchange (GM_OPT_EP_TIMEOUT_MS), the forward still completes, with
 * undefined output, and the status reports GM_ETIMEOUT. */
#define GM_EP_UNIQUE_ID_BYTES 128
int gm_ep_unique_id(void* out, size_t bytes);
int gm_moe_ep_init(gm_moe_t* h, const void* unique_id, int world);

/* Expert parallelism inside one process (the reference's ranks as handles of
 * one process, e.g. several handles sharing one GPU, or one handle per GPU
 * driven by one host thread).  gm_moe_ep_init_group joins `world` handles,
 * handles[g] created with rank g and degree world, all with the same
 * max_tokens; the exchange uses the members' buffers as plain pointers of
 * this process (peer access is enabled between their devices), no NCCL.
 * gm_moe_ep_forward_group runs one layer on every member: member g's T[g]
 * tokens x[g] -> out[g], on streams[g]; it issues the three phases of the
 * exchange (route and pack; experts and combine; final sum) for every member
 * before the next phase, so that members sharing a GPU never wait on a kernel
 * that has not been issued before them.  Members on one device must be given
 * the same stream (GM_EINVAL otherwise).  The result equals the multi-process
 * forward's bit for bit.  A lone gm_moe_forward on a member of a group that
 * shares a device has no peer running beside it: its exchange waits expire
 * (GM_OPT_EP_TIMEOUT_MS) and gm_moe_device_status reports GM_ETIMEOUT.
 * Destroy the members after their last forward; destroying one dissolves
 * the group (the others then return GM_ESTATE).
 * gm_moe_ep_set_placement_group: gm_moe_ep_set_placement for such a group
 * (one call for all members; expert weights move by device copies). */
int gm_moe_ep_init_group(gm_moe_t* const* handles, int world);
int gm_moe_ep_forward_group(gm_moe_t* const* handles, int world, int layer, const void* const* x,
                            void* const* out, const int* T, void* const* streams);
int gm_moe_ep_set_placement_group(gm_moe_t* const* handles, int world, const int32_t* expert_rank);

/* Optional load-based placement (no reference counterpart; the reference keeps
 * contiguous blocks).  expert_rank[128] (host) names the rank that holds each
 * expert, every rank exactly 128/world of them.  Collective (same map on every
 * rank), after gm_moe_ep_init and after every layer is registered: the layers
 * are still registered as the reference's contiguous blocks, and the library
 * exchanges expert weights (NCCL all-gather) so that each rank keeps its
 * assigned experts.  The per-rank partials are then sums over each rank's
 * placed experts, so results match the contiguous placement within rounding,
 * not bit for bit. */
int gm_moe_ep_set_placement(gm_moe_t* h, const int32_t* expert_rank);

/* Synchronises the handle's device and reports (then clears) the device-side
 * error word that kernels with bounded waits write when a wait expires:
 * *device_error = 0 and GM_OK when none did, GM_ETIMEOUT otherwise. */
int gm_moe_device_status(gm_moe_t* h, int* device_error);

/* Blocking form with the reference's calling convention (the reference's
 * dispatchers fan out and join before returning, kernels/helpers.mojo:295-327):
 * x and out may be host or device memory; host buffers are staged through the
 * handle's device buffers, except a page-locked, device-mapped `out` (for
 * example cudaHostAlloc memory), which the last kernel writes directly. */
int gm_moe_forward_sync(gm_moe_t* h, int layer, const void* x, void* out, int T);

/* ----------------------------------------------------- per-stage kernels --
 * Stateless entry points, one per reference dispatcher, for tests and for
 * callers that own their scratch.  Device pointers. */

/* dispatch_router_expert + dispatch_merge_router_candidates
 * (kernels/moe_router.mojo:206-244,333-389): route_idx i32 [T][8]
 * (logit-descending, ties to the lower id), route_w f32 [T][8] (softmax over
 * the 8, times per_expert_scale).  logits_ws: f32 workspace of
 * gm_router_workspace_bytes(T) bytes (split-K partial logits); on return its
 * first T*128 floats hold the logits [T][128]. */
size_t gm_router_workspace_bytes(int T);

int gm_router_select(const void* x, const void* router_w, const void* router_scale,
                     const void* per_expert_scale, int T, float* logits_ws, int32_t* route_idx,
                     float* route_w, void* stream);

/* gm_router_select without the caller's scratch buffer, for callers that
 * cannot allocate device memory (no cudaMalloc allowed where they run, fixed
 * memory pools only, or a binding that cannot own device buffers).  No
 * counterpart in the reference: its router scratch comes from the model's
 * phase-scoped pool.  Same inputs and outputs as gm_router_select, minus
 * logits_ws; the logits themselves are not returned.
 * Limit: T <= 256 (GM_EINVAL beyond).  The scratch is a fixed 1.38 MiB array
 * inside this library, present on every GPU that loads it until the process
 * exits, and shared by all calls on that GPU: calls that overlap on the GPU
 * race, so order them on one stream.  The first call on each device looks up
 * the array's device address (cudaGetSymbolAddress) with that device current;
 * make that first call before any stream capture.  That address is cached for
 * the life of the process: after cudaDeviceReset on a device, do not call this
 * entry point there again.  The call allocates nothing, but it does call the
 * CUDA runtime, so it cannot run inside a stream's host function. */
int gm_router_select_noalloc(const void* x, const void* router_w, const void* router_scale,
                             const void* per_expert_scale, int T, int32_t* route_idx,
                             float* route_w, void* stream);

/* dispatch_build_expert_schedules (kernels/moe_router.mojo:109-145) for the
 * experts [expert_base, expert_base+epr): expert_offset i32 [epr+1], routes
 * [T*8] (stable, token-major).  Extra outputs: route_pos i32 [T*8] (position of
 * route (t,k) in `routes`, -1 if not local) and chunk_off i32 [epr+1] (prefix
 * of ceil(n_e/route_chunk), the work split of the expert kernels). */
int gm_build_expert_schedules(const int32_t* route_idx, const float* route_w, int T,
                              int expert_base, int epr, int route_chunk, int32_t* expert_offset,
                              gm_sparse_route_t* routes, int32_t* route_pos, int32_t* chunk_off,
                              void* stream);

/* dispatch_rms_norm (kernels/rmsnorm.mojo:117) as used by dispatch_moe:
 * out = bf16(x*inv_rms*gamma). */
int gm_rms_norm(const void* x, const void* gamma, int T, void* out, void* stream);

/* fused_norm_residual_add (kernels/rmsnorm.mojo:48-64, norm_residual_add_row),
 * as the decoder layer applies it after the attention block
 * (modeling/gemma_4_moe_bq.mojo:1098-1102): per token,
 * out = bf16(residual + (src * inv_rms(src)) * weight), bf16 [T][2816]
 * (16-byte aligned).  out may be residual itself (the residual stream updated
 * in place). */
int gm_norm_residual_add(const void* src, const void* residual, const void* weight, int T, void* out,
                         void* stream);

/* dispatch_bq_norm_quant (butterquant_kernels/linear.mojo:58-82, block 128):
 * x_i8 [T][2816], x_sa f32 [T] (raw absmax). */
int gm_bq_norm_quant(const void* x, const void* gamma, int T, int8_t* x_i8, float* x_sa,
                     void* stream);

/* dispatch_bq_phase1_gate_up (butterquant_kernels/moe.mojo:132-164) fused with
 * dispatch_bq_block_quant of its output (butterquant_kernels/linear.mojo:
 * 182-205): bucket_i8 [R][704] + bucket_sa f32 [R][11]; bucket_bf16 [R][704]
 * (the reference's intermediate) is also written when non-NULL.  chunk_off
 * must come from gm_build_expert_schedules with route_chunk = GM_ROUTE_CHUNK_BQ.
 * T bounds the work (R <= T*8).  gate_up: VNNI-packed, as for register_layer_bq. */
int gm_bq_phase1_gate_up(const int8_t* x_i8, const float* x_sa, const int32_t* expert_offset,
                         const gm_sparse_route_t* routes, const int32_t* chunk_off, int epr, int T,
                         const void* gate_up, const float* gate_up_scale, int8_t* bucket_i8,
                         float* bucket_sa, void* bucket_bf16, void* stream);

/* dispatch_bq_block_quant[64, fwht] (butterquant_kernels/linear.mojo:182-205)
 * on a bf16 bucket [rows][704]. */
int gm_bq_block_quant(const void* bucket, long rows, int8_t* q, float* sa, void* stream);

/* dispatch_bq_phase2_down (butterquant_kernels/moe.mojo:298-335) without the
 * final accumulation: y f32 [R][2816], y[r] = facc*down_scale*route_weight of
 * route r.  gm_combine performs the per-token accumulation. */
int gm_bq_phase2_down(const int8_t* bucket_i8, const float* bucket_sa, const int32_t* expert_offset,
                      const gm_sparse_route_t* routes, const int32_t* chunk_off, int epr, int T,
                      const void* down, const float* down_scale, float* y, void* stream);

/* dispatch_phase1_gate_up (kernels/moe_experts.mojo:165-197), bf16; chunk_off
 * from route_chunk = GM_ROUTE_CHUNK_BF16.  bucket bf16 [R][704]. */
int gm_phase1_gate_up_bf16(const void* x_normed, const int32_t* expert_offset,
                           const gm_sparse_route_t* routes, const int32_t* chunk_off, int epr,
                           int T, const void* gate_up, void* bucket, void* stream);

/* dispatch_phase2_down (kernels/moe_experts.mojo:322-353) without the final
 * accumulation: y f32 [R][2816] = dot * route_weight. */
int gm_phase2_down_bf16(const void* bucket, const int32_t* expert_offset,
                        const gm_sparse_route_t* routes, const int32_t* chunk_off, int epr, int T,
                        const void* down, float* y, void* stream);

/* The accumulation tail of the phase-2 kernels (butterquant_kernels/moe.mojo:
 * 252-290): out[t] = bf16(sum of y[route_pos[t][k]] over the token's local
 * routes in ascending expert order, starting from 0). */
int gm_combine(const int32_t* route_idx, const int32_t* route_pos, const float* y, int T,
               void* out, void* stream);

/* ------------------------------------------------------- weight producer --
 * On-device restatement of the reference quantizer (quant/quantizer.mojo:
 * 963-1051 do_quant with butterquant/kernels.mojo:148-168 rotate_and_quant),
 * bit-identical to it: w bf16 [rows][cols] (* sqrt|gamma| if gamma != NULL),
 * FWHT-`fwht_block` along K, per-row absmax int8 q [rows][cols] row-major,
 * scale f32 [rows] = amax/127.  cols/block: 2816/128, 2816/64, 704/64 or
 * 2112/64 (the dense MLP's down_proj). */
int gm_bq_quantize_rows(const void* w, long rows, int cols, const void* gamma, int fwht_block,
                        int8_t* q, float* scale, void* stream);

/* Stages of the dense MLP on explicit buffers.  gm_bq_dense_gate_up:
 * dispatch_bq_linear on gate_proj and up_proj (butterquant_kernels/linear.mojo:
 * 85-130), dispatch_gelu_gate_up (kernels/elementwise.mojo:17-60) and
 * dispatch_bq_block_quant[64, fwht] (linear.mojo:159-205) in one pass:
 * x_i8 [T][2816], x_sa [T] -> h_i8 [T][2112], h_sa [T][33] (h_bf16
 * [T][2112], the GeGLU output, also written when non-NULL).
 * gm_bq_block_linear: dispatch_bq_block_linear (linear.mojo:208-270) with
 * n_rows 2816, k_dim 2112: h_i8, h_sa -> out bf16 [T][2816]. */
int gm_bq_dense_gate_up(const int8_t* x_i8, const float* x_sa, int T, const void* gate_proj,
                        const float* gate_scale, const void* up_proj, const float* up_scale,
                        int8_t* h_i8, float* h_sa, void* h_bf16, void* stream);
int gm_bq_block_linear(const int8_t* h_i8, const float* h_sa, int T, const void* down_proj,
                       const float* down_scale, void* out, void* stream);

/* ------------------------------------------------------ bq attention --
 * Decode attention of the butterquant model over its int8, FWHT-rotated,
 * paged KV cache.  Cache layout as the reference's (modeling/
 * gemma_4_moe_bq.mojo:123-160 KV slot groups): k/v int8 [rows][num_kv *
 * head_dim], k/v scales f32 [rows][num_kv] (the head's absmax).  Row of
 * position p (kernels/attention_ops.mojo:41-52 PagedKV):
 *   base_rows[run.rows_off + ((p >> page_shift) & page_mask)] + (p & row_mask)
 * with page_mask = pages-1 for the sliding ring and -1 for full layers.
 * Head geometries (modeling/gemma4_common.mojo:9-20): sliding head_dim 256,
 * rope_half 128, pair_stride 128; full head_dim 512, rope_half 64,
 * pair_stride 256 (others are refused).  All pointers are device memory. */
typedef struct gm_kv_run { /* kernels/attention_ops.mojo:55-60 KVRun */
  int32_t buf_start;  /* first token of the run in the batch */
  int32_t base_pos;   /* position of that token */
  int32_t rows_off;   /* first entry of the run's page list in base_rows */
  int32_t page_count;
} gm_kv_run_t;

/* dispatch_bq_attn_prep (butterquant_kernels/attention.mojo:474-610): T
 * tokens of q_src bf16 [T][num_q*head_dim], k_src / v_src bf16
 * [T][num_kv*head_dim] (v_src = k_src for the full layers) -> q_i8 [T][num_q *
 * head_dim], qi_bias = 128*sum(q_i8) and f_q = absmax [T][num_q], and the K/V
 * cache rows of the positions this rank holds (pos % cache_degree == rank).
 * cos/sin f32 [positions][rope_half].  Bit-identical to the reference's
 * 16-lane arithmetic. */
int gm_bq_attn_prep(const void* q_src, const void* k_src, const void* v_src, const void* q_norm,
                    const void* k_norm, int8_t* q_i8, float* qi_bias, float* f_q, int8_t* k_cache,
                    float* k_scale, int8_t* v_cache, float* v_scale, const float* cos_table,
                    const float* sin_table, const gm_kv_run_t* runs, int num_runs,
                    const int32_t* base_rows, int T, int head_dim, int num_q, int num_kv,
                    int rope_half, int pair_stride, int cache_degree, int rank, int page_shift,
                    int row_mask, int page_mask, void* stream);

/* The decode path of dispatch_bq_sliding_attention / dispatch_bq_full_attention
 * (attention.mojo:333-472, kernels/attention_dispatch_kernels.mojo:36-130):
 * T tokens, token t the newest position of run t (runs[t].buf_start = t).
 * Sliding (window > 0): the last min(pos+1, window) positions; full (window =
 * 0): positions 0..pos.  cache_degree must be 1 (rank 0); a cache sharded by
 * position over ranks goes through gm_bq_attention_partial + _merge below.
 * The KV range is split over CTAs and the
 * splits merged as kernels/logsum_merge.mojo does; out bf16 [T][num_q *
 * head_dim], in the rotated domain as the reference's.  The signed int8 dot
 * needs no qi_bias.  max_kv_len bounds the KV length of any token (sizes the
 * split count); workspace of gm_bq_attention_workspace_bytes. */
int gm_bq_attention_decode(const int8_t* q_i8, const float* f_q, const int8_t* k_cache,
                           const float* k_scale, const int8_t* v_cache, const float* v_scale,
                           const gm_kv_run_t* runs, const int32_t* base_rows, int T, int head_dim,
                           int num_q, int num_kv, int window, int cache_degree, int rank,
                           int page_shift, int row_mask, int page_mask, int max_kv_len, void* out,
                           float* workspace, size_t workspace_bytes, void* stream);
size_t gm_bq_attention_workspace_bytes(int T, int head_dim, int num_q, int num_kv, int max_kv_len);

/* The prefill path of the same dispatchers (attention.mojo:150-332
 * BqFlashPrefillSliding / BqFlashPrefillFull at cache_degree 1): runs as
 * gm_bq_attn_prep takes them (num_runs runs in buf_start order, a run's
 * tokens at consecutive positions from base_pos), every token attending to
 * its own causal range of its run -- sliding (window > 0): the last
 * min(pos+1, window) positions, full (window = 0): 0..pos -- in the cache the
 * prep has written.  Each CTA serves a tile of consecutive tokens, so one K/V
 * row read is shared by the tile's tokens and the GQA group's heads.  The
 * Gemma-4 geometries only: head_dim 256 with num_q = 2*num_kv (sliding) and
 * head_dim 512 with num_q = 8*num_kv (full).  out bf16 [T][num_q*head_dim]
 * (same tolerance to the reference as the decode: the accumulation order of
 * its tiles is not the reference's).  No workspace. */
int gm_bq_attention_prefill(const int8_t* q_i8, const float* f_q, const int8_t* k_cache,
                            const float* k_scale, const int8_t* v_cache, const float* v_scale,
                            const gm_kv_run_t* runs, int num_runs, const int32_t* base_rows, int T,
                            int head_dim, int num_q, int num_kv, int window, int page_shift, int row_mask,
                            int page_mask, void* out, void* stream);

/* A full-layer cache sharded by position over cache_degree ranks (the
 * reference's full attention at degree > 1, attention.mojo:236-332 with
 * kernels/logsum_merge.mojo:29-117): gm_bq_attention_partial computes, on one
 * rank, every token's attention over the positions this rank holds
 * (pos % cache_degree == rank, at cache row pos / cache_degree) and writes
 * the unnormalised log-sum partial per (token, head): partial f32
 * [T][num_q][head_dim + 2] = (m, l, acc[head_dim]) of
 * gm_bq_attention_partial_bytes(T, head_dim, num_q) bytes (arguments as
 * gm_bq_attention_decode; window must be 0 when cache_degree > 1).
 * gm_bq_attention_merge merges n_parts such partials (host array of device
 * pointers, rank order; a peer GPU's buffer may be passed where peer access
 * is enabled) with the reference's max-rescaled sums and writes
 * bf16(acc / l) [T][num_q * head_dim] (0 where no rank had a position). */
size_t gm_bq_attention_partial_bytes(int T, int head_dim, int num_q);
int gm_bq_attention_partial(const int8_t* q_i8, const float* f_q, const int8_t* k_cache,
                            const float* k_scale, const int8_t* v_cache, const float* v_scale,
                            const gm_kv_run_t* runs, const int32_t* base_rows, int T, int head_dim,
                            int num_q, int num_kv, int window, int cache_degree, int rank, int page_shift,
                            int row_mask, int page_mask, int max_kv_len, float* partial,
                            float* workspace, size_t workspace_bytes, void* stream);
int gm_bq_attention_merge(const float* const* partials, int n_parts, int T, int num_q, int head_dim, void* out,
                          void* stream);

/* butterquant/vnni.mojo:31-83 pack (and its inverse). rows%32 == 0, cols%64 == 0. */
int gm_vnni_pack(const int8_t* q, long rows, int cols, int8_t* packed, void* stream);
int gm_vnni_unpack(const int8_t* packed, long rows, int cols, int8_t* q, void* stream);

/* butterquant/kernels.mojo:218-224 router_center_softmax: out = bf16(W - mean_rows(W)). */
int gm_router_center(const void* w, int rows, int cols, void* out, void* stream);

/* butterquant/kernels.mojo:37-45 bake_split_gain_in_place (out may equal g). */
int gm_bake_split_gain(const void* g, void* out, int n, void* stream);

/* modeling/gemma4_topology.mojo:362-388 router scale bake: out = bf16(s/sqrt(2816)). */
int gm_bake_router_scale(const void* s, void* out, int n, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* GMOE_H */
