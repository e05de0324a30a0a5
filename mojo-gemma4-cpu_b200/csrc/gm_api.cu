// gm_api.cu -- the C ABI of include/gmoe.h: handle, weight registration, the
// MoE operator and the per-stage entry points.
#include <chrono>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "../../include/gmoe.h"
#include "ep.h"
#include "gm_kernels.h"

using namespace gm;

namespace {

thread_local std::string g_tls_error;

struct Layer {
  int kind = 0;  // 0 empty, 1 butterquant, 2 bf16
  int8_t* gu_q = nullptr;      // bq: VNNI-packed [epr*GU][H]
  float* gu_scale = nullptr;   // bq: [epr*GU]
  int8_t* dn_q = nullptr;      // bq: VNNI-packed [epr*H][I]
  float* dn_scale = nullptr;   // bq: [epr*H]
  uint16_t* gu_bf16 = nullptr;  // bf16: [epr][GU][H]
  uint16_t* dn_bf16 = nullptr;  // bf16: [epr][H][I]
  uint16_t* router = nullptr;   // [E][H]
  uint16_t* rscale = nullptr;   // [H]
  uint16_t* pes = nullptr;      // [E]
  uint16_t* gamma2 = nullptr;   // [H]
  int8_t* gu_rm = nullptr;      // bq: row-major copies for the tcgen05 prefill path
  int8_t* dn_rm = nullptr;
  // TMA descriptors of the tcgen05 prefill path: butterquant, over the
  // row-major int8 copies gu_rm (64-row boxes) / dn_rm (128-row boxes); bf16,
  // over the registered gate_up (64-row boxes) / down (128-row boxes)
  alignas(64) unsigned char tmap_gu[128] = {};
  alignas(64) unsigned char tmap_dn[128] = {};
  bool has_tc = false;
  // post-MoE tail (gm_moe_register_post)
  uint16_t* post_w1 = nullptr;  // post_feedforward_layernorm_1 [H]
  uint16_t* post_w2 = nullptr;  // post_feedforward_layernorm_2 [H]
  uint16_t* post_w = nullptr;   // post_feedforward_layernorm [H]
  float layer_scalar = 1.0f;
  // dense butterquant MLP (gm_moe_register_dense_bq), VNNI-packed
  int8_t* dg_q = nullptr;       // gate_proj [2112][H]
  float* dg_scale = nullptr;
  int8_t* du_q = nullptr;       // up_proj [2112][H]
  float* du_scale = nullptr;
  int8_t* dd_q = nullptr;       // down_proj [H][2112]
  float* dd_scale = nullptr;
  uint16_t* dgamma = nullptr;   // pre_feedforward_layernorm, split-gain baked
  // row-major copies for the dense tcgen05 path: gate rows then up rows, and
  // their scales in the same order; down
  int8_t* dgu_rm = nullptr;     // [4224][H]
  float* dgu_scale = nullptr;   // [4224]
  int8_t* dd_rm = nullptr;      // [H][2112]
  alignas(64) unsigned char tmap_dgu[128] = {};
  alignas(64) unsigned char tmap_ddn[128] = {};
  bool has_dense_tc = false;
};

}  // namespace

struct gm_moe {
  int device = 0, max_tokens = 0, num_layers = 0, rank = 0, degree = 1;
  int expert_base = 0, epr = E;
  std::vector<Layer> layers;
  std::string err;
  // workspace (one allocation, carved)
  void* ws = nullptr;
  size_t ws_bytes = 0;
  float* logits = nullptr;
  float* inv_rms = nullptr;
  int32_t* route_idx = nullptr;
  float* route_w = nullptr;
  int32_t* route_pos = nullptr;
  int32_t* expert_offset = nullptr;
  int32_t* chunk_off = nullptr;
  SparseRoute* routes = nullptr;
  int8_t* x_i8 = nullptr;
  float* x_sa = nullptr;
  uint16_t* x_normed = nullptr;
  uint16_t* bucket = nullptr;
  int8_t* bucket_i8 = nullptr;
  float* bucket_sa = nullptr;
  float* ybuf = nullptr;
  uint16_t* x_stage = nullptr;
  uint16_t* out_stage = nullptr;
  int8_t* xg = nullptr;         // routed activation rows in schedule order (tcgen05 A operand)
  float* xg_sa = nullptr;
  int* dev_err = nullptr;       // device-side error word (bounded waits that expired)
  int32_t* sched_counts = nullptr;  // per-chunk expert counts of the multi-CTA schedule
  int* router_counts = nullptr;     // router tile counters (zero between calls)
  alignas(64) unsigned char tmap_xg[128] = {};
  alignas(64) unsigned char tmap_bucket[128] = {};
  alignas(64) unsigned char tmap_y[128] = {};        // f32 route rows (TMA stores of the down product)
  alignas(64) unsigned char tmap_xgb[128] = {};      // bf16 gathered rows (in ybuf's memory)
  alignas(64) unsigned char tmap_bucketb[128] = {};  // bf16 bucket
  bool tc_ok = false;           // TMA descriptors available
  bool tcb_ok = false;
  int tc_min_tokens = 1024;     // GM_OPT_TC_MIN_TOKENS
  cudaStream_t own_stream = nullptr;
  cudaStream_t side_stream = nullptr;  // L2 prefetches forked off the forward's stream
  cudaEvent_t fork_event = nullptr;
  cudaEvent_t side_done = nullptr;   // joins the side stream back under stream capture
  // dense MLP of gm_ffn_forward, forked off the forward's stream and joined
  // before the post-MoE tail
  cudaStream_t dense_stream = nullptr;
  cudaEvent_t dense_fork = nullptr, dense_done = nullptr;
  bool dense_pending = false;
  int8_t* d_xi8 = nullptr;      // [T][H]
  float* d_xsa = nullptr;       // [T]
  float* d_inv = nullptr;       // [T]
  int8_t* d_hi8 = nullptr;      // [T][2112]
  float* d_hsa = nullptr;       // [T][33]
  uint16_t* d_out = nullptr;    // [T][H] dense_out
  alignas(64) unsigned char tmap_dx[128] = {};  // over d_xi8 (tcgen05 A operand)
  alignas(64) unsigned char tmap_dh[128] = {};  // over d_hi8
  bool dense_tc_ok = false;
  int dense_tc_min = 128;       // GM_OPT_DENSE_TC_MIN_TOKENS
  // stage profiler (GM_OPT_PROFILE) and kernel launch count
  struct PendingStage {
    int stat;
    long kernels;
    cudaEvent_t a, b;
  };
  bool profile = false;
  bool pdl = true;              // GM_OPT_PDL
  long launches = 0;
  std::vector<PendingStage> pending;
  std::vector<cudaEvent_t> event_pool;
  std::vector<gm_stage_stat_t> stats;
  // expert parallelism (gm_moe_ep_init): NCCL communicator and exchange buffers
  int ws_tokens = 0;            // activation rows the workspace holds
  ncclComm_t ep_comm = nullptr;
  void* ep_buf = nullptr;
  int32_t* ep_pos = nullptr;    // [max_tokens][degree]
  int32_t* ep_count = nullptr;  // [degree]
  uint8_t* ep_send_x = nullptr; // [degree*max_tokens][2*H] (int8 rows use the first H bytes)
  float* ep_send_sa = nullptr;
  int32_t* ep_send_idx = nullptr;
  float* ep_send_w = nullptr;
  uint8_t* ep_recv_x = nullptr;
  float* ep_recv_sa = nullptr;
  int32_t* ep_recv_idx = nullptr;
  float* ep_recv_w = nullptr;
  uint16_t* ep_partial = nullptr;  // [degree*max_tokens][H]
  uint16_t* ep_contrib = nullptr;
  int32_t* ep_rank_of = nullptr;   // [E] placement tables (device), used once placed
  int32_t* ep_local_of = nullptr;
  bool ep_placed = false;          // gm_moe_ep_set_placement done
  // peer-memory exchange (GM_OPT_EP_TRANSPORT 1): receive and contrib regions
  // in two parities, flags written by the peers, the exchange allocation of
  // every rank mapped into this process, the forward counter
  bool ep_p2p_ok = false;          // peers mapped
  bool ep_use_p2p = false;         // transport chosen
  EpPeers ep_peers[2];             // per parity
  uint32_t* ep_dflag = nullptr;    // [8] this rank's dispatch flags (slot per source)
  uint32_t* ep_cflag = nullptr;    // [8] combine flags
  int* ep_counters = nullptr;      // [2] last-CTA counters of the pack and the combine
  void* ep_peer_base[8] = {};      // IPC mappings (own base at this rank's index)
  uint32_t ep_epoch = 0;
  uint32_t ep_cur = 0;             // epoch of the forward whose phases are being issued
  bool ep_on = false;              // expert-parallel forward (either kind of group)
  // in-process group (gm_moe_ep_init_group): every member by rank; the peers'
  // exchange buffers are plain pointers of this process, no NCCL communicator
  bool ep_group = false;
  gm_moe* ep_members[8] = {};
  int ep_timeout_ms = 1000;        // GM_OPT_EP_TIMEOUT_MS: bound of each exchange wait
  int ep_init_timeout_ms = 120000; // GM_OPT_EP_INIT_TIMEOUT_MS: bound of gm_moe_ep_init
};

namespace {

constexpr int L2_PREFETCH_EXPERTS = 30;  // 30 x 3.97 MB of gate/up weights (L2 is 126 MB)

int set_err(gm_moe* h, int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  if (h) h->err = buf;
  g_tls_error = buf;
  return code;
}

int cuda_check(gm_moe* h, cudaError_t e, const char* what) {
  if (e == cudaSuccess) return GM_OK;
  return set_err(h, e == cudaErrorMemoryAllocation ? GM_ENOMEM : GM_ECUDA, "%s: %s", what,
                 cudaGetErrorString(e));
}

#define GM_TRY(h, expr, what)                         \
  do {                                                \
    int _rc = cuda_check((h), (expr), (what));        \
    if (_rc != GM_OK) return _rc;                     \
  } while (0)

inline cudaStream_t S(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// One stage of gm_moe_forward: its launches are counted and, with profiling
// on, timed under the label (StageScope below).
#define GM_STAGE(h, s, expr, what)              \
  do {                                          \
    StageScope _scope((h), (what), (s));        \
    GM_TRY((h), (expr), (what));                \
  } while (0)

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

struct Carve {
  size_t off = 0;
  template <typename T>
  size_t take(size_t count) {
    off = align_up(off, 256);
    size_t o = off;
    off += count * sizeof(T);
    return o;
  }
};

struct WsLayout {
  size_t logits, inv_rms, route_idx, route_w, route_pos, expert_offset, chunk_off, routes, x_i8, x_sa,
      x_normed, bucket, bucket_i8, bucket_sa, ybuf, x_stage, out_stage, xg, xg_sa, dev_err,
      sched_counts, router_counts, d_xi8, d_xsa, d_inv, d_hi8, d_hsa, d_out, total;
};

WsLayout ws_layout(int max_tokens) {
  const size_t T = (size_t)max_tokens, R = T * TOPK;
  Carve c;
  WsLayout L;
  const int m1 = std::min(max_tokens, 64), m2 = std::min(max_tokens, 1024);
  L.logits = c.take<float>(std::max({router_workspace_floats(m1), router_workspace_floats(m2),
                                     router_workspace_floats(max_tokens)}));
  L.inv_rms = c.take<float>(T);
  L.route_idx = c.take<int32_t>(R);
  L.route_w = c.take<float>(R);
  L.route_pos = c.take<int32_t>(R);
  L.expert_offset = c.take<int32_t>(E + 1);
  L.chunk_off = c.take<int32_t>(E + 1);
  L.routes = c.take<SparseRoute>(R);
  L.x_i8 = c.take<int8_t>(T * H);
  L.x_sa = c.take<float>(T);
  L.x_normed = c.take<uint16_t>(T * H);
  L.bucket = c.take<uint16_t>(R * I);
  L.bucket_i8 = c.take<int8_t>(R * I);
  L.bucket_sa = c.take<float>(R * NB_DOWN);
  L.ybuf = c.take<float>(R * H);
  L.x_stage = c.take<uint16_t>(T * H);
  L.out_stage = c.take<uint16_t>(T * H);
  L.xg = c.take<int8_t>(R * H);
  L.xg_sa = c.take<float>(R);
  L.dev_err = c.take<int>(1);
  L.sched_counts = c.take<int32_t>(schedule_counts_ints(max_tokens));
  L.router_counts = c.take<int>(router_tile_counters(max_tokens));
  L.d_xi8 = c.take<int8_t>(T * H);
  L.d_xsa = c.take<float>(T);
  L.d_inv = c.take<float>(T);
  L.d_hi8 = c.take<int8_t>(T * DENSE_I);
  L.d_hsa = c.take<float>(T * NB_DENSE);
  L.d_out = c.take<uint16_t>(T * H);
  L.total = align_up(c.off, 256);
  return L;
}

template <typename T>
int dev_copy(gm_moe* h, T** dst, const void* src, size_t count, const char* what) {
  if (!src) return set_err(h, GM_EINVAL, "%s: NULL pointer", what);
  if (*dst) {
    cudaFree(*dst);
    *dst = nullptr;
  }
  GM_TRY(h, cudaMalloc(reinterpret_cast<void**>(dst), count * sizeof(T)), what);
  GM_TRY(h, cudaMemcpy(*dst, src, count * sizeof(T), cudaMemcpyDefault), what);
  return GM_OK;
}

void free_layer(Layer& L) {
  void* ptrs[] = {L.gu_q, L.gu_scale, L.dn_q, L.dn_scale, L.gu_bf16, L.dn_bf16, L.router, L.rscale,
                  L.pes, L.gamma2, L.gu_rm, L.dn_rm, L.post_w1, L.post_w2, L.post_w,
                  L.dg_q, L.dg_scale, L.du_q, L.du_scale, L.dd_q, L.dd_scale, L.dgamma,
                  L.dgu_rm, L.dgu_scale, L.dd_rm};
  for (void* p : ptrs)
    if (p) cudaFree(p);
  L = Layer{};
}

// Frees a layer's expert weights only: the post-MoE gains and the dense MLP
// stay registered across a re-registration of the experts.
void free_moe(Layer& L) {
  Layer keep;
  keep.post_w1 = L.post_w1; keep.post_w2 = L.post_w2; keep.post_w = L.post_w;
  keep.layer_scalar = L.layer_scalar;
  keep.dg_q = L.dg_q; keep.dg_scale = L.dg_scale; keep.du_q = L.du_q; keep.du_scale = L.du_scale;
  keep.dd_q = L.dd_q; keep.dd_scale = L.dd_scale; keep.dgamma = L.dgamma;
  keep.dgu_rm = L.dgu_rm; keep.dgu_scale = L.dgu_scale; keep.dd_rm = L.dd_rm;
  memcpy(keep.tmap_dgu, L.tmap_dgu, sizeof keep.tmap_dgu);
  memcpy(keep.tmap_ddn, L.tmap_ddn, sizeof keep.tmap_ddn);
  keep.has_dense_tc = L.has_dense_tc;
  L.post_w1 = L.post_w2 = L.post_w = nullptr;
  L.dg_q = L.du_q = L.dd_q = nullptr;
  L.dg_scale = L.du_scale = L.dd_scale = nullptr;
  L.dgamma = nullptr;
  L.dgu_rm = L.dd_rm = nullptr;
  L.dgu_scale = nullptr;
  free_layer(L);
  L = keep;
}

int check_layer(gm_moe* h, int layer) {
  if (!h) return set_err(nullptr, GM_EINVAL, "NULL handle");
  if (layer < 0 || layer >= h->num_layers)
    return set_err(h, GM_EINVAL, "layer %d out of range [0,%d)", layer, h->num_layers);
  return GM_OK;
}

bool is_device_ptr(const void* p) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

// The device address of page-locked host memory mapped into the device's
// address space (cudaHostAlloc / pinned tensors), NULL for device, pageable or
// unmapped memory.
void* mapped_host_ptr(void* p) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  return a.type == cudaMemoryTypeHost ? a.devicePointer : nullptr;
}

// (Re)allocates the workspace for `tokens` activation rows and carves it.
int carve_workspace(gm_moe* h, int tokens) {
  if (h->ws) {
    cudaFree(h->ws);
    h->ws = nullptr;
  }
  WsLayout L = ws_layout(tokens);
  cudaError_t e = cudaMalloc(&h->ws, L.total);
  if (e != cudaSuccess) {
    h->ws = nullptr;
    return set_err(h, GM_ENOMEM, "workspace of %zu bytes: %s", L.total, cudaGetErrorString(e));
  }
  h->ws_bytes = L.total;
  h->ws_tokens = tokens;
  char* b = static_cast<char*>(h->ws);
  h->logits = reinterpret_cast<float*>(b + L.logits);
  h->inv_rms = reinterpret_cast<float*>(b + L.inv_rms);
  h->route_idx = reinterpret_cast<int32_t*>(b + L.route_idx);
  h->route_w = reinterpret_cast<float*>(b + L.route_w);
  h->route_pos = reinterpret_cast<int32_t*>(b + L.route_pos);
  h->expert_offset = reinterpret_cast<int32_t*>(b + L.expert_offset);
  h->chunk_off = reinterpret_cast<int32_t*>(b + L.chunk_off);
  h->routes = reinterpret_cast<SparseRoute*>(b + L.routes);
  h->x_i8 = reinterpret_cast<int8_t*>(b + L.x_i8);
  h->x_sa = reinterpret_cast<float*>(b + L.x_sa);
  h->x_normed = reinterpret_cast<uint16_t*>(b + L.x_normed);
  h->bucket = reinterpret_cast<uint16_t*>(b + L.bucket);
  h->bucket_i8 = reinterpret_cast<int8_t*>(b + L.bucket_i8);
  h->bucket_sa = reinterpret_cast<float*>(b + L.bucket_sa);
  h->ybuf = reinterpret_cast<float*>(b + L.ybuf);
  h->x_stage = reinterpret_cast<uint16_t*>(b + L.x_stage);
  h->out_stage = reinterpret_cast<uint16_t*>(b + L.out_stage);
  h->xg = reinterpret_cast<int8_t*>(b + L.xg);
  h->xg_sa = reinterpret_cast<float*>(b + L.xg_sa);
  h->dev_err = reinterpret_cast<int*>(b + L.dev_err);
  h->sched_counts = reinterpret_cast<int32_t*>(b + L.sched_counts);
  h->router_counts = reinterpret_cast<int*>(b + L.router_counts);
  h->d_xi8 = reinterpret_cast<int8_t*>(b + L.d_xi8);
  h->d_xsa = reinterpret_cast<float*>(b + L.d_xsa);
  h->d_inv = reinterpret_cast<float*>(b + L.d_inv);
  h->d_hi8 = reinterpret_cast<int8_t*>(b + L.d_hi8);
  h->d_hsa = reinterpret_cast<float*>(b + L.d_hsa);
  h->d_out = reinterpret_cast<uint16_t*>(b + L.d_out);
  h->dense_tc_ok = make_tmap_i8(h->tmap_dx, h->d_xi8, (long)tokens, H, 128) &&
                   make_tmap_i8(h->tmap_dh, h->d_hi8, (long)tokens, DENSE_I, 128);
  cudaMemset(h->dev_err, 0, sizeof(int));
  cudaMemset(h->router_counts, 0, sizeof(int) * router_tile_counters(tokens));
  h->tc_ok = make_tmap_i8(h->tmap_xg, h->xg, (long)tokens * TOPK, H, 128) &&
             make_tmap_i8(h->tmap_bucket, h->bucket_i8, (long)tokens * TOPK, I, 128) &&
             make_tmap_2d(h->tmap_y, h->ybuf, (long)tokens * TOPK, H, 4, 32);
  // bf16 prefill: the gathered activation rows live in ybuf, which is idle
  // until the down product writes it
  h->tcb_ok = make_tmap_2d(h->tmap_xgb, h->ybuf, (long)tokens * TOPK, H, 2, 128) &&
              make_tmap_2d(h->tmap_bucketb, h->bucket, (long)tokens * TOPK, I, 2, 128);
  return GM_OK;
}

// Exchange allocation of an expert-parallel handle: one cudaMalloc, the same
// offsets on every rank (same max_tokens and world), so a peer's buffer is
// its base plus these offsets.
struct EpLayout {
  size_t pos, cnt, sx, ssa, sidx, sw, rx, rsa, ridx, rw, part, con, rank, local;
  size_t rx1, rsa1, ridx1, rw1, con1;  // second parity of the regions peers write
  size_t dflag, cflag, ctr, total;
};

EpLayout ep_layout(int max_tokens, int world) {
  const size_t cap = (size_t)max_tokens, n = (size_t)world * cap;
  Carve c;
  EpLayout o;
  o.pos = c.take<int32_t>(cap * world);
  o.cnt = c.take<int32_t>(8);
  o.sx = c.take<uint8_t>(n * 2 * H);
  o.ssa = c.take<float>(n);
  o.sidx = c.take<int32_t>(n * TOPK);
  o.sw = c.take<float>(n * TOPK);
  o.rx = c.take<uint8_t>(n * 2 * H);
  o.rsa = c.take<float>(n);
  o.ridx = c.take<int32_t>(n * TOPK);
  o.rw = c.take<float>(n * TOPK);
  o.part = c.take<uint16_t>(n * H);
  o.con = c.take<uint16_t>(n * H);
  o.rank = c.take<int32_t>(E);
  o.local = c.take<int32_t>(E);
  o.rx1 = c.take<uint8_t>(n * 2 * H);
  o.rsa1 = c.take<float>(n);
  o.ridx1 = c.take<int32_t>(n * TOPK);
  o.rw1 = c.take<float>(n * TOPK);
  o.con1 = c.take<uint16_t>(n * H);
  o.dflag = c.take<uint32_t>(8);
  o.cflag = c.take<uint32_t>(8);
  o.ctr = c.take<int>(2);
  o.total = align_up(c.off, 256);
  return o;
}

// Workspace for world*max_tokens received rows plus the exchange allocation
// (zeroed: flags at epoch 0, counters re-armed), carved into the handle.
int ep_alloc(gm_moe* h, int world, EpLayout* out) {
  int rc = carve_workspace(h, world * h->max_tokens);
  if (rc) return rc;
  const EpLayout o = ep_layout(h->max_tokens, world);
  GM_TRY(h, cudaMalloc(&h->ep_buf, o.total), "ep buffers");
  GM_TRY(h, cudaMemset(h->ep_buf, 0, o.total), "ep buffers");
  char* b = static_cast<char*>(h->ep_buf);
  h->ep_pos = reinterpret_cast<int32_t*>(b + o.pos);
  h->ep_count = reinterpret_cast<int32_t*>(b + o.cnt);
  h->ep_send_x = reinterpret_cast<uint8_t*>(b + o.sx);
  h->ep_send_sa = reinterpret_cast<float*>(b + o.ssa);
  h->ep_send_idx = reinterpret_cast<int32_t*>(b + o.sidx);
  h->ep_send_w = reinterpret_cast<float*>(b + o.sw);
  h->ep_recv_x = reinterpret_cast<uint8_t*>(b + o.rx);
  h->ep_recv_sa = reinterpret_cast<float*>(b + o.rsa);
  h->ep_recv_idx = reinterpret_cast<int32_t*>(b + o.ridx);
  h->ep_recv_w = reinterpret_cast<float*>(b + o.rw);
  h->ep_partial = reinterpret_cast<uint16_t*>(b + o.part);
  h->ep_contrib = reinterpret_cast<uint16_t*>(b + o.con);
  h->ep_rank_of = reinterpret_cast<int32_t*>(b + o.rank);
  h->ep_local_of = reinterpret_cast<int32_t*>(b + o.local);
  h->ep_dflag = reinterpret_cast<uint32_t*>(b + o.dflag);
  h->ep_cflag = reinterpret_cast<uint32_t*>(b + o.cflag);
  h->ep_counters = reinterpret_cast<int*>(b + o.ctr);
  *out = o;
  return GM_OK;
}

// Peer tables of both parities from every rank's exchange base (IPC mappings
// across processes, plain pointers inside one process).
void ep_wire(gm_moe* h, int world, void* const* bases, const EpLayout& o) {
  const size_t rx[2] = {o.rx, o.rx1}, rsa[2] = {o.rsa, o.rsa1}, ridx[2] = {o.ridx, o.ridx1},
               rw[2] = {o.rw, o.rw1}, con[2] = {o.con, o.con1};
  for (int par = 0; par < 2; ++par)
    for (int q = 0; q < world; ++q) {
      char* pb = static_cast<char*>(bases[q]);
      EpPeers& P = h->ep_peers[par];
      P.recv_x[q] = reinterpret_cast<uint8_t*>(pb + rx[par]);
      P.recv_sa[q] = reinterpret_cast<float*>(pb + rsa[par]);
      P.recv_idx[q] = reinterpret_cast<int32_t*>(pb + ridx[par]);
      P.recv_w[q] = reinterpret_cast<float*>(pb + rw[par]);
      P.contrib[q] = reinterpret_cast<uint16_t*>(pb + con[par]);
      P.dflag[q] = reinterpret_cast<uint32_t*>(pb + o.dflag);
      P.cflag[q] = reinterpret_cast<uint32_t*>(pb + o.cflag);
    }
}

// ---------------------------------------------------------------- profiler
cudaEvent_t take_event(gm_moe* h) {
  if (!h->event_pool.empty()) {
    cudaEvent_t e = h->event_pool.back();
    h->event_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  if (cudaEventCreate(&e) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  return e;
}

int stat_index(gm_moe* h, const char* label) {
  for (size_t i = 0; i < h->stats.size(); ++i)
    if (!strncmp(h->stats[i].label, label, sizeof(h->stats[i].label))) return (int)i;
  gm_stage_stat_t st = {};
  snprintf(st.label, sizeof st.label, "%s", label);
  st.min_ms = 1e300;
  h->stats.push_back(st);
  return (int)h->stats.size() - 1;
}

// Waits for every recorded stage and folds its duration into the statistics.
int drain_profile(gm_moe* h) {
  int rc = GM_OK;
  for (auto& p : h->pending) {
    float ms = 0.0f;
    cudaError_t e = cudaEventSynchronize(p.b);
    if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, p.a, p.b);
    if (e == cudaSuccess) {
      gm_stage_stat_t& st = h->stats[p.stat];
      st.calls += 1;
      st.kernels += p.kernels;
      st.total_ms += ms;
      st.min_ms = std::min(st.min_ms, (double)ms);
      st.max_ms = std::max(st.max_ms, (double)ms);
    } else if (rc == GM_OK) {
      rc = cuda_check(h, e, "profile event");
    }
    h->event_pool.push_back(p.a);
    h->event_pool.push_back(p.b);
  }
  h->pending.clear();
  return rc;
}

// Scope of one forward stage: counts the kernels launched inside it and, with
// GM_OPT_PROFILE on, brackets them with events on the forward's stream.
struct StageScope {
  gm_moe* h;
  const char* label;
  cudaStream_t s;
  cudaEvent_t a = nullptr;
  long n0;
  StageScope(gm_moe* h_, const char* label_, cudaStream_t s_)
      : h(h_), label(label_), s(s_), n0(tls_kernel_launches) {
    if (h->profile && (a = take_event(h)) && cudaEventRecord(a, s) != cudaSuccess) {
      cudaGetLastError();
      h->event_pool.push_back(a);
      a = nullptr;
    }
  }
  ~StageScope() {
    const long k = tls_kernel_launches - n0;
    h->launches += k;
    if (!a) return;
    cudaEvent_t b = take_event(h);
    if (b && cudaEventRecord(b, s) == cudaSuccess) {
      h->pending.push_back({stat_index(h, label), k, a, b});
    } else {
      cudaGetLastError();
      h->event_pool.push_back(a);
      if (b) h->event_pool.push_back(b);
    }
  }
};

// The post-MoE tail reads dense_out: wait for the dense MLP forked by
// gm_ffn_forward (no-op otherwise).
int join_dense(gm_moe* h, cudaStream_t s) {
  if (!h->dense_pending) return GM_OK;
  h->dense_pending = false;
  return cuda_check(h, cudaStreamWaitEvent(s, h->dense_done, 0), "dense join");
}

// Where experts_and_combine puts each row's finished MoE value: a local bf16
// output, the post-MoE tail (x_main updated in place), or -- expert-parallel
// forward over peer memory -- the partial row stored into its source rank's
// contribution block, followed by the combine flags.
struct CombineTarget {
  uint16_t* out = nullptr;
  const PostParams* post = nullptr;
  const EpPeers* peers = nullptr;
  uint32_t epoch = 0;
};

// Expert products and combine for Tn activation rows whose schedule
// (expert_offset, routes, route_pos, chunk_off) is in the workspace: rows are
// x_i8/x_sa (butterquant) or x_normed (bf16), route_idx their top-8.
int experts_and_combine(gm_moe* h, const Layer& L, int Tn, const int8_t* x_i8, const float* x_sa,
                        const uint16_t* x_normed, const int32_t* route_idx, const CombineTarget& ct,
                        cudaStream_t s, bool rows_gathered = false) {
  if (L.kind == 1) {
    if (L.has_tc && h->tc_ok && Tn >= h->tc_min_tokens) {
      // prefill: routed rows in schedule order (already there when the norm
      // kernel wrote them itself), then the tcgen05 GEMMs
      if (!rows_gathered)
        GM_STAGE(h, s, launch_gather_rows(x_i8, H, x_sa, h->routes, h->expert_offset, h->epr, Tn, h->xg,
                                          h->xg_sa, s),
                 "gather_rows");
      GM_STAGE(h, s, launch_tc_phase1(h->tmap_xg, L.tmap_gu, h->expert_offset, h->epr, Tn, h->xg_sa,
                                      L.gu_scale, h->bucket_i8, h->bucket_sa, nullptr, h->dev_err, s),
               "bq_phase1_gate_up.tc");
      GM_STAGE(h, s, launch_tc_phase2(h->tmap_bucket, L.tmap_dn, h->tmap_y, h->expert_offset, h->epr, Tn,
                                      h->bucket_sa, h->routes, L.dn_scale, h->ybuf, h->dev_err, s),
               "bq_phase2_down.tc");
    } else {
      GM_STAGE(h, s, launch_bq_phase1(x_i8, x_sa, h->expert_offset, h->routes, h->chunk_off, h->epr,
                                      Tn, L.gu_q, L.gu_scale, h->bucket_i8, h->bucket_sa, nullptr, s),
               "bq_phase1_gate_up");
      GM_STAGE(h, s, launch_bq_phase2(h->bucket_i8, h->bucket_sa, h->expert_offset, h->routes,
                                      h->chunk_off, h->epr, Tn, L.dn_q, L.dn_scale, h->ybuf, true, s),
               "bq_phase2_down");
    }
  } else if (L.has_tc && h->tcb_ok && Tn >= h->tc_min_tokens) {
    if (!rows_gathered)
      GM_STAGE(h, s, launch_gather_rows(x_normed, 2 * H, nullptr, h->routes, h->expert_offset, h->epr, Tn,
                                        h->ybuf, nullptr, s),
               "gather_rows");
    GM_STAGE(h, s, launch_tcb_phase1(h->tmap_xgb, L.tmap_gu, h->expert_offset, h->epr, Tn, h->bucket,
                                     h->dev_err, s),
             "phase1_gate_up.tc");
    GM_STAGE(h, s, launch_tcb_phase2(h->tmap_bucketb, L.tmap_dn, h->expert_offset, h->epr, Tn, h->routes,
                                     h->ybuf, h->dev_err, s),
             "phase2_down.tc");
  } else {
    GM_STAGE(h, s, launch_bf16_phase1(x_normed, h->expert_offset, h->routes, h->chunk_off, h->epr, Tn,
                                      L.gu_bf16, h->bucket, s),
             "phase1_gate_up");
    GM_STAGE(h, s, launch_bf16_phase2(h->bucket, h->expert_offset, h->routes, h->chunk_off, h->epr, Tn,
                                      L.dn_bf16, h->ybuf, s),
             "phase2_down");
  }
  if (ct.peers) {
    GM_STAGE(h, s, launch_combine_p2p(route_idx, h->route_pos, h->ybuf, Tn, h->max_tokens, *ct.peers,
                                      h->degree, h->rank, ct.epoch, h->ep_counters + 1, s),
             "combine.p2p");
    return GM_OK;
  }
  if (ct.post && join_dense(h, s)) return GM_ECUDA;
  if (ct.post)
    GM_STAGE(h, s, launch_combine_post(route_idx, h->route_pos, h->ybuf, Tn, *ct.post, s), "combine.post");
  else
    GM_STAGE(h, s, launch_combine(route_idx, h->route_pos, h->ybuf, Tn, ct.out, s), "combine");
  return GM_OK;
}

// With a non-blocking communicator every NCCL call may return
// ncclInProgress; the call is complete once the communicator's state leaves
// that value (polled for at most `limit_ms`).
ncclResult_t nccl_settle(ncclComm_t comm, ncclResult_t r, int limit_ms) {
  if (r != ncclInProgress || !comm) return r;
  const NcclApi* nc = nccl_api(nullptr);
  const auto t0 = std::chrono::steady_clock::now();
  ncclResult_t st = ncclInProgress;
  while (nc->comm_get_async_error(comm, &st) == ncclSuccess && st == ncclInProgress) {
    if (std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(limit_ms)) return ncclInProgress;
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
  return st;
}

int nccl_check(gm_moe* h, ncclResult_t r, const char* what) {
  r = nccl_settle(h ? h->ep_comm : nullptr, r, 60000);
  if (r == ncclSuccess) return GM_OK;
  if (r == ncclInProgress) return set_err(h, GM_ETIMEOUT, "%s: NCCL call did not complete in 60 s", what);
  const NcclApi* nc = nccl_api(nullptr);
  return set_err(h, GM_ENCCL, "%s: %s", what, nc ? nc->get_error_string(r) : "NCCL error");
}

#define GM_NCCL(h, expr, what)                         \
  do {                                                 \
    int _rc = nccl_check((h), (expr), (what));         \
    if (_rc != GM_OK) return _rc;                      \
  } while (0)

// A member of an in-process group whose peer was destroyed has no exchange.
int ep_group_intact(gm_moe* h) {
  if (!h->ep_group) return GM_OK;
  for (int q = 0; q < h->degree; ++q)
    if (!h->ep_members[q])
      return set_err(h, GM_ESTATE, "member %d of this handle's expert-parallel group was destroyed", q);
  return GM_OK;
}

uint64_t ep_limit_ns(const gm_moe* h) { return (uint64_t)h->ep_timeout_ms * 1000000ull; }

EpPlacement ep_placement(const gm_moe* h) {
  EpPlacement pl;
  if (h->ep_placed) {
    pl.rank_of = h->ep_rank_of;
    pl.local_of = h->ep_local_of;
  }
  return pl;
}

// Expert-parallel forward in three phases, so that an in-process group can
// issue each phase for every member before the next one (the waits of phase
// B and C then find their flags already published, see
// gm_moe_ep_forward_group).  A one-handle-per-process forward runs A, B, C.
//
// Phase A: local activation prep, router logits and top-8 of this rank's T
// tokens, the destination plan and, with the peer-memory transport, the pack
// that stores each row into its receivers' buffers.
int ep_phase_a(gm_moe* h, const Layer& L, const uint16_t* xb, int T, cudaStream_t s) {
  const int G = h->degree, cap = h->max_tokens;
  const bool bq = L.kind == 1;
  if (T > 0) {
    if (bq)
      GM_STAGE(h, s, launch_bq_norm_quant(xb, L.gamma2, T, h->x_i8, h->x_sa, h->inv_rms, s), "bq_norm_quant");
    else
      GM_STAGE(h, s, launch_rms_norm_bf16(xb, L.gamma2, T, h->x_normed, h->inv_rms, s), "rms_norm");
    GM_STAGE(h, s, launch_router_logits(xb, L.router, L.rscale, T, h->logits, h->dev_err, h->router_counts, s),
             "router_expert");
    GM_STAGE(h, s, launch_topk(h->logits, L.pes, h->inv_rms, T, h->route_idx, h->route_w, s), "router_merge");
  }
  const EpPlacement pl = ep_placement(h);
  GM_STAGE(h, s, launch_ep_plan(h->route_idx, T, G, h->epr, pl, h->ep_pos, h->ep_count, s), "ep_plan");
  if (!h->ep_use_p2p) return GM_OK;
  h->ep_cur = ++h->ep_epoch;
  const EpPeers& P = h->ep_peers[h->ep_cur & 1];
  GM_STAGE(h, s, launch_ep_pack_p2p(bq ? static_cast<const void*>(h->x_i8) : static_cast<const void*>(h->x_normed),
                                    bq ? H : 2 * H, bq ? h->x_sa : nullptr, h->route_idx, h->route_w, T, G, cap,
                                    h->epr, pl, h->ep_pos, h->ep_count, P, h->rank, h->ep_cur,
                                    h->ep_counters, s),
           "ep_pack.p2p");
  return GM_OK;
}

// Phase B (peer memory): wait until every source stored its rows here, run
// this rank's experts over them, and store each row's partial into its
// source's contribution block.
int ep_phase_b(gm_moe* h, const Layer& L, cudaStream_t s) {
  const int G = h->degree, cap = h->max_tokens, n = G * cap;
  const bool bq = L.kind == 1;
  const EpPeers& P = h->ep_peers[h->ep_cur & 1];
  GM_STAGE(h, s, launch_ep_wait(h->ep_dflag, G, h->ep_cur, ep_limit_ns(h), h->dev_err, s), "ep_dispatch.wait");
  const uint8_t* rx = P.recv_x[h->rank];
  const int32_t* ridx = P.recv_idx[h->rank];
  const int rc_chunk = bq ? GM_ROUTE_CHUNK_BQ : GM_ROUTE_CHUNK_BF16;
  if (n <= 1024)
    GM_STAGE(h, s, launch_build_schedule(ridx, P.recv_w[h->rank], n, h->expert_base, h->epr, rc_chunk,
                                         h->expert_offset, h->routes, h->route_pos, h->chunk_off, s),
             "ep_schedule");
  else
    GM_STAGE(h, s, launch_schedule_multi(ridx, P.recv_w[h->rank], n, h->expert_base, h->epr, rc_chunk,
                                         h->sched_counts, h->expert_offset, h->routes, h->route_pos,
                                         h->chunk_off, s),
             "ep_schedule");
  // the experts; each row's partial goes into its source's contribution block
  CombineTarget ct;
  ct.peers = &P;
  ct.epoch = h->ep_cur;
  return experts_and_combine(h, L, n, reinterpret_cast<const int8_t*>(rx), P.recv_sa[h->rank],
                             reinterpret_cast<const uint16_t*>(rx), ridx, ct, s);
}

// Phase C (peer memory): wait for every destination's partial rows, then sum
// them in rank order (and run the post-MoE tail when asked).
int ep_phase_c(gm_moe* h, uint16_t* out, int T, cudaStream_t s, const PostParams* post) {
  const int G = h->degree, cap = h->max_tokens;
  const EpPeers& P = h->ep_peers[h->ep_cur & 1];
  GM_STAGE(h, s, launch_ep_wait(h->ep_cflag, G, h->ep_cur, ep_limit_ns(h), h->dev_err, s), "ep_combine.wait");
  const uint16_t* contrib = P.contrib[h->rank];
  if (post && join_dense(h, s)) return GM_ECUDA;
  if (post)
    GM_STAGE(h, s, launch_ep_final_post(contrib, h->ep_pos, T, G, cap, *post, s), "ep_final.post");
  else
    GM_STAGE(h, s, launch_ep_final(contrib, h->ep_pos, T, G, cap, out, s), "ep_final");
  return GM_OK;
}

// Expert-parallel forward, NCCL transport (after phase A): send/recv of the
// packed blocks, the experts, send/recv of the partial rows, the rank-order sum.
int ep_forward_nccl(gm_moe* h, const Layer& L, uint16_t* out, int T, cudaStream_t s,
                    const PostParams* post) {
  const NcclApi* nc = nccl_api(nullptr);
  if (!h->ep_comm || !nc) return set_err(h, GM_ESTATE, "the NCCL transport needs gm_moe_ep_init");
  const int G = h->degree, cap = h->max_tokens, n = G * cap;
  const bool bq = L.kind == 1;
  const int row_bytes = bq ? H : 2 * H;
  const EpPlacement pl = ep_placement(h);
  GM_STAGE(h, s, launch_ep_pack(bq ? static_cast<const void*>(h->x_i8) : static_cast<const void*>(h->x_normed),
                                row_bytes, bq ? h->x_sa : nullptr, h->route_idx, h->route_w, T, G, cap,
                                h->epr, pl, h->ep_pos, h->ep_count, h->ep_send_x, h->ep_send_sa,
                                h->ep_send_idx, h->ep_send_w, s),
           "ep_pack");
  // dispatch: block p of every array goes to rank p
  {
    StageScope scope(h, "ep_dispatch", s);
    GM_NCCL(h, nc->group_start(), "ep dispatch");
    for (int p = 0; p < G; ++p) {
      const size_t r0 = (size_t)p * cap;
      GM_NCCL(h, nc->send(h->ep_send_x + r0 * row_bytes, (size_t)cap * row_bytes, ncclUint8, p, h->ep_comm, s), "send x");
      GM_NCCL(h, nc->recv(h->ep_recv_x + r0 * row_bytes, (size_t)cap * row_bytes, ncclUint8, p, h->ep_comm, s), "recv x");
      if (bq) {
        GM_NCCL(h, nc->send(h->ep_send_sa + r0, (size_t)cap, ncclFloat32, p, h->ep_comm, s), "send sa");
        GM_NCCL(h, nc->recv(h->ep_recv_sa + r0, (size_t)cap, ncclFloat32, p, h->ep_comm, s), "recv sa");
      }
      GM_NCCL(h, nc->send(h->ep_send_idx + r0 * TOPK, (size_t)cap * TOPK, ncclInt32, p, h->ep_comm, s), "send idx");
      GM_NCCL(h, nc->recv(h->ep_recv_idx + r0 * TOPK, (size_t)cap * TOPK, ncclInt32, p, h->ep_comm, s), "recv idx");
      GM_NCCL(h, nc->send(h->ep_send_w + r0 * TOPK, (size_t)cap * TOPK, ncclFloat32, p, h->ep_comm, s), "send w");
      GM_NCCL(h, nc->recv(h->ep_recv_w + r0 * TOPK, (size_t)cap * TOPK, ncclFloat32, p, h->ep_comm, s), "recv w");
    }
    GM_NCCL(h, nc->group_end(), "ep dispatch");
  }
  // this rank's experts over the n received rows (unused rows route nowhere)
  const int rc_chunk = bq ? GM_ROUTE_CHUNK_BQ : GM_ROUTE_CHUNK_BF16;
  if (n <= 1024)
    GM_STAGE(h, s, launch_build_schedule(h->ep_recv_idx, h->ep_recv_w, n, h->expert_base, h->epr, rc_chunk,
                                         h->expert_offset, h->routes, h->route_pos, h->chunk_off, s),
             "ep_schedule");
  else
    GM_STAGE(h, s, launch_schedule_multi(h->ep_recv_idx, h->ep_recv_w, n, h->expert_base, h->epr, rc_chunk,
                                         h->sched_counts, h->expert_offset, h->routes, h->route_pos,
                                         h->chunk_off, s),
             "ep_schedule");
  CombineTarget ct;
  ct.out = h->ep_partial;
  int rc = experts_and_combine(h, L, n, reinterpret_cast<const int8_t*>(h->ep_recv_x), h->ep_recv_sa,
                               reinterpret_cast<const uint16_t*>(h->ep_recv_x), h->ep_recv_idx, ct, s);
  if (rc) return rc;
  // combine exchange: partial rows go back to the rank they came from
  {
    StageScope scope(h, "ep_combine", s);
    GM_NCCL(h, nc->group_start(), "ep combine");
    for (int p = 0; p < G; ++p) {
      const size_t r0 = (size_t)p * cap * H;
      GM_NCCL(h, nc->send(h->ep_partial + r0, (size_t)cap * H, ncclBfloat16, p, h->ep_comm, s), "send partial");
      GM_NCCL(h, nc->recv(h->ep_contrib + r0, (size_t)cap * H, ncclBfloat16, p, h->ep_comm, s), "recv partial");
    }
    GM_NCCL(h, nc->group_end(), "ep combine");
  }
  // sum of the ranks' partials in rank order (then the post-MoE tail)
  if (post && join_dense(h, s)) return GM_ECUDA;
  if (post)
    GM_STAGE(h, s, launch_ep_final_post(h->ep_contrib, h->ep_pos, T, G, cap, *post, s), "ep_final.post");
  else
    GM_STAGE(h, s, launch_ep_final(h->ep_contrib, h->ep_pos, T, G, cap, out, s), "ep_final");
  return GM_OK;
}

// Expert-parallel forward of one handle (after gm_moe_ep_init or
// gm_moe_ep_init_group): this rank's T tokens in, their full MoE output out.
int ep_forward(gm_moe* h, const Layer& L, const uint16_t* xb, uint16_t* out, int T, cudaStream_t s,
               const PostParams* post) {
  int rc = ep_phase_a(h, L, xb, T, s);
  if (rc) return rc;
  if (!h->ep_use_p2p) return ep_forward_nccl(h, L, out, T, s, post);
  if ((rc = ep_phase_b(h, L, s))) return rc;
  return ep_phase_c(h, out, T, s, post);
}

}  // namespace

namespace gm {
void set_thread_error(const char* msg) { g_tls_error = msg; }

int handle_shard(const gm_moe* h, int* device, int* expert_base, int* epr, int* num_layers) {
  if (!h) return set_err(nullptr, GM_EINVAL, "NULL handle");
  *device = h->device;
  *expert_base = h->expert_base;
  *epr = h->epr;
  *num_layers = h->num_layers;
  return GM_OK;
}

int handle_fail(gm_moe* h, int code, const char* msg) { return set_err(h, code, "%s", msg); }
}  // namespace gm

extern "C" {

const char* gm_version(void) { return "gmoe 0.1 (sm_100a)"; }

const char* gm_last_error(const gm_moe_t* h) {
  return h ? h->err.c_str() : g_tls_error.c_str();
}

size_t gm_router_workspace_bytes(int T) {
  return T > 0 ? router_workspace_floats(T) * sizeof(float) : 0;
}

size_t gm_moe_workspace_bytes(int max_tokens) {
  return max_tokens > 0 ? ws_layout(max_tokens).total : 0;
}

int gm_moe_create(gm_moe_t** out, int device, int max_tokens, int num_layers, int rank,
                  int degree) {
  if (!out) return set_err(nullptr, GM_EINVAL, "gm_moe_create: NULL out");
  *out = nullptr;
  if (max_tokens <= 0 || num_layers <= 0)
    return set_err(nullptr, GM_EINVAL, "gm_moe_create: max_tokens=%d num_layers=%d", max_tokens,
                   num_layers);
  if (degree < 1 || E % degree || rank < 0 || rank >= degree)
    return set_err(nullptr, GM_EINVAL, "gm_moe_create: rank=%d degree=%d (degree must divide 128)",
                   rank, degree);
  if (cudaSetDevice(device) != cudaSuccess)
    return set_err(nullptr, GM_ECUDA, "gm_moe_create: cudaSetDevice(%d) failed", device);
  gm_moe* h = new gm_moe();
  h->device = device;
  h->max_tokens = max_tokens;
  h->num_layers = num_layers;
  h->rank = rank;
  h->degree = degree;
  h->epr = E / degree;
  h->expert_base = rank * h->epr;
  h->layers.resize(num_layers);
  int rc = carve_workspace(h, max_tokens);
  if (rc != GM_OK) {
    delete h;
    return rc;
  }
  if (cudaStreamCreateWithFlags(&h->side_stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaEventCreateWithFlags(&h->fork_event, cudaEventDisableTiming) != cudaSuccess ||
      cudaEventCreateWithFlags(&h->side_done, cudaEventDisableTiming) != cudaSuccess) {
    cudaGetLastError();
    h->side_stream = nullptr;  // prefetch disabled; everything else works
  }
  if (cudaStreamCreateWithFlags(&h->dense_stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaEventCreateWithFlags(&h->dense_fork, cudaEventDisableTiming) != cudaSuccess ||
      cudaEventCreateWithFlags(&h->dense_done, cudaEventDisableTiming) != cudaSuccess) {
    cudaGetLastError();
    h->dense_stream = nullptr;  // the dense MLP then runs on the forward's stream
  }
  if (cudaStreamCreateWithFlags(&h->own_stream, cudaStreamNonBlocking) != cudaSuccess) {
    cudaFree(h->ws);
    delete h;
    return set_err(nullptr, GM_ECUDA, "gm_moe_create: stream creation failed");
  }
  *out = h;
  return GM_OK;
}

int gm_moe_destroy(gm_moe_t* h) {
  if (!h) return GM_OK;
  cudaSetDevice(h->device);
  for (auto& L : h->layers) free_layer(L);
  drain_profile(h);
  for (cudaEvent_t e : h->event_pool) cudaEventDestroy(e);
  if (h->ep_comm) {
    cudaDeviceSynchronize();
    for (int q = 0; q < 8; ++q)
      if (h->ep_peer_base[q] && q != h->rank) cudaIpcCloseMemHandle(h->ep_peer_base[q]);
    if (const NcclApi* nc = nccl_api(nullptr)) nc->comm_destroy(h->ep_comm);
  }
  if (h->ep_group) {
    // no member may still be storing into this handle's exchange buffers, and
    // none may use them afterwards: the group is dissolved
    for (int q = 0; q < h->degree; ++q)
      if (gm_moe* m = h->ep_members[q]) {
        cudaSetDevice(m->device);
        cudaDeviceSynchronize();
      }
    for (int q = 0; q < h->degree; ++q)
      if (gm_moe* m = h->ep_members[q])
        if (m != h) m->ep_members[h->rank] = nullptr;
    cudaSetDevice(h->device);
  }
  if (h->ep_buf) cudaFree(h->ep_buf);
  if (h->ws) cudaFree(h->ws);
  if (h->own_stream) cudaStreamDestroy(h->own_stream);
  if (h->side_stream) cudaStreamDestroy(h->side_stream);
  if (h->fork_event) cudaEventDestroy(h->fork_event);
  if (h->side_done) cudaEventDestroy(h->side_done);
  if (h->dense_stream) cudaStreamDestroy(h->dense_stream);
  if (h->dense_fork) cudaEventDestroy(h->dense_fork);
  if (h->dense_done) cudaEventDestroy(h->dense_done);
  delete h;
  return GM_OK;
}

int gm_moe_register_layer_bq(gm_moe_t* h, int layer, const void* gate_up,
                             const float* gate_up_scale, const void* down,
                             const float* down_scale, const void* router_centered,
                             const void* router_scale, const void* per_expert_scale,
                             const void* pre_ffn_norm_2) {
  int rc = check_layer(h, layer);
  if (rc) return rc;
  if (h->ep_placed)
    return set_err(h, GM_ESTATE, "layers are registered before gm_moe_ep_set_placement");
  GM_TRY(h, cudaSetDevice(h->device), "register_layer_bq");
  Layer& L = h->layers[layer];
  free_moe(L);
  const size_t epr = (size_t)h->epr;
  if ((rc = dev_copy(h, &L.gu_q, gate_up, epr * GU * H, "gate_up"))) return rc;
  if ((rc = dev_copy(h, &L.gu_scale, gate_up_scale, epr * GU, "gate_up_scale"))) return rc;
  if ((rc = dev_copy(h, &L.dn_q, down, epr * H * I, "down"))) return rc;
  if ((rc = dev_copy(h, &L.dn_scale, down_scale, epr * H, "down_scale"))) return rc;
  if ((rc = dev_copy(h, &L.router, router_centered, (size_t)E * H, "router_centered"))) return rc;
  if ((rc = dev_copy(h, &L.rscale, router_scale, (size_t)H, "router_scale"))) return rc;
  if ((rc = dev_copy(h, &L.pes, per_expert_scale, (size_t)E, "per_expert_scale"))) return rc;
  if ((rc = dev_copy(h, &L.gamma2, pre_ffn_norm_2, (size_t)H, "pre_ffn_norm_2"))) return rc;
  // Row-major (K-contiguous) copy of gate_up for the tcgen05 prefill path: the
  // VNNI tile order is a byte permutation, undone once here on the device.  A
  // handle that can never reach the prefill path -- the most rows one call
  // processes (max_tokens, times the expert shards under expert parallelism)
  // below GM_OPT_TC_MIN_TOKENS -- keeps the VNNI copy only.
  L.has_tc = false;
  if ((long long)h->max_tokens * (E / h->epr) >= h->tc_min_tokens) {
    GM_TRY(h, cudaMalloc(reinterpret_cast<void**>(&L.gu_rm), epr * GU * H), "gate_up row-major copy");
    GM_TRY(h, launch_vnni_permute(L.gu_q, (long)(epr * GU), H, L.gu_rm, 1, h->own_stream), "vnni unpack");
    GM_TRY(h, cudaMalloc(reinterpret_cast<void**>(&L.dn_rm), epr * H * I), "down row-major copy");
    GM_TRY(h, launch_vnni_permute(L.dn_q, (long)(epr * H), I, L.dn_rm, 1, h->own_stream), "vnni unpack");
    GM_TRY(h, cudaStreamSynchronize(h->own_stream), "vnni unpack");
    L.has_tc = make_tmap_i8(L.tmap_gu, L.gu_rm, (long)(epr * GU), H, 64) &&
               make_tmap_i8(L.tmap_dn, L.dn_rm, (long)(epr * H), I, 128);
  }
  L.kind = 1;
  return GM_OK;
}

int gm_moe_register_layer_bf16(gm_moe_t* h, int layer, const void* gate_up, const void* down,
                               const void* router_proj, const void* router_scale,
                               const void* per_expert_scale, const void* pre_ffn_norm_2) {
  int rc = check_layer(h, layer);
  if (rc) return rc;
  if (h->ep_placed)
    return set_err(h, GM_ESTATE, "layers are registered before gm_moe_ep_set_placement");
  GM_TRY(h, cudaSetDevice(h->device), "register_layer_bf16");
  Layer& L = h->layers[layer];
  free_moe(L);
  const size_t epr = (size_t)h->epr;
  if ((rc = dev_copy(h, &L.gu_bf16, gate_up, epr * GU * H, "gate_up"))) return rc;
  if ((rc = dev_copy(h, &L.dn_bf16, down, epr * H * I, "down"))) return rc;
  if ((rc = dev_copy(h, &L.router, router_proj, (size_t)E * H, "router_proj"))) return rc;
  if ((rc = dev_copy(h, &L.rscale, router_scale, (size_t)H, "router_scale"))) return rc;
  if ((rc = dev_copy(h, &L.pes, per_expert_scale, (size_t)E, "per_expert_scale"))) return rc;
  if ((rc = dev_copy(h, &L.gamma2, pre_ffn_norm_2, (size_t)H, "pre_ffn_norm_2"))) return rc;
  L.has_tc = make_tmap_2d(L.tmap_gu, L.gu_bf16, (long)(epr * GU), H, 2, 64) &&
             make_tmap_2d(L.tmap_dn, L.dn_bf16, (long)(epr * H), I, 2, 128);
  L.kind = 2;
  return GM_OK;
}

namespace {
// Applies the handle's GM_OPT_PDL to launch_k for the scope of one forward.
struct PdlScope {
  bool saved;
  explicit PdlScope(bool on) : saved(tls_pdl) { tls_pdl = on; }
  ~PdlScope() { tls_pdl = saved; }
};
}  // namespace

namespace {
// gm_moe_forward (post == NULL) and gm_moe_forward_ffn (post-MoE tail fused
// into the final kernel, x_main updated in place).
int forward_impl(gm_moe* h, int layer, const void* x, void* out, int T, void* stream,
                 const PostParams* post) {
  int rc = check_layer(h, layer);
  if (rc) return rc;
  const Layer& L = h->layers[layer];
  if (L.kind == 0) return set_err(h, GM_ESTATE, "layer %d has no registered weights", layer);
  if (T < 0 || T > h->max_tokens)
    return set_err(h, GM_EINVAL, "T=%d outside [0, max_tokens=%d]", T, h->max_tokens);
  if (!x || !out) return set_err(h, GM_EINVAL, "NULL x/out");
  cudaStream_t s = S(stream);
  if (h->pending.size() > 4096 && (rc = drain_profile(h))) return rc;  // bound the event backlog
  PdlScope pdl_scope(h->pdl);
  if (h->ep_on) {
    if ((rc = ep_group_intact(h))) return rc;
    return ep_forward(h, L, static_cast<const uint16_t*>(x), static_cast<uint16_t*>(out), T, s, post);
  }
  if (T == 0) return GM_OK;
  const uint16_t* xb = static_cast<const uint16_t*>(x);
  // 0. decode batches route to nearly every expert: pull the gate/up weights
  // phase 1 reads first into L2 while the router runs (HBM is idle then).  The
  // prefetch runs on a side stream forked from `s`: nothing waits for it.
  bool forked = false;
  if (L.kind == 1 && T >= 32 && !(L.has_tc && h->tc_ok && T >= h->tc_min_tokens) && h->side_stream) {
    forked = true;
    GM_TRY(h, cudaEventRecord(h->fork_event, s), "prefetch fork");
    GM_TRY(h, cudaStreamWaitEvent(h->side_stream, h->fork_event, 0), "prefetch fork");
    const bool pdl = tls_pdl;
    tls_pdl = false;
    const long n0 = tls_kernel_launches;
    // every other expert from the second on (when the rank holds enough):
    // the first wave of phase 1 then mixes experts already in L2 with experts
    // streamed from HBM, instead of running from L2 while HBM idles
    const int npf = std::min(h->epr, L2_PREFETCH_EXPERTS);
    const int stride = 2 * npf <= h->epr ? 2 : 1;
    const cudaError_t pe =
        launch_l2_prefetch(L.gu_q, (size_t)GU * H, npf, stride == 2 ? 1 : 0, stride, h->side_stream);
    h->launches += tls_kernel_launches - n0;
    tls_pdl = pdl;
    GM_TRY(h, pe, "l2_prefetch");
  }
  // (the order needs the tcgen05 router, which can wait before reading x)
  const bool tc_rows = T >= h->tc_min_tokens && T >= ROUTER_TC_MIN_TOKENS && L.has_tc &&
                       (L.kind == 1 ? h->tc_ok : h->tcb_ok);
  if (tc_rows) {
    // tcgen05 prefill: the router first (it waits for x), the top-8 computes
    // each token's inv_rms itself, and the norm follows the schedule, writing
    // every token's row (int8 for bq, bf16 otherwise) straight into its
    // routes' rows of the gathered operand (no normalised copy and no gather
    // pass)
    GM_STAGE(h, s, launch_router_logits(xb, L.router, L.rscale, T, h->logits, h->dev_err, h->router_counts, s,
                                        true),
             "router_expert");
    GM_STAGE(h, s, launch_topk_inv_schedule(xb, h->logits, L.pes, h->inv_rms, T, h->route_idx, h->route_w,
                                            h->expert_base, h->epr,
                                            L.kind == 1 ? GM_ROUTE_CHUNK_BQ : GM_ROUTE_CHUNK_BF16,
                                            h->expert_offset, h->routes, h->route_pos, h->chunk_off,
                                            h->sched_counts, s),
             "router_merge.schedule");
    if (L.kind == 1)
      GM_STAGE(h, s, launch_bq_norm_gather(xb, L.gamma2, h->inv_rms, T, h->route_pos, h->xg, h->xg_sa, s),
               "bq_norm_gather");
    else
      GM_STAGE(h, s, launch_rms_norm_gather_bf16(xb, L.gamma2, h->inv_rms, T, h->route_pos,
                                                 reinterpret_cast<uint16_t*>(h->ybuf), s),
               "rms_norm_gather");
    CombineTarget ct;
    ct.out = static_cast<uint16_t*>(out);
    ct.post = post;
    return experts_and_combine(h, L, T, nullptr, nullptr, nullptr, h->route_idx, ct, s, true);
  }
  // 1. activation norm (+ inv_rms shared with the router)
  if (L.kind == 1)
    GM_STAGE(h, s, launch_bq_norm_quant(xb, L.gamma2, T, h->x_i8, h->x_sa, h->inv_rms, s), "bq_norm_quant");
  else
    GM_STAGE(h, s, launch_rms_norm_bf16(xb, L.gamma2, T, h->x_normed, h->inv_rms, s), "rms_norm");
  // 2. router logits, 3. top-8 + schedule
  GM_STAGE(h, s, launch_router_logits(xb, L.router, L.rscale, T, h->logits, h->dev_err, h->router_counts, s), "router_expert");
  const int rc_chunk = L.kind == 1 ? GM_ROUTE_CHUNK_BQ : GM_ROUTE_CHUNK_BF16;
  GM_STAGE(h, s, launch_topk_schedule(h->logits, L.pes, h->inv_rms, T, h->route_idx, h->route_w, h->expert_base,
                                 h->epr, rc_chunk, h->expert_offset, h->routes, h->route_pos,
                                 h->chunk_off, h->sched_counts, s),
         "router_merge.schedule");
  // 4. experts, 5. combine (+ post-MoE tail)
  CombineTarget ct;
  ct.out = static_cast<uint16_t*>(out);
  ct.post = post;
  rc = experts_and_combine(h, L, T, h->x_i8, h->x_sa, h->x_normed, h->route_idx, ct, s);
  if (rc == GM_OK && forked) {
    // Nothing waits for the prefetch when the forward runs eagerly; while `s`
    // is being captured into a CUDA graph, every stream forked from it must
    // join it again before the capture ends, so the side stream joins here.
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    GM_TRY(h, cudaStreamIsCapturing(s, &cs), "capture status");
    if (cs == cudaStreamCaptureStatusActive) {
      GM_TRY(h, cudaEventRecord(h->side_done, h->side_stream), "prefetch join");
      GM_TRY(h, cudaStreamWaitEvent(s, h->side_done, 0), "prefetch join");
    }
  }
  return rc;
}
}  // namespace

int gm_moe_forward(gm_moe_t* h, int layer, const void* x, void* out, int T, void* stream) {
  return forward_impl(h, layer, x, out, T, stream, nullptr);
}

int gm_moe_register_post(gm_moe_t* h, int layer, const void* post_ffn_norm_1,
                         const void* post_ffn_norm_2, const void* post_ffn_norm, float layer_scalar) {
  int rc = check_layer(h, layer);
  if (rc) return rc;
  GM_TRY(h, cudaSetDevice(h->device), "register_post");
  Layer& L = h->layers[layer];
  if ((rc = dev_copy(h, &L.post_w1, post_ffn_norm_1, (size_t)H, "post_ffn_norm_1"))) return rc;
  if ((rc = dev_copy(h, &L.post_w2, post_ffn_norm_2, (size_t)H, "post_ffn_norm_2"))) return rc;
  if ((rc = dev_copy(h, &L.post_w, post_ffn_norm, (size_t)H, "post_ffn_norm"))) return rc;
  L.layer_scalar = layer_scalar;
  return GM_OK;
}

int gm_moe_forward_ffn(gm_moe_t* h, int layer, void* x_main, const void* dense_out, int T,
                       void* stream) {
  int rc = check_layer(h, layer);
  if (rc) return rc;
  const Layer& L = h->layers[layer];
  if (!L.post_w1) return set_err(h, GM_ESTATE, "layer %d: gm_moe_register_post not called", layer);
  if (!x_main || !dense_out) return set_err(h, GM_EINVAL, "NULL x_main/dense_out");
  if (h->degree > 1 && !h->ep_on)
    return set_err(h, GM_ESTATE, "the post-MoE tail needs the complete MoE output: degree %d "
                   "without gm_moe_ep_init yields partials", h->degree);
  PostParams p{static_cast<const uint16_t*>(dense_out), static_cast<uint16_t*>(x_main), L.post_w1,
               L.post_w2, L.post_w, L.layer_scalar};
  return forward_impl(h, layer, x_main, x_main, T, stream, &p);
}

namespace {
// The dense MLP of dispatch_bq_ffn (modeling/gemma_4_moe_bq.mojo:749-783)
// on stream s: norm+quant with pre_feedforward_layernorm, gate/up + GeGLU +
// block quant, down -> out bf16 [T][H].
int run_dense(gm_moe* h, const Layer& L, const uint16_t* x, uint16_t* out, int T, cudaStream_t s) {
  if (T == 0) return GM_OK;
  GM_STAGE(h, s, launch_bq_norm_quant(x, L.dgamma, T, h->d_xi8, h->d_xsa, h->d_inv, s),
           "dense.bq_norm_quant");
  if (L.has_dense_tc && h->dense_tc_ok && T >= h->dense_tc_min) {
    GM_STAGE(h, s, launch_tc_dense_gate_up(h->tmap_dx, L.tmap_dgu, T, h->d_xsa, L.dgu_scale, h->d_hi8,
                                           h->d_hsa, nullptr, h->dev_err, s),
             "bq_linear.gate_up.tc");
    GM_STAGE(h, s, launch_tc_dense_down(h->tmap_dh, L.tmap_ddn, T, h->d_hsa, L.dd_scale, out,
                                        h->dev_err, s),
             "bq_block_linear.tc");
    return GM_OK;
  }
  GM_STAGE(h, s, launch_dense_gate_up(h->d_xi8, h->d_xsa, T, L.dg_q, L.dg_scale, L.du_q, L.du_scale,
                                      h->d_hi8, h->d_hsa, nullptr, s),
           "bq_linear.gate_up");
  GM_STAGE(h, s, launch_dense_down(h->d_hi8, h->d_hsa, T, L.dd_q, L.dd_scale, out, s), "bq_block_linear");
  return GM_OK;
}

int check_dense(gm_moe* h, int layer, const void* x, int T) {
  int rc = check_layer(h, layer);
  if (rc) return rc;
  if (!h->layers[layer].dg_q)
    return set_err(h, GM_ESTATE, "layer %d: gm_moe_register_dense_bq not called", layer);
  if (T < 0 || T > h->max_tokens)
    return set_err(h, GM_EINVAL, "T=%d outside [0, max_tokens=%d]", T, h->max_tokens);
  if (!x) return set_err(h, GM_EINVAL, "NULL activation");
  return GM_OK;
}
}  // namespace

int gm_moe_register_dense_bq(gm_moe_t* h, int layer, const void* gate_proj, const float* gate_scale,
                             const void* up_proj, const float* up_scale, const void* down_proj,
                             const float* down_scale, const void* pre_ffn_norm) {
  int rc = check_layer(h, layer);
  if (rc) return rc;
  GM_TRY(h, cudaSetDevice(h->device), "register_dense_bq");
  Layer& L = h->layers[layer];
  if ((rc = dev_copy(h, &L.dg_q, gate_proj, (size_t)DENSE_I * H, "gate_proj"))) return rc;
  if ((rc = dev_copy(h, &L.dg_scale, gate_scale, (size_t)DENSE_I, "gate_proj scale"))) return rc;
  if ((rc = dev_copy(h, &L.du_q, up_proj, (size_t)DENSE_I * H, "up_proj"))) return rc;
  if ((rc = dev_copy(h, &L.du_scale, up_scale, (size_t)DENSE_I, "up_proj scale"))) return rc;
  if ((rc = dev_copy(h, &L.dd_q, down_proj, (size_t)H * DENSE_I, "down_proj"))) return rc;
  if ((rc = dev_copy(h, &L.dd_scale, down_scale, (size_t)H, "down_proj scale"))) return rc;
  if ((rc = dev_copy(h, &L.dgamma, pre_ffn_norm, (size_t)H, "pre_ffn_norm"))) return rc;
  // row-major copies and tensor maps for the tcgen05 path
  for (void* p : {(void*)L.dgu_rm, (void*)L.dgu_scale, (void*)L.dd_rm})
    if (p) cudaFree(p);
  L.dgu_rm = L.dd_rm = nullptr;
  L.dgu_scale = nullptr;
  GM_TRY(h, cudaMalloc(reinterpret_cast<void**>(&L.dgu_rm), (size_t)2 * DENSE_I * H), "dense gate|up copy");
  GM_TRY(h, cudaMalloc(reinterpret_cast<void**>(&L.dgu_scale), (size_t)2 * DENSE_I * 4), "dense scales");
  GM_TRY(h, cudaMalloc(reinterpret_cast<void**>(&L.dd_rm), (size_t)H * DENSE_I), "dense down copy");
  GM_TRY(h, launch_vnni_permute(L.dg_q, DENSE_I, H, L.dgu_rm, 1, h->own_stream), "vnni unpack");
  GM_TRY(h, launch_vnni_permute(L.du_q, DENSE_I, H, L.dgu_rm + (size_t)DENSE_I * H, 1, h->own_stream),
         "vnni unpack");
  GM_TRY(h, launch_vnni_permute(L.dd_q, H, DENSE_I, L.dd_rm, 1, h->own_stream), "vnni unpack");
  GM_TRY(h, cudaMemcpyAsync(L.dgu_scale, L.dg_scale, DENSE_I * 4, cudaMemcpyDeviceToDevice, h->own_stream),
         "dense scales");
  GM_TRY(h, cudaMemcpyAsync(L.dgu_scale + DENSE_I, L.du_scale, DENSE_I * 4, cudaMemcpyDeviceToDevice,
                            h->own_stream),
         "dense scales");
  GM_TRY(h, cudaStreamSynchronize(h->own_stream), "dense copies");
  L.has_dense_tc = make_tmap_i8(L.tmap_dgu, L.dgu_rm, 2L * DENSE_I, H, 64) &&
                   make_tmap_i8(L.tmap_ddn, L.dd_rm, (long)H, DENSE_I, 128);
  return GM_OK;
}

int gm_dense_forward(gm_moe_t* h, int layer, const void* x, void* dense_out, int T, void* stream) {
  int rc = check_dense(h, layer, x, T);
  if (rc) return rc;
  if (!dense_out) return set_err(h, GM_EINVAL, "NULL dense_out");
  PdlScope pdl_scope(h->pdl);
  return run_dense(h, h->layers[layer], static_cast<const uint16_t*>(x),
                   static_cast<uint16_t*>(dense_out), T, S(stream));
}

int gm_ffn_forward(gm_moe_t* h, int layer, void* x_main, int T, void* stream) {
  int rc = check_dense(h, layer, x_main, T);
  if (rc) return rc;
  const Layer& L = h->layers[layer];
  if (L.kind == 0) return set_err(h, GM_ESTATE, "layer %d has no registered experts", layer);
  if (!L.post_w1) return set_err(h, GM_ESTATE, "layer %d: gm_moe_register_post not called", layer);
  if (h->degree > 1 && !h->ep_on)
    return set_err(h, GM_ESTATE, "the post-MoE tail needs the complete MoE output: degree %d "
                   "without gm_moe_ep_init yields partials", h->degree);
  cudaStream_t s = S(stream);
  const uint16_t* x = static_cast<const uint16_t*>(x_main);
  {
    PdlScope pdl_scope(h->pdl);
    if (h->dense_stream && T > 0) {
      // the dense MLP runs beside the MoE on the same input; the tail joins it
      GM_TRY(h, cudaEventRecord(h->dense_fork, s), "dense fork");
      GM_TRY(h, cudaStreamWaitEvent(h->dense_stream, h->dense_fork, 0), "dense fork");
      if ((rc = run_dense(h, L, x, h->d_out, T, h->dense_stream))) return rc;
      GM_TRY(h, cudaEventRecord(h->dense_done, h->dense_stream), "dense done");
      h->dense_pending = true;
    } else if ((rc = run_dense(h, L, x, h->d_out, T, s))) {
      return rc;
    }
  }
  PostParams p{h->d_out, static_cast<uint16_t*>(x_main), L.post_w1, L.post_w2, L.post_w, L.layer_scalar};
  return forward_impl(h, layer, x_main, x_main, T, s, &p);
}

int gm_moe_set_option(gm_moe_t* h, int option, long value) {
  if (!h) return set_err(nullptr, GM_EINVAL, "NULL handle");
  switch (option) {
    case GM_OPT_TC_MIN_TOKENS:
      if (value < 1) return set_err(h, GM_EINVAL, "GM_OPT_TC_MIN_TOKENS must be >= 1");
      h->tc_min_tokens = value > 0x7FFFFFFF ? 0x7FFFFFFF : (int)value;
      return GM_OK;
    case GM_OPT_DENSE_TC_MIN_TOKENS:
      if (value < 1) return set_err(h, GM_EINVAL, "GM_OPT_DENSE_TC_MIN_TOKENS must be >= 1");
      h->dense_tc_min = value > 0x7FFFFFFF ? 0x7FFFFFFF : (int)value;
      return GM_OK;
    case GM_OPT_EP_TRANSPORT:
      if (value != 0 && value != 1) return set_err(h, GM_EINVAL, "GM_OPT_EP_TRANSPORT must be 0 or 1");
      if (value == 1 && !h->ep_p2p_ok)
        return set_err(h, GM_ESTATE, "peer-memory transport unavailable (not initialised or not mapped)");
      if (value == 0 && !h->ep_comm)
        return set_err(h, GM_ESTATE, "the NCCL transport needs gm_moe_ep_init (an in-process group has "
                       "no communicator)");
      h->ep_use_p2p = value == 1;
      return GM_OK;
    case GM_OPT_EP_TIMEOUT_MS:
      if (value < 1 || value > 600000)
        return set_err(h, GM_EINVAL, "GM_OPT_EP_TIMEOUT_MS must be in [1, 600000]");
      h->ep_timeout_ms = (int)value;
      return GM_OK;
    case GM_OPT_EP_INIT_TIMEOUT_MS:
      if (value < 1 || value > 3600000)
        return set_err(h, GM_EINVAL, "GM_OPT_EP_INIT_TIMEOUT_MS must be in [1, 3600000]");
      h->ep_init_timeout_ms = (int)value;
      return GM_OK;
    case GM_OPT_PDL:
      if (value != 0 && value != 1) return set_err(h, GM_EINVAL, "GM_OPT_PDL must be 0 or 1");
      h->pdl = value != 0;
      return GM_OK;
    case GM_OPT_PROFILE: {
      if (value != 0 && value != 1) return set_err(h, GM_EINVAL, "GM_OPT_PROFILE must be 0 or 1");
      GM_TRY(h, cudaSetDevice(h->device), "GM_OPT_PROFILE");
      const int rc = drain_profile(h);
      h->stats.clear();
      h->launches = 0;
      h->profile = value != 0;
      return rc;
    }
    default:
      return set_err(h, GM_EINVAL, "unknown option %d", option);
  }
}

int gm_moe_profile_read(gm_moe_t* h, gm_stage_stat_t* stats, int max_stats, int* n_stats,
                        long* kernel_launches) {
  if (!h || !n_stats || max_stats < 0 || (max_stats > 0 && !stats))
    return set_err(h, GM_EINVAL, "gm_moe_profile_read: bad arguments");
  GM_TRY(h, cudaSetDevice(h->device), "profile_read");
  const int rc = drain_profile(h);
  const int n = (int)h->stats.size();
  for (int i = 0; i < n && i < max_stats; ++i) {
    stats[i] = h->stats[i];
    if (stats[i].calls == 0) stats[i].min_ms = 0.0;
  }
  *n_stats = n;
  if (kernel_launches) *kernel_launches = h->launches;
  return rc;
}

int gm_ep_unique_id(void* out, size_t bytes) {
  if (!out || bytes < sizeof(ncclUniqueId))
    return set_err(nullptr, GM_EINVAL, "gm_ep_unique_id: need %zu bytes", sizeof(ncclUniqueId));
  const char* why = nullptr;
  const NcclApi* nc = nccl_api(&why);
  if (!nc) return set_err(nullptr, GM_ENCCL, "%s", why ? why : "NCCL unavailable");
  ncclUniqueId id;
  const ncclResult_t r = nc->get_unique_id(&id);
  if (r != ncclSuccess) return set_err(nullptr, GM_ENCCL, "ncclGetUniqueId: %s", nc->get_error_string(r));
  memcpy(out, &id, sizeof id);
  return GM_OK;
}

int gm_moe_ep_init(gm_moe_t* h, const void* unique_id, int world) {
  if (!h || !unique_id) return set_err(h, GM_EINVAL, "gm_moe_ep_init: NULL argument");
  if (h->ep_on) return set_err(h, GM_ESTATE, "gm_moe_ep_init: already initialised");
  if (world != h->degree || world < 1 || world > 8)
    return set_err(h, GM_EINVAL, "gm_moe_ep_init: world=%d must equal the handle's degree (%d), 1..8",
                   world, h->degree);
  const char* why = nullptr;
  const NcclApi* nc = nccl_api(&why);
  if (!nc) return set_err(h, GM_ENCCL, "%s", why ? why : "NCCL unavailable");
  GM_TRY(h, cudaSetDevice(h->device), "ep_init");
  EpLayout o;
  int rc = ep_alloc(h, world, &o);
  if (rc) return rc;
  // Non-blocking communicator: the initialisation is polled against a host
  // deadline (GM_OPT_EP_INIT_TIMEOUT_MS) and aborted when a rank never
  // arrives, instead of blocking the caller for good.
  ncclUniqueId id;
  memcpy(&id, unique_id, sizeof id);
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  ncclComm_t comm = nullptr;
  ncclResult_t r = nc->comm_init_rank_config(&comm, world, id, h->rank, &cfg);
  if (r == ncclInProgress) r = nccl_settle(comm, r, h->ep_init_timeout_ms);
  if (r != ncclSuccess) {
    if (comm) nc->comm_abort(comm);
    if (r == ncclInProgress)
      return set_err(h, GM_ETIMEOUT, "ncclCommInitRankConfig: the group of %d ranks did not form within "
                     "%d ms (a rank never joined); communicator aborted", world, h->ep_init_timeout_ms);
    return set_err(h, GM_ENCCL, "ncclCommInitRankConfig: %s", nc->get_error_string(r));
  }
  h->ep_comm = comm;
  h->ep_on = true;
  // Peer-memory transport: map every rank's exchange allocation (the carve
  // offsets are the same on every rank: same max_tokens and world).
  bool ok = true;
  cudaIpcMemHandle_t mine_h;
  if (cudaIpcGetMemHandle(&mine_h, h->ep_buf) != cudaSuccess) ok = false;
  std::vector<cudaIpcMemHandle_t> all(world);
  void* dev_h = nullptr;
  if (ok && cudaMalloc(&dev_h, sizeof(cudaIpcMemHandle_t) * (world + 1)) != cudaSuccess) ok = false;
  // every rank takes part in the all-gather (a rank that failed sends zeros)
  if (dev_h) {
    cudaMemcpy(dev_h, &mine_h, sizeof mine_h, cudaMemcpyHostToDevice);
    char* dh = static_cast<char*>(dev_h);
    ncclResult_t gr = nccl_settle(comm, nc->all_gather(dh, dh + sizeof(cudaIpcMemHandle_t), sizeof(cudaIpcMemHandle_t),
                                                       ncclUint8, comm, h->own_stream), 60000);
    if (gr != ncclSuccess || cudaStreamSynchronize(h->own_stream) != cudaSuccess) ok = false;
    if (ok) cudaMemcpy(all.data(), dh + sizeof(cudaIpcMemHandle_t), sizeof(cudaIpcMemHandle_t) * world,
                       cudaMemcpyDeviceToHost);
    cudaFree(dev_h);
  }
  for (int q = 0; ok && q < world; ++q) {
    if (q == h->rank) {
      h->ep_peer_base[q] = h->ep_buf;
    } else if (cudaIpcOpenMemHandle(&h->ep_peer_base[q], all[q], cudaIpcMemLazyEnablePeerAccess) !=
               cudaSuccess) {
      h->ep_peer_base[q] = nullptr;
      ok = false;
    }
  }
  cudaGetLastError();
  if (ok) ep_wire(h, world, h->ep_peer_base, o);
  // every rank must choose the same transport: agree on "all ranks mapped"
  int* dflag_ok = nullptr;
  bool all_ok = false;
  if (cudaMalloc(&dflag_ok, sizeof(int) * (world + 1)) == cudaSuccess) {
    const int v = ok ? 1 : 0;
    cudaMemcpy(dflag_ok, &v, sizeof v, cudaMemcpyHostToDevice);
    if (nccl_settle(comm, nc->all_gather(dflag_ok, dflag_ok + 1, 1, ncclInt32, comm, h->own_stream), 60000) ==
            ncclSuccess &&
        cudaStreamSynchronize(h->own_stream) == cudaSuccess) {
      std::vector<int> v_all(world);
      cudaMemcpy(v_all.data(), dflag_ok + 1, sizeof(int) * world, cudaMemcpyDeviceToHost);
      all_ok = true;
      for (int x : v_all) all_ok = all_ok && x == 1;
    }
    cudaFree(dflag_ok);
  }
  cudaGetLastError();
  h->ep_p2p_ok = all_ok;
  h->ep_use_p2p = all_ok;
  return GM_OK;
}

int gm_moe_ep_init_group(gm_moe_t* const* handles, int world) {
  if (!handles || world < 1 || world > 8)
    return set_err(nullptr, GM_EINVAL, "gm_moe_ep_init_group: world=%d (1..8) or NULL handles", world);
  for (int g = 0; g < world; ++g) {
    gm_moe* h = handles[g];
    if (!h) return set_err(nullptr, GM_EINVAL, "gm_moe_ep_init_group: handle %d is NULL", g);
    if (h->ep_on) return set_err(h, GM_ESTATE, "gm_moe_ep_init_group: handle %d already initialised", g);
    if (h->degree != world || h->rank != g)
      return set_err(h, GM_EINVAL, "gm_moe_ep_init_group: handle %d has rank %d of degree %d (want %d of %d)",
                     g, h->rank, h->degree, g, world);
    if (h->max_tokens != handles[0]->max_tokens)
      return set_err(h, GM_EINVAL, "gm_moe_ep_init_group: every handle needs the same max_tokens");
    for (int q = 0; q < g; ++q)
      if (handles[q] == h) return set_err(h, GM_EINVAL, "gm_moe_ep_init_group: handle %d repeated", g);
  }
  // members on different devices store into each other's memory directly
  for (int g = 0; g < world; ++g)
    for (int q = 0; q < world; ++q) {
      const int dg = handles[g]->device, dq = handles[q]->device;
      if (dg == dq) continue;
      int can = 0;
      if (cudaDeviceCanAccessPeer(&can, dg, dq) != cudaSuccess || !can)
        return set_err(handles[g], GM_ECUDA, "gm_moe_ep_init_group: device %d cannot access device %d", dg, dq);
      GM_TRY(handles[g], cudaSetDevice(dg), "ep_init_group");
      const cudaError_t e = cudaDeviceEnablePeerAccess(dq, 0);
      if (e != cudaSuccess && e != cudaErrorPeerAccessAlreadyEnabled)
        return cuda_check(handles[g], e, "cudaDeviceEnablePeerAccess");
      cudaGetLastError();
    }
  EpLayout o;
  void* bases[8] = {};
  for (int g = 0; g < world; ++g) {
    GM_TRY(handles[g], cudaSetDevice(handles[g]->device), "ep_init_group");
    int rc = ep_alloc(handles[g], world, &o);
    if (rc) return rc;
    bases[g] = handles[g]->ep_buf;
  }
  for (int g = 0; g < world; ++g) {
    gm_moe* h = handles[g];
    ep_wire(h, world, bases, o);
    for (int q = 0; q < world; ++q) {
      h->ep_members[q] = handles[q];
      h->ep_peer_base[q] = bases[q];
    }
    h->ep_group = true;
    h->ep_on = true;
    h->ep_p2p_ok = h->ep_use_p2p = true;
  }
  return GM_OK;
}

int gm_moe_ep_forward_group(gm_moe_t* const* handles, int world, int layer, const void* const* x,
                            void* const* out, const int* T, void* const* streams) {
  if (!handles || !x || !out || !T || !streams || world < 1 || world > 8)
    return set_err(nullptr, GM_EINVAL, "gm_moe_ep_forward_group: NULL argument or world=%d", world);
  for (int g = 0; g < world; ++g) {
    gm_moe* h = handles[g];
    if (!h || !h->ep_group || h->degree != world || h->ep_members[g] != h || h->ep_members[0] != handles[0])
      return set_err(h, GM_EINVAL, "gm_moe_ep_forward_group: handle %d is not member %d of one group "
                     "(gm_moe_ep_init_group)", g, g);
    int rc = ep_group_intact(h);
    if (rc) return rc;
    rc = check_layer(h, layer);
    if (rc) return rc;
    if (h->layers[layer].kind == 0) return set_err(h, GM_ESTATE, "layer %d has no registered weights", layer);
    if (T[g] < 0 || T[g] > h->max_tokens)
      return set_err(h, GM_EINVAL, "member %d: T=%d outside [0, max_tokens=%d]", g, T[g], h->max_tokens);
    if (!x[g] || !out[g]) return set_err(h, GM_EINVAL, "member %d: NULL x/out", g);
    // members sharing a GPU run their phases on one stream, in issue order: a
    // wait kernel then never spins on a kernel that has not yet run
    for (int q = 0; q < g; ++q)
      if (handles[q]->device == h->device && streams[q] != streams[g])
        return set_err(h, GM_EINVAL, "members %d and %d share device %d: pass them the same stream", q, g,
                       h->device);
  }
  for (int phase = 0; phase < 3; ++phase)
    for (int g = 0; g < world; ++g) {
      gm_moe* h = handles[g];
      GM_TRY(h, cudaSetDevice(h->device), "ep_forward_group");
      if (h->pending.size() > 4096) {
        int rc = drain_profile(h);
        if (rc) return rc;
      }
      PdlScope pdl_scope(h->pdl);
      const Layer& L = h->layers[layer];
      cudaStream_t s = S(streams[g]);
      int rc = phase == 0 ? ep_phase_a(h, L, static_cast<const uint16_t*>(x[g]), T[g], s)
             : phase == 1 ? ep_phase_b(h, L, s)
                          : ep_phase_c(h, static_cast<uint16_t*>(out[g]), T[g], s, nullptr);
      if (rc) return rc;
    }
  return GM_OK;
}

namespace {
// Checks an expert -> rank map (every rank exactly 128/world experts) and
// derives the device tables: rank_of[e], local_of[e] (index among its rank's
// experts, ascending id order) and, per rank, its experts in ascending order.
int placement_tables(gm_moe* h, const int32_t* expert_rank, std::vector<int32_t>& rank_of,
                     std::vector<int32_t>& local_of, std::vector<std::vector<int>>& mine) {
  const int G = h->degree, epr = h->epr;
  rank_of.assign(E, 0);
  local_of.assign(E, 0);
  mine.assign(G, {});
  for (int e = 0; e < E; ++e) {
    const int r = expert_rank[e];
    if (r < 0 || r >= G) return set_err(h, GM_EINVAL, "expert %d placed on rank %d of %d", e, r, G);
    rank_of[e] = r;
    local_of[e] = (int32_t)mine[r].size();
    mine[r].push_back(e);
  }
  for (int r = 0; r < G; ++r)
    if ((int)mine[r].size() != epr)
      return set_err(h, GM_EINVAL, "rank %d holds %zu experts; every rank must hold %d", r, mine[r].size(), epr);
  return GM_OK;
}

// The per-expert tensors of a layer, with their bytes per expert.
std::vector<std::pair<void*, size_t>> expert_tensors(Layer& L) {
  if (L.kind == 1)
    return {{L.gu_q, (size_t)GU * H}, {L.gu_scale, GU * sizeof(float)}, {L.dn_q, (size_t)H * I},
            {L.dn_scale, H * sizeof(float)}};
  if (L.kind == 2) return {{L.gu_bf16, (size_t)GU * H * 2}, {L.dn_bf16, (size_t)H * I * 2}};
  return {};
}

// After the expert tensors moved: the tcgen05 path's row-major copies (same
// buffers, so the TMA descriptors stay valid) and the placement tables.
int finish_placement(gm_moe* h, const std::vector<int32_t>& rank_of, const std::vector<int32_t>& local_of) {
  cudaStream_t s = h->own_stream;
  for (auto& L : h->layers)
    if (L.kind == 1 && L.gu_rm) {
      GM_TRY(h, launch_vnni_permute(L.gu_q, (long)h->epr * GU, H, L.gu_rm, 1, s), "vnni unpack");
      GM_TRY(h, launch_vnni_permute(L.dn_q, (long)h->epr * H, I, L.dn_rm, 1, s), "vnni unpack");
    }
  GM_TRY(h, cudaMemcpyAsync(h->ep_rank_of, rank_of.data(), E * sizeof(int32_t), cudaMemcpyHostToDevice, s),
         "placement tables");
  GM_TRY(h, cudaMemcpyAsync(h->ep_local_of, local_of.data(), E * sizeof(int32_t), cudaMemcpyHostToDevice, s),
         "placement tables");
  GM_TRY(h, cudaStreamSynchronize(s), "placement tables");
  h->ep_placed = true;
  return GM_OK;
}
}  // namespace

int gm_moe_ep_set_placement(gm_moe_t* h, const int32_t* expert_rank) {
  if (!h || !expert_rank) return set_err(h, GM_EINVAL, "gm_moe_ep_set_placement: NULL argument");
  if (!h->ep_comm)
    return set_err(h, GM_ESTATE, "gm_moe_ep_set_placement: gm_moe_ep_init first (an in-process group "
                   "uses gm_moe_ep_set_placement_group)");
  if (h->ep_placed) return set_err(h, GM_ESTATE, "gm_moe_ep_set_placement: placement already set");
  const int epr = h->epr;
  std::vector<int32_t> rank_of, local_of;
  std::vector<std::vector<int>> mine;
  int rc = placement_tables(h, expert_rank, rank_of, local_of, mine);
  if (rc) return rc;
  const NcclApi* nc = nccl_api(nullptr);
  GM_TRY(h, cudaSetDevice(h->device), "ep_set_placement");
  cudaStream_t s = h->own_stream;
  // Every registered layer arrived as the reference's contiguous block of this
  // rank: gather all blocks (global expert order) and keep this rank's experts.
  for (auto& L : h->layers)
    for (auto& t : expert_tensors(L)) {
      void* full = nullptr;
      GM_TRY(h, cudaMalloc(&full, t.second * E), "ep placement gather buffer");
      rc = nccl_check(h, nc->all_gather(t.first, full, t.second * epr, ncclUint8, h->ep_comm, s),
                      "ep placement all-gather");
      for (int i = 0; rc == GM_OK && i < epr; ++i)
        rc = cuda_check(h, cudaMemcpyAsync(static_cast<char*>(t.first) + i * t.second,
                                           static_cast<char*>(full) + mine[h->rank][i] * t.second, t.second,
                                           cudaMemcpyDeviceToDevice, s),
                        "ep placement copy");
      if (rc == GM_OK) rc = cuda_check(h, cudaStreamSynchronize(s), "ep placement");
      cudaFree(full);
      if (rc) return rc;
    }
  return finish_placement(h, rank_of, local_of);
}

int gm_moe_ep_set_placement_group(gm_moe_t* const* handles, int world, const int32_t* expert_rank) {
  if (!handles || !expert_rank || world < 1 || world > 8)
    return set_err(nullptr, GM_EINVAL, "gm_moe_ep_set_placement_group: NULL argument or world=%d", world);
  for (int g = 0; g < world; ++g) {
    gm_moe* h = handles[g];
    if (!h || !h->ep_group || h->degree != world || h->ep_members[g] != h || h->ep_members[0] != handles[0])
      return set_err(h, GM_EINVAL, "gm_moe_ep_set_placement_group: handle %d is not member %d of one group", g, g);
    if (int rc = ep_group_intact(h)) return rc;
    if (h->ep_placed) return set_err(h, GM_ESTATE, "gm_moe_ep_set_placement_group: placement already set");
    if (h->num_layers != handles[0]->num_layers)
      return set_err(h, GM_EINVAL, "gm_moe_ep_set_placement_group: members differ in their layer count");
    for (int l = 0; l < h->num_layers; ++l)
      if (h->layers[l].kind != handles[0]->layers[l].kind)
        return set_err(h, GM_ESTATE, "layer %d is not registered alike on every member", l);
  }
  gm_moe* h0 = handles[0];
  const int epr = h0->epr;
  std::vector<int32_t> rank_of, local_of;
  std::vector<std::vector<int>> mine;
  int rc = placement_tables(h0, expert_rank, rank_of, local_of, mine);
  if (rc) return rc;
  // every member's contiguous block, in global expert order, on member 0's
  // device; then each member copies out its placed experts
  GM_TRY(h0, cudaSetDevice(h0->device), "ep_set_placement_group");
  for (int l = 0; l < h0->num_layers; ++l) {
    const size_t nt = expert_tensors(h0->layers[l]).size();
    for (size_t ti = 0; ti < nt; ++ti) {
      const size_t per = expert_tensors(h0->layers[l])[ti].second;
      void* full = nullptr;
      GM_TRY(h0, cudaSetDevice(h0->device), "ep_set_placement_group");
      GM_TRY(h0, cudaMalloc(&full, per * E), "ep placement gather buffer");
      for (int g = 0; rc == GM_OK && g < world; ++g) {
        void* src = expert_tensors(handles[g]->layers[l])[ti].first;
        rc = cuda_check(h0, cudaMemcpyPeer(static_cast<char*>(full) + (size_t)g * epr * per, h0->device, src,
                                           handles[g]->device, per * epr),
                        "ep placement gather");
      }
      for (int g = 0; rc == GM_OK && g < world; ++g) {
        void* dst = expert_tensors(handles[g]->layers[l])[ti].first;
        for (int i = 0; rc == GM_OK && i < epr; ++i)
          rc = cuda_check(h0, cudaMemcpyPeer(static_cast<char*>(dst) + (size_t)i * per, handles[g]->device,
                                             static_cast<char*>(full) + (size_t)mine[g][i] * per, h0->device, per),
                          "ep placement copy");
      }
      cudaSetDevice(h0->device);
      cudaFree(full);
      if (rc) return rc;
    }
  }
  for (int g = 0; g < world; ++g) {
    GM_TRY(handles[g], cudaSetDevice(handles[g]->device), "ep_set_placement_group");
    if ((rc = finish_placement(handles[g], rank_of, local_of))) return rc;
  }
  return GM_OK;
}

int gm_moe_device_status(gm_moe_t* h, int* device_error) {
  if (!h || !device_error) return set_err(h, GM_EINVAL, "NULL argument");
  GM_TRY(h, cudaSetDevice(h->device), "device_status");
  GM_TRY(h, cudaDeviceSynchronize(), "device_status");
  GM_TRY(h, cudaMemcpy(device_error, h->dev_err, sizeof(int), cudaMemcpyDeviceToHost), "device_status");
  GM_TRY(h, cudaMemset(h->dev_err, 0, sizeof(int)), "device_status");
  if (*device_error) {
    // a kernel that gave up may have left self-re-arming counters mid-count
    cudaMemset(h->router_counts, 0, sizeof(int) * router_tile_counters(h->ws_tokens));
    if (h->ep_counters) cudaMemset(h->ep_counters, 0, 2 * sizeof(int));
    cudaDeviceSynchronize();
    return set_err(h, GM_ETIMEOUT, "a kernel's bounded wait expired (code %d)", *device_error);
  }
  return GM_OK;
}

int gm_moe_forward_sync(gm_moe_t* h, int layer, const void* x, void* out, int T) {
  int rc = check_layer(h, layer);
  if (rc) return rc;
  if (T < 0 || T > h->max_tokens)
    return set_err(h, GM_EINVAL, "T=%d outside [0, max_tokens=%d]", T, h->max_tokens);
  if (T == 0) return GM_OK;
  GM_TRY(h, cudaSetDevice(h->device), "forward_sync");
  cudaStream_t s = h->own_stream;
  const size_t bytes = (size_t)T * H * sizeof(uint16_t);
  const bool x_dev = is_device_ptr(x), o_dev = is_device_ptr(out);
  const void* xd = x;
  if (!x_dev) {
    GM_TRY(h, cudaMemcpyAsync(h->x_stage, x, bytes, cudaMemcpyHostToDevice, s), "stage x");
    xd = h->x_stage;
  }
  // A mapped page-locked `out` is written by the last kernel directly over the
  // bus (overlapped with its own work) instead of a copy after it; other host
  // memory goes through the staging buffer.
  void* o_map = o_dev ? nullptr : mapped_host_ptr(out);
  void* od = o_dev ? out : o_map ? o_map : h->out_stage;
  if ((rc = gm_moe_forward(h, layer, xd, od, T, s))) return rc;
  if (!o_dev && !o_map) GM_TRY(h, cudaMemcpyAsync(out, od, bytes, cudaMemcpyDeviceToHost, s), "stage out");
  GM_TRY(h, cudaStreamSynchronize(s), "forward_sync");
  return GM_OK;
}

// ------------------------------------------------------------ per-stage
#define STAGE(expr, what)                                            \
  do {                                                               \
    cudaError_t _e = (expr);                                         \
    if (_e != cudaSuccess) return cuda_check(nullptr, _e, (what));   \
    return GM_OK;                                                    \
  } while (0)

int gm_router_select(const void* x, const void* router_w, const void* router_scale,
                     const void* per_expert_scale, int T, float* logits_ws, int32_t* route_idx,
                     float* route_w, void* stream) {
  if (T < 0) return set_err(nullptr, GM_EINVAL, "router_select: T=%d", T);
  STAGE(launch_router(static_cast<const uint16_t*>(x), static_cast<const uint16_t*>(router_w),
                      static_cast<const uint16_t*>(router_scale),
                      static_cast<const uint16_t*>(per_expert_scale), T, logits_ws, route_idx,
                      route_w, S(stream)),
        "router_select");
}

int gm_build_expert_schedules(const int32_t* route_idx, const float* route_w, int T,
                              int expert_base, int epr, int route_chunk, int32_t* expert_offset,
                              gm_sparse_route_t* routes, int32_t* route_pos, int32_t* chunk_off,
                              void* stream) {
  if (T < 0 || epr < 1 || epr > E || route_chunk < 1)
    return set_err(nullptr, GM_EINVAL, "build_expert_schedules: T=%d epr=%d route_chunk=%d", T, epr,
                   route_chunk);
  STAGE(launch_build_schedule(route_idx, route_w, T, expert_base, epr, route_chunk, expert_offset,
                              reinterpret_cast<SparseRoute*>(routes), route_pos, chunk_off,
                              S(stream)),
        "build_expert_schedules");
}

int gm_rms_norm(const void* x, const void* gamma, int T, void* out, void* stream) {
  STAGE(launch_rms_norm_bf16(static_cast<const uint16_t*>(x), static_cast<const uint16_t*>(gamma),
                             T, static_cast<uint16_t*>(out), nullptr, S(stream)),
        "rms_norm");
}

int gm_norm_residual_add(const void* src, const void* residual, const void* weight, int T, void* out,
                         void* stream) {
  if (T < 0 || (T > 0 && (!src || !residual || !weight || !out)))
    return set_err(nullptr, GM_EINVAL, "norm_residual_add: T=%d or a NULL pointer", T);
  if (((uintptr_t)src | (uintptr_t)residual | (uintptr_t)weight | (uintptr_t)out) & 15)
    return set_err(nullptr, GM_EINVAL, "norm_residual_add: buffers must be 16-byte aligned");
  STAGE(launch_norm_residual_add(static_cast<const uint16_t*>(src), static_cast<const uint16_t*>(residual),
                                 static_cast<const uint16_t*>(weight), T, static_cast<uint16_t*>(out),
                                 S(stream)),
        "norm_residual_add");
}

int gm_bq_norm_quant(const void* x, const void* gamma, int T, int8_t* x_i8, float* x_sa,
                     void* stream) {
  STAGE(launch_bq_norm_quant(static_cast<const uint16_t*>(x), static_cast<const uint16_t*>(gamma),
                             T, x_i8, x_sa, nullptr, S(stream)),
        "bq_norm_quant");
}

int gm_bq_phase1_gate_up(const int8_t* x_i8, const float* x_sa, const int32_t* expert_offset,
                         const gm_sparse_route_t* routes, const int32_t* chunk_off, int epr, int T,
                         const void* gate_up, const float* gate_up_scale, int8_t* bucket_i8,
                         float* bucket_sa, void* bucket_bf16, void* stream) {
  if (epr < 1 || epr > E || T < 0) return set_err(nullptr, GM_EINVAL, "bq_phase1: epr=%d T=%d", epr, T);
  STAGE(launch_bq_phase1(x_i8, x_sa, expert_offset, reinterpret_cast<const SparseRoute*>(routes),
                         chunk_off, epr, T, static_cast<const int8_t*>(gate_up), gate_up_scale,
                         bucket_i8, bucket_sa, static_cast<uint16_t*>(bucket_bf16), S(stream)),
        "bq_phase1_gate_up");
}

int gm_bq_block_quant(const void* bucket, long rows, int8_t* q, float* sa, void* stream) {
  STAGE(launch_block_quant(static_cast<const uint16_t*>(bucket), rows, q, sa, S(stream)),
        "bq_block_quant");
}

int gm_bq_phase2_down(const int8_t* bucket_i8, const float* bucket_sa, const int32_t* expert_offset,
                      const gm_sparse_route_t* routes, const int32_t* chunk_off, int epr, int T,
                      const void* down, const float* down_scale, float* y, void* stream) {
  if (epr < 1 || epr > E || T < 0) return set_err(nullptr, GM_EINVAL, "bq_phase2: epr=%d T=%d", epr, T);
  STAGE(launch_bq_phase2(bucket_i8, bucket_sa, expert_offset,
                         reinterpret_cast<const SparseRoute*>(routes), chunk_off, epr, T,
                         static_cast<const int8_t*>(down), down_scale, y, false, S(stream)),
        "bq_phase2_down");
}

int gm_bq_dense_gate_up(const int8_t* x_i8, const float* x_sa, int T, const void* gate_proj,
                        const float* gate_scale, const void* up_proj, const float* up_scale,
                        int8_t* h_i8, float* h_sa, void* h_bf16, void* stream) {
  if (T < 0) return set_err(nullptr, GM_EINVAL, "bq_dense_gate_up: T=%d", T);
  STAGE(launch_dense_gate_up(x_i8, x_sa, T, static_cast<const int8_t*>(gate_proj), gate_scale,
                             static_cast<const int8_t*>(up_proj), up_scale, h_i8, h_sa,
                             static_cast<uint16_t*>(h_bf16), S(stream)),
        "bq_dense_gate_up");
}

int gm_bq_block_linear(const int8_t* h_i8, const float* h_sa, int T, const void* down_proj,
                       const float* down_scale, void* out, void* stream) {
  if (T < 0) return set_err(nullptr, GM_EINVAL, "bq_block_linear: T=%d", T);
  STAGE(launch_dense_down(h_i8, h_sa, T, static_cast<const int8_t*>(down_proj), down_scale,
                          static_cast<uint16_t*>(out), S(stream)),
        "bq_block_linear");
}

int gm_bq_linear(const int8_t* x_i8, const float* x_sa, int T, const void* w, const float* w_scale,
                 int n_rows, void* out, void* stream) {
  if (T < 0 || n_rows <= 0 || n_rows % 32)
    return set_err(nullptr, GM_EINVAL, "bq_linear: T=%d n_rows=%d (a multiple of 32)", T, n_rows);
  const int8_t* wl[1] = {static_cast<const int8_t*>(w)};
  const float* sl[1] = {w_scale};
  uint16_t* ol[1] = {static_cast<uint16_t*>(out)};
  STAGE(launch_bq_linear_multi(x_i8, x_sa, T, 1, wl, sl, ol, &n_rows, S(stream)), "bq_linear");
}

int gm_bq_qkv(const int8_t* x_i8, const float* x_sa, int T, const void* q_w, const float* q_scale, int qn,
              const void* k_w, const float* k_scale, const void* v_w, const float* v_scale, int kvn,
              void* q_out, void* k_out, void* v_out, void* stream) {
  if (T < 0 || qn <= 0 || qn % 32 || kvn <= 0 || kvn % 32)
    return set_err(nullptr, GM_EINVAL, "bq_qkv: T=%d qn=%d kvn=%d (multiples of 32)", T, qn, kvn);
  if (!q_w || !k_w || !q_out || !k_out || (v_w && !v_out))
    return set_err(nullptr, GM_EINVAL, "bq_qkv: NULL weight or output");
  const int nseg = v_w ? 3 : 2;  // full layers: K = V, no v projection
  const int8_t* wl[3] = {static_cast<const int8_t*>(q_w), static_cast<const int8_t*>(k_w),
                         static_cast<const int8_t*>(v_w)};
  const float* sl[3] = {q_scale, k_scale, v_scale};
  uint16_t* ol[3] = {static_cast<uint16_t*>(q_out), static_cast<uint16_t*>(k_out), static_cast<uint16_t*>(v_out)};
  const int nl[3] = {qn, kvn, kvn};
  STAGE(launch_bq_linear_multi(x_i8, x_sa, T, nseg, wl, sl, ol, nl, S(stream)), "bq_qkv");
}

int gm_bq_block_quant_ex(const void* x, long rows, int cols, int block, int apply_fwht, int8_t* q, float* sa,
                         void* stream) {
  if (rows < 0 || cols <= 0 || !(block == 64 || block == 128 || block == 256 || block == 512) ||
      cols % block || (apply_fwht && block != 64))
    return set_err(nullptr, GM_EINVAL, "bq_block_quant_ex: rows=%ld cols=%d block=%d fwht=%d", rows, cols,
                   block, apply_fwht);
  STAGE(launch_block_quant_ex(static_cast<const uint16_t*>(x), rows, cols, block, apply_fwht, q, sa, S(stream)),
        "bq_block_quant_ex");
}

int gm_bq_block_linear_ex(const int8_t* h_i8, const float* h_sa, int T, int k, int block, const void* w,
                          const float* w_scale, int n_rows, void* out, void* stream) {
  if (T < 0 || !(block == 64 || block == 128 || block == 256 || block == 512) || k <= 0 || k % block ||
      ((k / block) % 4 && (k / block) % 3) || n_rows <= 0 || n_rows % 32 || (size_t)16 * (k + 16) > 200 * 1024)
    return set_err(nullptr, GM_EINVAL, "bq_block_linear_ex: T=%d k=%d block=%d n_rows=%d (k/block a "
                   "multiple of 4 or 3, k <= 12800, n_rows a multiple of 32)", T, k, block, n_rows);
  STAGE(launch_block_linear_ex(h_i8, h_sa, T, k, block, static_cast<const int8_t*>(w), w_scale, n_rows,
                               static_cast<uint16_t*>(out), S(stream)),
        "bq_block_linear_ex");
}

namespace {
int check_attn_geometry(int head_dim, int num_q, int num_kv, int cache_degree, int rank) {
  if (head_dim != 256 && head_dim != 512)
    return set_err(nullptr, GM_EINVAL, "attention: head_dim %d (256 or 512)", head_dim);
  if (num_q < 1 || num_kv < 1 || num_q % num_kv || (num_q / num_kv) % 2 || (num_q / num_kv) > 8)
    return set_err(nullptr, GM_EINVAL, "attention: num_q %d / num_kv %d (an even ratio <= 8)", num_q,
                   num_kv);
  if (cache_degree < 1 || rank < 0 || rank >= cache_degree)
    return set_err(nullptr, GM_EINVAL, "attention: cache_degree %d rank %d", cache_degree, rank);
  return GM_OK;
}
}  // namespace

int gm_bq_attn_prep(const void* q_src, const void* k_src, const void* v_src, const void* q_norm,
                    const void* k_norm, int8_t* q_i8, float* qi_bias, float* f_q, int8_t* k_cache,
                    float* k_scale, int8_t* v_cache, float* v_scale, const float* cos_table,
                    const float* sin_table, const gm_kv_run_t* runs, int num_runs,
                    const int32_t* base_rows, int T, int head_dim, int num_q, int num_kv,
                    int rope_half, int pair_stride, int cache_degree, int rank, int page_shift,
                    int row_mask, int page_mask, void* stream) {
  int rc = check_attn_geometry(head_dim, num_q, num_kv, cache_degree, rank);
  if (rc) return rc;
  if (T < 0 || (T > 0 && num_runs < 1)) return set_err(nullptr, GM_EINVAL, "attn_prep: T=%d runs=%d", T, num_runs);
  if (!((head_dim == 256 && rope_half == 128 && pair_stride == 128) ||
        (head_dim == 512 && rope_half == 64 && pair_stride == 256)))
    return set_err(nullptr, GM_EINVAL, "attn_prep: head_dim %d rope_half %d pair_stride %d is not a "
                   "Gemma-4 geometry", head_dim, rope_half, pair_stride);
  STAGE(launch_attn_prep(static_cast<const uint16_t*>(q_src), static_cast<const uint16_t*>(k_src),
                         static_cast<const uint16_t*>(v_src), static_cast<const uint16_t*>(q_norm),
                         static_cast<const uint16_t*>(k_norm), q_i8, qi_bias, f_q, k_cache, k_scale, v_cache,
                         v_scale, cos_table, sin_table, runs, num_runs, base_rows, T, head_dim, num_q, num_kv,
                         rope_half, pair_stride, cache_degree, rank, page_shift, row_mask, page_mask,
                         S(stream)),
        "bq_attn_prep");
}

size_t gm_bq_attention_workspace_bytes(int T, int head_dim, int num_q, int num_kv, int max_kv_len) {
  if (T <= 0 || num_kv <= 0) return 0;
  return attention_workspace_floats(T, head_dim, num_q, num_kv, max_kv_len) * sizeof(float);
}

int gm_bq_attention_decode(const int8_t* q_i8, const float* f_q, const int8_t* k_cache,
                           const float* k_scale, const int8_t* v_cache, const float* v_scale,
                           const gm_kv_run_t* runs, const int32_t* base_rows, int T, int head_dim,
                           int num_q, int num_kv, int window, int cache_degree, int rank,
                           int page_shift, int row_mask, int page_mask, int max_kv_len, void* out,
                           float* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_attn_geometry(head_dim, num_q, num_kv, cache_degree, rank);
  if (rc) return rc;
  if (T < 0 || window < 0 || max_kv_len < 0)
    return set_err(nullptr, GM_EINVAL, "attention_decode: T=%d window=%d max_kv_len=%d", T, window,
                   max_kv_len);
  // One GPU holds every position of its sequences.  A cache sharded by
  // position (the reference's full layers at degree > 1) would need each
  // rank's unnormalised partials (m, l, acc) merged across ranks, which this
  // entry point does not return, so it takes the whole cache only.
  if (cache_degree != 1)
    return set_err(nullptr, GM_EINVAL, "attention_decode: cache_degree %d (the decode takes an "
                   "unsharded cache: cache_degree 1)", cache_degree);
  const size_t need = gm_bq_attention_workspace_bytes(T, head_dim, num_q, num_kv, max_kv_len);
  if (workspace_bytes < need)
    return set_err(nullptr, GM_EINVAL, "attention_decode: workspace %zu bytes, %zu needed", workspace_bytes,
                   need);
  STAGE(launch_attn_decode(q_i8, f_q, k_cache, k_scale, v_cache, v_scale, runs, base_rows, T, head_dim, num_q,
                           num_kv, window, cache_degree, rank, page_shift, row_mask, page_mask, max_kv_len,
                           workspace, static_cast<uint16_t*>(out), S(stream)),
        "bq_attention_decode");
}

int gm_bq_attention_prefill(const int8_t* q_i8, const float* f_q, const int8_t* k_cache,
                            const float* k_scale, const int8_t* v_cache, const float* v_scale,
                            const gm_kv_run_t* runs, int num_runs, const int32_t* base_rows, int T,
                            int head_dim, int num_q, int num_kv, int window, int page_shift, int row_mask,
                            int page_mask, void* out, void* stream) {
  int rc = check_attn_geometry(head_dim, num_q, num_kv, 1, 0);
  if (rc) return rc;
  if (!((head_dim == 256 && num_q == 2 * num_kv) || (head_dim == 512 && num_q == 8 * num_kv)))
    return set_err(nullptr, GM_EINVAL, "attention_prefill: head_dim %d with %d query heads per KV head is not "
                   "a Gemma-4 geometry (256 x 2, 512 x 8)", head_dim, num_q / num_kv);
  if (T < 0 || window < 0 || (T > 0 && (num_runs < 1 || !runs || !out)))
    return set_err(nullptr, GM_EINVAL, "attention_prefill: T=%d window=%d num_runs=%d", T, window, num_runs);
  STAGE(launch_attn_prefill(q_i8, f_q, k_cache, k_scale, v_cache, v_scale, runs, num_runs, base_rows, T, head_dim,
                            num_q, num_kv, window, page_shift, row_mask, page_mask, static_cast<uint16_t*>(out),
                            S(stream)),
        "bq_attention_prefill");
}

size_t gm_bq_attention_partial_bytes(int T, int head_dim, int num_q) {
  if (T <= 0 || num_q <= 0 || (head_dim != 256 && head_dim != 512)) return 0;
  return (size_t)T * num_q * (head_dim + 2) * sizeof(float);
}

int gm_bq_attention_partial(const int8_t* q_i8, const float* f_q, const int8_t* k_cache,
                            const float* k_scale, const int8_t* v_cache, const float* v_scale,
                            const gm_kv_run_t* runs, const int32_t* base_rows, int T, int head_dim,
                            int num_q, int num_kv, int window, int cache_degree, int rank, int page_shift,
                            int row_mask, int page_mask, int max_kv_len, float* partial,
                            float* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_attn_geometry(head_dim, num_q, num_kv, cache_degree, rank);
  if (rc) return rc;
  if (T < 0 || window < 0 || max_kv_len < 0 || !partial)
    return set_err(nullptr, GM_EINVAL, "attention_partial: T=%d window=%d max_kv_len=%d", T, window, max_kv_len);
  if (cache_degree > 1 && window > 0)
    return set_err(nullptr, GM_EINVAL, "attention_partial: a sliding window keeps every position on each "
                   "rank (cache_degree 1)");
  const size_t need = gm_bq_attention_workspace_bytes(T, head_dim, num_q, num_kv, max_kv_len);
  if (workspace_bytes < need)
    return set_err(nullptr, GM_EINVAL, "attention_partial: workspace %zu bytes, %zu needed", workspace_bytes,
                   need);
  cudaError_t e = launch_attn_decode(q_i8, f_q, k_cache, k_scale, v_cache, v_scale, runs, base_rows, T,
                                     head_dim, num_q, num_kv, window, cache_degree, rank, page_shift, row_mask,
                                     page_mask, max_kv_len, workspace, nullptr, S(stream));
  if (e == cudaSuccess)
    e = launch_attn_rank_partial(workspace, T, num_q, head_dim, attention_splits(T, head_dim, num_q, num_kv, max_kv_len),
                                 partial, S(stream));
  return cuda_check(nullptr, e, "bq_attention_partial");
}

int gm_bq_attention_merge(const float* const* partials, int n_parts, int T, int num_q, int head_dim, void* out,
                          void* stream) {
  if (!partials || n_parts < 1 || n_parts > 8 || T < 0 || num_q <= 0 || (head_dim != 256 && head_dim != 512) ||
      !out)
    return set_err(nullptr, GM_EINVAL, "attention_merge: n_parts=%d (1..8) T=%d num_q=%d head_dim=%d", n_parts, T,
                   num_q, head_dim);
  for (int r = 0; r < n_parts; ++r)
    if (!partials[r]) return set_err(nullptr, GM_EINVAL, "attention_merge: partial %d is NULL", r);
  STAGE(launch_attn_merge_parts(partials, n_parts, T, num_q, head_dim, static_cast<uint16_t*>(out), S(stream)),
        "bq_attention_merge");
}

int gm_phase1_gate_up_bf16(const void* x_normed, const int32_t* expert_offset,
                           const gm_sparse_route_t* routes, const int32_t* chunk_off, int epr,
                           int T, const void* gate_up, void* bucket, void* stream) {
  if (epr < 1 || epr > E || T < 0) return set_err(nullptr, GM_EINVAL, "phase1_bf16: epr=%d T=%d", epr, T);
  STAGE(launch_bf16_phase1(static_cast<const uint16_t*>(x_normed), expert_offset,
                           reinterpret_cast<const SparseRoute*>(routes), chunk_off, epr, T,
                           static_cast<const uint16_t*>(gate_up), static_cast<uint16_t*>(bucket),
                           S(stream)),
        "phase1_gate_up_bf16");
}

int gm_phase2_down_bf16(const void* bucket, const int32_t* expert_offset,
                        const gm_sparse_route_t* routes, const int32_t* chunk_off, int epr, int T,
                        const void* down, float* y, void* stream) {
  if (epr < 1 || epr > E || T < 0) return set_err(nullptr, GM_EINVAL, "phase2_bf16: epr=%d T=%d", epr, T);
  STAGE(launch_bf16_phase2(static_cast<const uint16_t*>(bucket), expert_offset,
                           reinterpret_cast<const SparseRoute*>(routes), chunk_off, epr, T,
                           static_cast<const uint16_t*>(down), y, S(stream)),
        "phase2_down_bf16");
}

int gm_combine(const int32_t* route_idx, const int32_t* route_pos, const float* y, int T,
               void* out, void* stream) {
  STAGE(launch_combine(route_idx, route_pos, y, T, static_cast<uint16_t*>(out), S(stream)),
        "combine");
}

int gm_bq_quantize_rows(const void* w, long rows, int cols, const void* gamma, int fwht_block,
                        int8_t* q, float* scale, void* stream) {
  STAGE(launch_quantize_rows(static_cast<const uint16_t*>(w), rows, cols,
                             static_cast<const uint16_t*>(gamma), fwht_block, q, scale, S(stream)),
        "bq_quantize_rows");
}

int gm_vnni_pack(const int8_t* q, long rows, int cols, int8_t* packed, void* stream) {
  STAGE(launch_vnni_permute(q, rows, cols, packed, 0, S(stream)), "vnni_pack");
}

int gm_vnni_unpack(const int8_t* packed, long rows, int cols, int8_t* q, void* stream) {
  STAGE(launch_vnni_permute(packed, rows, cols, q, 1, S(stream)), "vnni_unpack");
}

int gm_router_center(const void* w, int rows, int cols, void* out, void* stream) {
  STAGE(launch_router_center(static_cast<const uint16_t*>(w), rows, cols,
                             static_cast<uint16_t*>(out), S(stream)),
        "router_center");
}

int gm_bake_split_gain(const void* g, void* out, int n, void* stream) {
  STAGE(launch_bake(static_cast<const uint16_t*>(g), static_cast<uint16_t*>(out), n, 0, S(stream)),
        "bake_split_gain");
}

int gm_bake_router_scale(const void* s, void* out, int n, void* stream) {
  STAGE(launch_bake(static_cast<const uint16_t*>(s), static_cast<uint16_t*>(out), n, 1, S(stream)),
        "bake_router_scale");
}

}  // extern "C"
