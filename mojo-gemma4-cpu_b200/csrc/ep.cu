// ep.cu -- expert-parallel dispatch and combine over NCCL (one process per GPU).
//
// The reference shards the experts by rank (modeling/gemma4_topology.mojo:
// 109-114) but replicates the activations and all-reduces the per-rank bf16
// partial outputs (modeling/gemma_4_moe_bq.mojo:711-713,
// kernels/reductions.mojo:186-204).  Here every rank keeps its own tokens:
//
//   plan     per token, the set of destination ranks (ranks owning one of its
//            8 experts) and its row in each destination's send block, in
//            token order;
//   pack     one row per (token, destination): the quantised activation row
//            (int8 + scale for butterquant, normalised bf16 for bf16 layers)
//            and the token's full top-8 (ids, weights); the receiver's
//            schedule keeps only its own experts.  Unused rows of a block get
//            expert id -1 (no local route);
//   dispatch NCCL send/recv of every block to its destination;
//   experts  the receiver's usual schedule -> expert products -> combine over
//            the received rows gives, per row, bf16(sum over its local
//            experts in ascending id order) -- the reference's per-rank
//            partial for that token;
//   combine  NCCL send/recv of the partial rows back to their source;
//   final    out[t] = bf16(sum over destination ranks in ascending order of
//            f32(partial)), the reference's all-reduce order (rank order,
//            kernels/reductions.mojo:88-93).
//
// Blocks have a fixed capacity (the handle's max_tokens rows per peer), so
// the exchange needs no host-side knowledge of the counts: the forward stays
// asynchronous and stream-ordered.
#include <dlfcn.h>
#include <nccl.h>

#include <mutex>
#include <string>

#include "combine_dev.cuh"
#include "ep.h"
#include "ep_dev.cuh"
#include "post_moe.cuh"

namespace gm {

// ------------------------------------------------------------- NCCL loader
namespace {
NcclApi g_nccl;
std::once_flag g_nccl_once;
std::string g_nccl_err;

template <typename F>
bool sym(void* lib, const char* name, F& f) {
  f = reinterpret_cast<F>(dlsym(lib, name));
  if (!f) g_nccl_err = std::string("NCCL symbol missing: ") + name;
  return f != nullptr;
}
}  // namespace

const NcclApi* nccl_api(const char** err) {
  std::call_once(g_nccl_once, [] {
    void* lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!lib) lib = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!lib) {
      g_nccl_err = std::string("cannot load libnccl.so.2: ") + dlerror();
      return;
    }
    bool ok = sym(lib, "ncclGetUniqueId", g_nccl.get_unique_id) &&
              sym(lib, "ncclCommInitRankConfig", g_nccl.comm_init_rank_config) &&
              sym(lib, "ncclCommDestroy", g_nccl.comm_destroy) &&
              sym(lib, "ncclCommAbort", g_nccl.comm_abort) &&
              sym(lib, "ncclCommGetAsyncError", g_nccl.comm_get_async_error) &&
              sym(lib, "ncclGroupStart", g_nccl.group_start) &&
              sym(lib, "ncclGroupEnd", g_nccl.group_end) && sym(lib, "ncclSend", g_nccl.send) &&
              sym(lib, "ncclRecv", g_nccl.recv) && sym(lib, "ncclAllGather", g_nccl.all_gather) &&
              sym(lib, "ncclGetErrorString", g_nccl.get_error_string);
    g_nccl.loaded = ok;
  });
  if (!g_nccl.loaded) {
    if (err) *err = g_nccl_err.c_str();
    return nullptr;
  }
  return &g_nccl;
}

// ------------------------------------------------------------- kernels
// One CTA of 1024 threads walks the tokens in chunks of 1024: per destination
// rank a block-wide exclusive scan of "token has a route there" gives the
// token's row in that destination's block (token order).
__global__ void __launch_bounds__(1024)
ep_plan_kernel(const int32_t* __restrict__ route_idx, int T, int G, int epr,
               const int32_t* __restrict__ rank_of, int32_t* __restrict__ pos,
               int32_t* __restrict__ count) {
  __shared__ int s_cnt[32];   // per-warp counts of the current destination
  __shared__ int s_pre[32];   // their exclusive prefix
  __shared__ int s_tot;       // chunk total
  __shared__ int s_base[8];   // rows already assigned per destination
  pdl_wait();
  pdl_trigger();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid < 8) s_base[tid] = 0;
  __syncthreads();
  for (int c0 = 0; c0 < T; c0 += 1024) {
    const int t = c0 + tid;
    uint32_t mask = 0;
    if (t < T) {
#pragma unroll
      for (int k = 0; k < TOPK; ++k) {
        const int e = route_idx[t * TOPK + k];
        if (e >= 0 && e < E) mask |= 1u << (rank_of ? __ldg(rank_of + e) : e / epr);
      }
    }
    for (int d = 0; d < G; ++d) {
      const bool f = (mask >> d) & 1u;
      const uint32_t b = __ballot_sync(0xffffffffu, f);
      const int below = __popc(b & ((1u << lane) - 1u));
      if (lane == 0) s_cnt[warp] = __popc(b);
      __syncthreads();
      if (warp == 0) {
        const int v = s_cnt[lane];
        int inc = v;
#pragma unroll
        for (int m = 1; m < 32; m <<= 1) {
          const int o = __shfl_up_sync(0xffffffffu, inc, m);
          if (lane >= m) inc += o;
        }
        s_pre[lane] = inc - v;
        if (lane == 31) s_tot = inc;
      }
      __syncthreads();
      if (t < T) pos[(size_t)t * G + d] = f ? s_base[d] + s_pre[warp] + below : -1;
      __syncthreads();
      if (tid == 0) s_base[d] += s_tot;
      __syncthreads();
    }
  }
  if (tid < G) count[tid] = s_base[tid];
}

// One warp per source token: copies its row into each destination block it
// routes to.  A grid-stride tail marks the unused rows of every block.
__global__ void __launch_bounds__(256)
ep_pack_kernel(const uint8_t* __restrict__ x_rows, int row_bytes, const float* __restrict__ x_sa,
               const int32_t* __restrict__ route_idx, const float* __restrict__ route_w, int T,
               int G, int cap, int epr, const int32_t* __restrict__ rank_of,
               const int32_t* __restrict__ local_of, const int32_t* __restrict__ pos,
               const int32_t* __restrict__ count, uint8_t* __restrict__ send_x,
               float* __restrict__ send_sa, int32_t* __restrict__ send_idx,
               float* __restrict__ send_w) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int warps = gridDim.x * (blockDim.x >> 5);
  for (int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < T; t += warps) {
    for (int d = 0; d < G; ++d) {
      const int p = pos[(size_t)t * G + d];
      if (p < 0) continue;
      const size_t row = (size_t)d * cap + p;
      const uint4* src = reinterpret_cast<const uint4*>(x_rows + (size_t)t * row_bytes);
      uint4* dst = reinterpret_cast<uint4*>(send_x + row * row_bytes);
      for (int i = lane; i < row_bytes / 16; i += 32) dst[i] = src[i];
      if (lane < TOPK) {
        int e = route_idx[t * TOPK + lane];
        if (rank_of && e >= 0 && e < E)
          e = __ldg(rank_of + e) == d ? d * epr + __ldg(local_of + e) : -1;
        send_idx[row * TOPK + lane] = e;
        send_w[row * TOPK + lane] = route_w[t * TOPK + lane];
      }
      if (lane == 0 && x_sa) send_sa[row] = x_sa[t];
    }
  }
  const size_t n = (size_t)G * cap;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    const int d = (int)(i / cap), p = (int)(i % cap);
    if (p >= count[d]) {
#pragma unroll
      for (int k = 0; k < TOPK; ++k) send_idx[i * TOPK + k] = -1;
    }
  }
}

// out[t] = bf16(sum over destinations d ascending of f32(contrib[d*cap + pos])).
__global__ void __launch_bounds__(352)
ep_final_kernel(const uint16_t* __restrict__ contrib, const int32_t* __restrict__ pos, int T, int G,
                int cap, uint16_t* __restrict__ out) {
  __shared__ int s_row[8];
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  if (threadIdx.x < 8) {
    const int d = threadIdx.x;
    const int p = d < G ? pos[(size_t)t * G + d] : -1;
    s_row[d] = p < 0 ? -1 : d * cap + p;
  }
  __syncthreads();
  for (int c4 = threadIdx.x; c4 < H / 4; c4 += blockDim.x) {
    float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
    for (int d = 0; d < G; ++d) {
      const int r = s_row[d];
      if (r < 0) continue;
      const uint2 v = *reinterpret_cast<const uint2*>(contrib + (size_t)r * H + c4 * 4);
      a0 = __fadd_rn(a0, bf2f(v.x & 0xFFFFu));
      a1 = __fadd_rn(a1, bf2f(v.x >> 16));
      a2 = __fadd_rn(a2, bf2f(v.y & 0xFFFFu));
      a3 = __fadd_rn(a3, bf2f(v.y >> 16));
    }
    uint2 o;
    o.x = (uint32_t)f2bf(a0) | ((uint32_t)f2bf(a1) << 16);
    o.y = (uint32_t)f2bf(a2) | ((uint32_t)f2bf(a3) << 16);
    *reinterpret_cast<uint2*>(out + (size_t)t * H + c4 * 4) = o;
  }
}

// ep_final followed by the post-MoE tail (post_moe.cuh) on the same row.
__global__ void __launch_bounds__(POST_THREADS)
ep_final_post_kernel(const uint16_t* __restrict__ contrib, const int32_t* __restrict__ pos, int T,
                     int G, int cap, PostParams p) {
  __shared__ int s_row[8];
  __shared__ float red[POST_THREADS / 32];
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  if (threadIdx.x < 8) {
    const int d = threadIdx.x;
    const int q = d < G ? pos[(size_t)t * G + d] : -1;
    s_row[d] = q < 0 ? -1 : d * cap + q;
  }
  __syncthreads();
  float m[8];
#pragma unroll
  for (int g = 0; g < 2; ++g) {
    const int c4 = threadIdx.x + g * POST_THREADS;
    float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
    for (int d = 0; d < G; ++d) {
      const int r = s_row[d];
      if (r < 0) continue;
      const uint2 v = *reinterpret_cast<const uint2*>(contrib + (size_t)r * H + c4 * 4);
      a0 = __fadd_rn(a0, bf2f(v.x & 0xFFFFu));
      a1 = __fadd_rn(a1, bf2f(v.x >> 16));
      a2 = __fadd_rn(a2, bf2f(v.y & 0xFFFFu));
      a3 = __fadd_rn(a3, bf2f(v.y >> 16));
    }
    m[4 * g] = bf2f(f2bf(a0));
    m[4 * g + 1] = bf2f(f2bf(a1));
    m[4 * g + 2] = bf2f(f2bf(a2));
    m[4 * g + 3] = bf2f(f2bf(a3));
  }
  post_moe_row(m, t, p, red);
}

cudaError_t launch_ep_final_post(const uint16_t* contrib, const int32_t* pos, int T, int G, int cap,
                                 const PostParams& p, cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  return launch_k(ep_final_post_kernel, dim3(T), dim3(POST_THREADS), 0, s, contrib, pos, T, G, cap, p);
}

// ------------------------------------------------- peer-memory exchange
__device__ __forceinline__ uint64_t ep_global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__global__ void __launch_bounds__(256)
ep_pack_p2p_kernel(const uint8_t* __restrict__ x_rows, int row_bytes, const float* __restrict__ x_sa,
                   const int32_t* __restrict__ route_idx, const float* __restrict__ route_w, int T,
                   int G, int cap, int epr, const int32_t* __restrict__ rank_of,
                   const int32_t* __restrict__ local_of, const int32_t* __restrict__ pos,
                   const int32_t* __restrict__ count, EpPeers peers, int my_rank, uint32_t epoch,
                   int* __restrict__ done_counter) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int warps = gridDim.x * (blockDim.x >> 5);
  const size_t src_row0 = (size_t)my_rank * cap;  // this source's block in every receiver
  for (int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < T; t += warps) {
    for (int d = 0; d < G; ++d) {
      const int p = pos[(size_t)t * G + d];
      if (p < 0) continue;
      const size_t row = src_row0 + p;
      const uint4* src = reinterpret_cast<const uint4*>(x_rows + (size_t)t * row_bytes);
      uint4* dst = reinterpret_cast<uint4*>(peers.recv_x[d] + row * row_bytes);
      for (int i = lane; i < row_bytes / 16; i += 32) dst[i] = src[i];
      if (lane < TOPK) {
        int e = route_idx[t * TOPK + lane];
        if (rank_of && e >= 0 && e < E)
          e = __ldg(rank_of + e) == d ? d * epr + __ldg(local_of + e) : -1;
        peers.recv_idx[d][row * TOPK + lane] = e;
        peers.recv_w[d][row * TOPK + lane] = route_w[t * TOPK + lane];
      }
      if (lane == 0 && x_sa) peers.recv_sa[d][row] = x_sa[t];
    }
  }
  // rows beyond each destination's count route nowhere
  const size_t n = (size_t)G * cap;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    const int d = (int)(i / cap), p = (int)(i % cap);
    if (p >= count[d]) {
#pragma unroll
      for (int k = 0; k < TOPK; ++k) peers.recv_idx[d][(src_row0 + p) * TOPK + k] = -1;
    }
  }
  publish_when_last(done_counter, peers.dflag, G, my_rank, epoch);
}

__global__ void ep_wait_kernel(const uint32_t* __restrict__ flags, int G, uint32_t epoch,
                               uint64_t limit_ns, int* __restrict__ err) {
  pdl_wait();
  pdl_trigger();
  if (threadIdx.x >= G) return;
  const uint64_t t0 = ep_global_ns();
  uint32_t it = 0;
  while ((int32_t)(ld_acquire_sys(flags + threadIdx.x) - epoch) < 0) {
    if ((++it & 255) == 0 && ep_global_ns() - t0 > limit_ns) {
      atomicExch(err, 3);  // a peer did not publish within the limit
      return;
    }
  }
  __threadfence_system();
}

__global__ void __launch_bounds__(352)
combine_p2p_kernel(const int32_t* __restrict__ route_idx, const int32_t* __restrict__ route_pos,
                   const float* __restrict__ ybuf, int n, int cap, EpPeers peers, int G, int my_rank,
                   uint32_t epoch, int* __restrict__ done_counter) {
  pdl_wait();
  pdl_trigger();
  for (int r = blockIdx.x; r < n; r += gridDim.x) {
    int pos[TOPK];
    routes_by_expert(route_idx, route_pos, r, pos);
    if (pos[0] < 0) continue;  // rows with no route here were never sent (or are unused)
    const int src = r / cap;
    uint16_t* dst = peers.contrib[src] + ((size_t)my_rank * cap + (r % cap)) * H;
    // 352 threads: two column groups each, loads of both in flight together
    float4 a0, a1;
    sum_routes4x2(ybuf, pos, threadIdx.x, threadIdx.x + H / 8, a0, a1);
    *reinterpret_cast<uint2*>(dst + threadIdx.x * 4) = pack_bf16x4(a0);
    *reinterpret_cast<uint2*>(dst + (threadIdx.x + H / 8) * 4) = pack_bf16x4(a1);
  }
  publish_when_last(done_counter, peers.cflag, G, my_rank, epoch);
}

cudaError_t launch_ep_pack_p2p(const void* x_rows, int row_bytes, const float* x_sa,
                               const int32_t* route_idx, const float* route_w, int T, int G, int cap,
                               int epr, EpPlacement pl, const int32_t* pos, const int32_t* count,
                               const EpPeers& peers, int my_rank, uint32_t epoch, int* done_counter,
                               cudaStream_t s) {
  const int blocks = std::max(1, std::min(1184, (std::max(T, G * cap) + 7) / 8));
  return launch_k(ep_pack_p2p_kernel, dim3(blocks), dim3(256), 0, s,
                  static_cast<const uint8_t*>(x_rows), row_bytes, x_sa, route_idx, route_w, T, G, cap,
                  epr, pl.rank_of, pl.local_of, pos, count, peers, my_rank, epoch, done_counter);
}

cudaError_t launch_ep_wait(const uint32_t* flags, int G, uint32_t epoch, uint64_t limit_ns, int* err,
                           cudaStream_t s) {
  return launch_k(ep_wait_kernel, dim3(1), dim3(32), 0, s, flags, G, epoch, limit_ns, err);
}

cudaError_t launch_combine_p2p(const int32_t* route_idx, const int32_t* route_pos, const float* ybuf,
                               int n, int cap, const EpPeers& peers, int G, int my_rank, uint32_t epoch,
                               int* done_counter, cudaStream_t s) {
  const int blocks = std::max(1, std::min(n, 148 * 8));
  return launch_k(combine_p2p_kernel, dim3(blocks), dim3(352), 0, s, route_idx, route_pos, ybuf, n, cap,
                  peers, G, my_rank, epoch, done_counter);
}

cudaError_t launch_ep_plan(const int32_t* route_idx, int T, int G, int epr, EpPlacement pl,
                           int32_t* pos, int32_t* count, cudaStream_t s) {
  return launch_k(ep_plan_kernel, dim3(1), dim3(1024), 0, s, route_idx, T, G, epr, pl.rank_of, pos,
                  count);
}

cudaError_t launch_ep_pack(const void* x_rows, int row_bytes, const float* x_sa,
                           const int32_t* route_idx, const float* route_w, int T, int G, int cap,
                           int epr, EpPlacement pl, const int32_t* pos, const int32_t* count,
                           void* send_x, float* send_sa, int32_t* send_idx, float* send_w,
                           cudaStream_t s) {
  const int blocks = std::max(1, std::min(1184, (std::max(T, G * cap) + 7) / 8));
  return launch_k(ep_pack_kernel, dim3(blocks), dim3(256), 0, s,
                  static_cast<const uint8_t*>(x_rows), row_bytes, x_sa, route_idx, route_w, T, G, cap,
                  epr, pl.rank_of, pl.local_of, pos, count, static_cast<uint8_t*>(send_x), send_sa,
                  send_idx, send_w);
}

cudaError_t launch_ep_final(const uint16_t* contrib, const int32_t* pos, int T, int G, int cap,
                            uint16_t* out, cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  return launch_k(ep_final_kernel, dim3(T), dim3(352), 0, s, contrib, pos, T, G, cap, out);
}

}  // namespace gm
