// schedule.cu -- token-to-expert dispatch schedule.
//
// Reference: kernels/moe_router.mojo:72-101 (BuildScheduleKernel): histogram of
// the routes that fall in this rank's expert range, exclusive prefix sum into
// expert_offset[epr+1], then a STABLE permute (token-major, then slot k) of
// SparseRoute{token, weight} records into per-expert segments.
//
// B200 shape: one 1024-thread CTA.  The histogram uses shared-memory atomics;
// the stable rank of a route inside its expert segment is computed per
// 1024-token chunk from per-expert token bitmasks (popcount of the bits below
// the token), so the output order is exactly the reference's sequential order.
// Extra outputs for the GPU pipeline: route_pos[t*8+k] (segment position of
// each route, -1 if the expert is not local) and chunk_off[epr+1] (prefix of
// ceil(n_e / route_chunk), the work decomposition of the expert kernels).
#include "gm_kernels.h"
#include "router_dev.cuh"

namespace gm {

struct ScheduleSmem {
  int cnt[E];
  int base[E];
  uint32_t mask[E][33];  // padded: thread e scans row e without bank conflicts
  int wpre[E][33];
};

// Body shared by the schedule kernel and the fused top-8 + schedule kernel
// (one CTA of 1024 threads).
__device__ void schedule_body(const int32_t* __restrict__ route_idx,
                              const float* __restrict__ route_w, int T, int expert_base, int epr,
                              int route_chunk, int32_t* __restrict__ expert_offset,
                              SparseRoute* __restrict__ routes, int32_t* __restrict__ route_pos,
                              int32_t* __restrict__ chunk_off, ScheduleSmem& sm) {
  int* cnt = sm.cnt;
  int* base = sm.base;
  auto& mask = sm.mask;
  auto& wpre = sm.wpre;
  const int tid = threadIdx.x;
  for (int e = tid; e < E; e += 1024) cnt[e] = 0;
  __syncthreads();
  const int R = T * TOPK;
  for (int i = tid; i < R; i += 1024) {
    int e = route_idx[i] - expert_base;
    if (e >= 0 && e < epr) atomicAdd(&cnt[e], 1);
  }
  __syncthreads();
  if (tid < 32) {
    // warp-level exclusive scans over <=128 experts (4 per lane)
    int c[4], cc[4];
    int s = 0, sc = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      int e = tid * 4 + j;
      c[j] = e < epr ? cnt[e] : 0;
      cc[j] = e < epr ? (c[j] + route_chunk - 1) / route_chunk : 0;
      s += c[j];
      sc += cc[j];
    }
    int inc = s, incc = sc;
#pragma unroll
    for (int m = 1; m < 32; m <<= 1) {
      int o = __shfl_up_sync(0xffffffffu, inc, m);
      int oc = __shfl_up_sync(0xffffffffu, incc, m);
      if (tid >= m) { inc += o; incc += oc; }
    }
    int run = inc - s, crun = incc - sc;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      int e = tid * 4 + j;
      if (e < epr) {
        expert_offset[e] = run;
        base[e] = run;
        chunk_off[e] = crun;
      }
      run += c[j];
      crun += cc[j];
    }
    if (tid == 31) {
      expert_offset[epr] = run;
      chunk_off[epr] = crun;
    }
  }
  __syncthreads();

  for (int c0 = 0; c0 < T; c0 += 1024) {
    const int nw = min(32, (T - c0 + 31) >> 5);  // mask words holding this chunk's tokens
    for (int i = tid; i < epr * 32; i += 1024) mask[i >> 5][i & 31] = 0u;
    __syncthreads();
    const int t = c0 + tid;
    int le[TOPK];
#pragma unroll
    for (int k = 0; k < TOPK; ++k) {
      le[k] = -1;
      if (t < T) {
        int e = route_idx[t * TOPK + k] - expert_base;
        if (e >= 0 && e < epr) {
          le[k] = e;
          atomicOr(&mask[e][tid >> 5], 1u << (tid & 31));
        }
      }
    }
    __syncthreads();
    if (tid < epr) {
      int s = 0;
      for (int w = 0; w < nw; ++w) {
        wpre[tid][w] = s;
        s += __popc(mask[tid][w]);
      }
      wpre[tid][32] = s;
    }
    __syncthreads();
    if (t < T) {
#pragma unroll
      for (int k = 0; k < TOPK; ++k) {
        int pos = -1;
        int e = le[k];
        if (e >= 0) {
          pos = base[e] + wpre[e][tid >> 5] +
                __popc(mask[e][tid >> 5] & ((1u << (tid & 31)) - 1u));
          routes[pos] = SparseRoute{t, route_w[t * TOPK + k]};
        }
        route_pos[t * TOPK + k] = pos;
      }
    }
    __syncthreads();
    if (tid < epr) base[tid] += wpre[tid][32];
    __syncthreads();
  }
}

__global__ void __launch_bounds__(1024)
build_schedule_kernel(const int32_t* __restrict__ route_idx, const float* __restrict__ route_w,
                      int T, int expert_base, int epr, int route_chunk,
                      int32_t* __restrict__ expert_offset, SparseRoute* __restrict__ routes,
                      int32_t* __restrict__ route_pos, int32_t* __restrict__ chunk_off) {
  __shared__ ScheduleSmem sm;
  pdl_wait();
  pdl_trigger();
  schedule_body(route_idx, route_w, T, expert_base, epr, route_chunk, expert_offset, routes,
                route_pos, chunk_off, sm);
}

// Top-8 selection of every token (32 warps, one token per warp at a time) and
// then the schedule, in one CTA: for decode-sized T this saves a launch and a
// round trip of the routes through a separate kernel boundary.
__global__ void __launch_bounds__(1024)
topk_schedule_kernel(float* __restrict__ logits, int ksplit, const uint16_t* __restrict__ pes,
                     const float* __restrict__ inv_rms, int T, int32_t* __restrict__ route_idx,
                     float* __restrict__ route_w,
                     int expert_base, int epr, int route_chunk, int32_t* __restrict__ expert_offset,
                     SparseRoute* __restrict__ routes, int32_t* __restrict__ route_pos,
                     int32_t* __restrict__ chunk_off) {
  __shared__ ScheduleSmem sm;
  pdl_wait();
  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int t = warp; t < T; t += 32)
    topk_token(logits, ksplit, pes, inv_rms, T, t, lane, route_idx, route_w);
  __syncthreads();  // route_idx / route_w written by this CTA are now visible to it
  schedule_body(route_idx, route_w, T, expert_base, epr, route_chunk, expert_offset, routes,
                route_pos, chunk_off, sm);
}

// ---- multi-CTA schedule for large T: chunks of 256 tokens, one CTA each.
// Pass 1 counts the local routes of every expert per chunk; pass 2 derives
// each chunk's first position per expert (expert prefix + earlier chunks) and
// places its routes with the same bitmask/popcount ranking, so the order is
// the reference's sequential token-major order.
constexpr int SCHED_CHUNK = 256;

__global__ void __launch_bounds__(SCHED_CHUNK)
schedule_count_kernel(const int32_t* __restrict__ route_idx, int T, int expert_base, int epr,
                      int32_t* __restrict__ counts) {
  __shared__ int cnt[E];
  pdl_wait();
  pdl_trigger();
  const int tid = threadIdx.x, c = blockIdx.x;
  if (tid < E) cnt[tid] = 0;
  __syncthreads();
  const int t = c * SCHED_CHUNK + tid;
  if (t < T) {
#pragma unroll
    for (int k = 0; k < TOPK; ++k) {
      const int e = route_idx[t * TOPK + k] - expert_base;
      if (e >= 0 && e < epr) atomicAdd(&cnt[e], 1);
    }
  }
  __syncthreads();
  if (tid < E) counts[(size_t)c * E + tid] = tid < epr ? cnt[tid] : 0;
}

__global__ void __launch_bounds__(SCHED_CHUNK)
schedule_scatter_kernel(const int32_t* __restrict__ route_idx, const float* __restrict__ route_w,
                        int T, int expert_base, int epr, int route_chunk,
                        const int32_t* __restrict__ counts, int nchunks,
                        int32_t* __restrict__ expert_offset, SparseRoute* __restrict__ routes,
                        int32_t* __restrict__ route_pos, int32_t* __restrict__ chunk_off) {
  __shared__ int tot[E], before[E], base[E];
  __shared__ uint32_t mask[E][SCHED_CHUNK / 32];
  __shared__ int wpre[E][SCHED_CHUNK / 32 + 1];
  pdl_wait();
  pdl_trigger();
  const int tid = threadIdx.x, c = blockIdx.x;
  if (tid < E) {
    int s = 0, b = 0;
    if (tid < epr)
      for (int cc = 0; cc < nchunks; ++cc) {
        const int v = counts[(size_t)cc * E + tid];
        if (cc < c) b += v;
        s += v;
      }
    tot[tid] = s;
    before[tid] = b;
  }
  for (int i = tid; i < E * (SCHED_CHUNK / 32); i += SCHED_CHUNK) mask[i / (SCHED_CHUNK / 32)][i % (SCHED_CHUNK / 32)] = 0u;
  __syncthreads();
  if (tid < 32) {
    int cv[4], cc4[4], s = 0, sc = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int e = tid * 4 + j;
      cv[j] = e < epr ? tot[e] : 0;
      cc4[j] = e < epr ? (cv[j] + route_chunk - 1) / route_chunk : 0;
      s += cv[j];
      sc += cc4[j];
    }
    int inc = s, incc = sc;
#pragma unroll
    for (int m = 1; m < 32; m <<= 1) {
      const int o = __shfl_up_sync(0xffffffffu, inc, m);
      const int oc = __shfl_up_sync(0xffffffffu, incc, m);
      if (tid >= m) { inc += o; incc += oc; }
    }
    int run = inc - s, crun = incc - sc;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int e = tid * 4 + j;
      if (e < epr) {
        base[e] = run + before[e];
        if (c == 0) {
          expert_offset[e] = run;
          chunk_off[e] = crun;
        }
      }
      run += cv[j];
      crun += cc4[j];
    }
    if (c == 0 && tid == 31) {
      expert_offset[epr] = run;
      chunk_off[epr] = crun;
    }
  }
  const int t = c * SCHED_CHUNK + tid;
  int le[TOPK];
#pragma unroll
  for (int k = 0; k < TOPK; ++k) {
    le[k] = -1;
    if (t < T) {
      const int e = route_idx[t * TOPK + k] - expert_base;
      if (e >= 0 && e < epr) {
        le[k] = e;
        atomicOr(&mask[e][tid >> 5], 1u << (tid & 31));
      }
    }
  }
  __syncthreads();
  if (tid < epr) {
    int s = 0;
#pragma unroll
    for (int w = 0; w < SCHED_CHUNK / 32; ++w) {
      wpre[tid][w] = s;
      s += __popc(mask[tid][w]);
    }
  }
  __syncthreads();
  if (t < T) {
#pragma unroll
    for (int k = 0; k < TOPK; ++k) {
      int pos = -1;
      const int e = le[k];
      if (e >= 0) {
        pos = base[e] + wpre[e][tid >> 5] + __popc(mask[e][tid >> 5] & ((1u << (tid & 31)) - 1u));
        routes[pos] = SparseRoute{t, route_w[t * TOPK + k]};
      }
      route_pos[t * TOPK + k] = pos;
    }
  }
}

int schedule_counts_ints(int T) { return ((T + SCHED_CHUNK - 1) / SCHED_CHUNK) * E; }

cudaError_t launch_schedule_multi(const int32_t* route_idx, const float* route_w, int T,
                                  int expert_base, int epr, int route_chunk, int32_t* counts,
                                  int32_t* expert_offset, SparseRoute* routes, int32_t* route_pos,
                                  int32_t* chunk_off, cudaStream_t s) {
  const int nchunks = (T + SCHED_CHUNK - 1) / SCHED_CHUNK;
  cudaError_t e = launch_k(schedule_count_kernel, dim3(nchunks), dim3(SCHED_CHUNK), 0, s, route_idx,
                           T, expert_base, epr, counts);
  if (e != cudaSuccess) return e;
  return launch_k(schedule_scatter_kernel, dim3(nchunks), dim3(SCHED_CHUNK), 0, s, route_idx,
                  route_w, T, expert_base, epr, route_chunk, (const int32_t*)counts, nchunks,
                  expert_offset, routes, route_pos, chunk_off);
}

cudaError_t launch_build_schedule(const int32_t* route_idx, const float* route_w, int T,
                                  int expert_base, int epr, int route_chunk,
                                  int32_t* expert_offset, SparseRoute* routes, int32_t* route_pos,
                                  int32_t* chunk_off, cudaStream_t s) {
  return launch_k(build_schedule_kernel, dim3(1), dim3(1024), 0, s, route_idx, route_w, T,
                  expert_base, epr, route_chunk, expert_offset, routes, route_pos, chunk_off);
}

cudaError_t launch_topk_schedule(float* logits, const uint16_t* pes, const float* inv_rms, int T,
                                 int32_t* route_idx, float* route_w, int expert_base, int epr,
                                 int route_chunk, int32_t* expert_offset, SparseRoute* routes,
                                 int32_t* route_pos, int32_t* chunk_off, int32_t* counts, cudaStream_t s) {
  // one CTA up to TOPK_SCHEDULE_FUSED_MAX tokens (32 warps, one token each;
  // the router has reduced its K slices); above, the top-8 is spread over
  // T/4 CTAs first
  if (T <= TOPK_SCHEDULE_FUSED_MAX)
    return launch_k(topk_schedule_kernel, dim3(1), dim3(1024), 0, s, logits, router_ksplit(T), pes,
                    inv_rms, T, route_idx, route_w, expert_base, epr, route_chunk, expert_offset, routes,
                    route_pos, chunk_off);
  cudaError_t e = launch_topk(logits, pes, inv_rms, T, route_idx, route_w, s);
  if (e != cudaSuccess) return e;
  if (counts && T > 1024)
    return launch_schedule_multi(route_idx, route_w, T, expert_base, epr, route_chunk, counts,
                                 expert_offset, routes, route_pos, chunk_off, s);
  return launch_build_schedule(route_idx, route_w, T, expert_base, epr, route_chunk, expert_offset,
                               routes, route_pos, chunk_off, s);
}

cudaError_t launch_topk_inv_schedule(const uint16_t* x, float* logits, const uint16_t* pes, float* inv_rms,
                                     int T, int32_t* route_idx, float* route_w, int expert_base, int epr,
                                     int route_chunk, int32_t* expert_offset, SparseRoute* routes,
                                     int32_t* route_pos, int32_t* chunk_off, int32_t* counts, cudaStream_t s) {
  cudaError_t e = launch_topk_inv(x, logits, pes, inv_rms, T, route_idx, route_w, s);
  if (e != cudaSuccess) return e;
  if (counts && T > 1024)
    return launch_schedule_multi(route_idx, route_w, T, expert_base, epr, route_chunk, counts,
                                 expert_offset, routes, route_pos, chunk_off, s);
  return launch_build_schedule(route_idx, route_w, T, expert_base, epr, route_chunk, expert_offset,
                               routes, route_pos, chunk_off, s);
}

}  // namespace gm
