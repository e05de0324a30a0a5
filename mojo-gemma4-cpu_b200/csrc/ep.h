// ep.h -- expert-parallel exchange (ep.cu): NCCL entry points, loaded at run
// time so that single-GPU use needs no NCCL, and the plan/pack/final kernels.
#pragma once
#include <nccl.h>

#include "gm_kernels.h"
#include "post_moe.cuh"

namespace gm {

struct NcclApi {
  bool loaded = false;
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank_config)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*comm_abort)(ncclComm_t) = nullptr;
  ncclResult_t (*comm_get_async_error)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*group_start)() = nullptr;
  ncclResult_t (*group_end)() = nullptr;
  ncclResult_t (*send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  const char* (*get_error_string)(ncclResult_t) = nullptr;
};

// NCCL loaded on first use (nullptr and *err set when it cannot be).
const NcclApi* nccl_api(const char** err);

// Expert placement (device tables, E entries each): rank_of[e] = the rank
// holding expert e, local_of[e] = its index among that rank's experts.  Null
// tables mean the reference's contiguous blocks (rank e / epr, index e % epr).
struct EpPlacement {
  const int32_t* rank_of = nullptr;
  const int32_t* local_of = nullptr;
};
// pos[t][d]: row of token t in destination d's send block, or -1; count[d].
cudaError_t launch_ep_plan(const int32_t* route_idx, int T, int G, int epr, EpPlacement pl,
                           int32_t* pos, int32_t* count, cudaStream_t s);
// Pack the send blocks [G][cap] (rows of row_bytes; x_sa may be null).  With
// a placement, the ids sent to rank d are rewritten to d*epr + local index
// for d's experts and -1 for the others, so the receiver's contiguous
// schedule applies unchanged.
cudaError_t launch_ep_pack(const void* x_rows, int row_bytes, const float* x_sa,
                           const int32_t* route_idx, const float* route_w, int T, int G, int cap,
                           int epr, EpPlacement pl, const int32_t* pos, const int32_t* count,
                           void* send_x, float* send_sa, int32_t* send_idx, float* send_w,
                           cudaStream_t s);
// out[t] = bf16(sum_d f32(contrib[d*cap + pos[t][d]])), d ascending.
cudaError_t launch_ep_final(const uint16_t* contrib, const int32_t* pos, int T, int G, int cap,
                            uint16_t* out, cudaStream_t s);
// the same sum, then the post-MoE tail updating p.x_main
cudaError_t launch_ep_final_post(const uint16_t* contrib, const int32_t* pos, int T, int G, int cap,
                                 const PostParams& p, cudaStream_t s);

// Peer-memory exchange: the buffers of every rank (this rank's own at index
// rank), mapped into this process by CUDA IPC, for the current forward's
// parity.  dflag[r] / cflag[r] point at rank r's dispatch / combine flag
// arrays (one slot per source rank).
struct EpPeers {
  uint8_t* recv_x[8];
  float* recv_sa[8];
  int32_t* recv_idx[8];
  float* recv_w[8];
  uint16_t* contrib[8];
  uint32_t* dflag[8];
  uint32_t* cflag[8];
};

// Pack with peer stores: rows go straight into rank d's receive block of this
// source; the last CTA to finish (done_counter) publishes dflag[d][my_rank] =
// epoch on every rank d (release, system scope).
cudaError_t launch_ep_pack_p2p(const void* x_rows, int row_bytes, const float* x_sa,
                               const int32_t* route_idx, const float* route_w, int T, int G, int cap,
                               int epr, EpPlacement pl, const int32_t* pos, const int32_t* count,
                               const EpPeers& peers, int my_rank, uint32_t epoch, int* done_counter,
                               cudaStream_t s);
// Waits (bounded: limit_ns of the GPU's global timer) until flags[0..G) all
// reach epoch; on expiry writes 3 to *err and returns.
cudaError_t launch_ep_wait(const uint32_t* flags, int G, uint32_t epoch, uint64_t limit_ns, int* err,
                           cudaStream_t s);
// Combine with peer stores: received row r = (src, p) is summed over this
// rank's experts (ascending id, from 0.0, bf16) and written into rank src's
// contrib block of this rank; then cflag[src][my_rank] = epoch on every rank.
cudaError_t launch_combine_p2p(const int32_t* route_idx, const int32_t* route_pos, const float* ybuf,
                               int n, int cap, const EpPeers& peers, int G, int my_rank, uint32_t epoch,
                               int* done_counter, cudaStream_t s);

}  // namespace gm
