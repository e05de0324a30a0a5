// ep_dev.cuh -- device side of the peer-memory exchange shared by the
// exchange kernels (ep.cu) and the kernels that store into peers' buffers
// themselves (the fused combine of gemm_tc.cu): system-scope release/acquire
// flag accesses and the "last CTA publishes" step.
#pragma once
#include <cstdint>

namespace gm {

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Called by every thread of a CTA after its peer stores: the last CTA of the
// grid (done_counter) publishes `epoch` into flag[d][my_rank] of every rank d.
__device__ __forceinline__ void publish_when_last(int* done_counter, uint32_t* const* flags, int G,
                                                  int my_rank, uint32_t epoch) {
  __shared__ int s_last;
  __threadfence_system();  // this thread's peer stores are visible system-wide
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(done_counter, 1) == (int)gridDim.x - 1;
  __syncthreads();
  if (s_last && threadIdx.x < G) {
    __threadfence_system();
    st_release_sys(flags[threadIdx.x] + my_rank, epoch);
    if (threadIdx.x == 0) *done_counter = 0;  // re-armed for the next forward
  }
}

}  // namespace gm
