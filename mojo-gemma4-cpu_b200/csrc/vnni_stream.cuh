// vnni_stream.cuh -- streaming the reference's VNNI-packed int8 weights
// (butterquant/vnni.mojo:31-83: per 32-row N-tile and 64-col K-step a
// 2048-byte tile, two 16-row halves, byte (k/4)*64 + n*4 + k%4) straight into
// mma.m16n8k32 s8 A fragments with 128-bit no-L1 loads.  One lane load
// returns one 4-byte K-group for 4 consecutive rows; two such loads (K groups
// q and q+4 of a 32-wide K chunk) are the A fragments of two m16n8k32 tiles
// whose logical rows are permuted physical rows (acc_row gives the physical
// row of an accumulator element).
#pragma once
#include "gm_common.cuh"

namespace gm {

constexpr float INV127 = 1.0f / 127.0f;   // f32(1)/f32(127)

// Byte offset of lane (g,q)'s first 16-byte load inside a 2048-byte K-step
// tile, for K chunk cc (0/1) of that step.  The second load is +256 bytes.
__device__ __forceinline__ int vnni_lane_off(int g, int q, int cc) {
  return (g >> 2) * 1024 + (8 * cc + q) * 64 + (g & 3) * 16;
}

// Row (0..31) inside the N-tile of accumulator element i of MMA m for lane g.
__device__ __forceinline__ int acc_row(int g, int m, int i) {
  return 16 * (g >> 2) + 4 * (g & 3) + 2 * m + (i >> 1);
}

template <int DEPTH>
__device__ __forceinline__ void prefetch_chunks(uint4 (&buf)[DEPTH][2], const int8_t* wt, int c0,
                                                int g, int q) {
#pragma unroll
  for (int d = 0; d < DEPTH; ++d) {
    const int gc = c0 + d;
    const int8_t* p = wt + (gc >> 1) * 2048 + vnni_lane_off(g, q, gc & 1);
    buf[d][0] = ldg_stream(p);
    buf[d][1] = ldg_stream(p + 256);
  }
}

}  // namespace gm
