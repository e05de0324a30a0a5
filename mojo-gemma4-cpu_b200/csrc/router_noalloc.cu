// router_noalloc.cu -- the router entry point for callers that cannot allocate.
//
// gm_router_select needs a caller-provided scratch buffer (split-K partial
// logits and the per-token inv_rms).  Some callers cannot produce one: code
// running where cudaMalloc is not allowed or not wanted (under an allocator
// that forbids device allocations, a runtime that hands out fixed memory
// pools only, or a foreign-language binding with no way to own device
// memory).  gm_router_select_noalloc keeps that scratch in a fixed array
// compiled into this library instead.  It still calls the CUDA runtime
// (symbol lookup, a memset, kernel launches), so it cannot be called where
// CUDA calls are forbidden, such as inside a stream's host function.
//
// The array lives in every GPU's memory once the library is loaded and stays
// there until the process exits.  All calls on one GPU share it and the last
// call's contents stay in it; calls that overlap on the GPU (different streams
// without ordering between them) race on it and must not be issued.  The
// array's device address is cached per device for the life of the process;
// cudaDeviceReset (or any teardown of the device's primary context) makes
// that cached address stale, so this entry point must not be called on a
// device after such a reset.
#include <cstdio>
#include <mutex>

#include "../../include/gmoe.h"
#include "gm_kernels.h"

namespace gm {

// Largest T the shared scratch holds: 11 K-slices x 256 tokens x 128 experts of
// partial logits plus 256 inv_rms values = 360,704 floats (1.38 MiB).
constexpr int NOALLOC_MAX_TOKENS = 256;
constexpr size_t NOALLOC_SCRATCH_FLOATS =
    (size_t)(H / 256) * NOALLOC_MAX_TOKENS * E + NOALLOC_MAX_TOKENS + NOALLOC_MAX_TOKENS / 8 * (E / 32);

static __device__ __align__(256) float g_router_scratch[NOALLOC_SCRATCH_FLOATS];

namespace {

constexpr int MAX_DEVICES = 64;
std::mutex g_mu;
float* g_scratch_ptr[MAX_DEVICES] = {};

// Device address of g_router_scratch on the current device.  The host-side
// name of the array is not a device address, so it is looked up once per
// device with that device current.
cudaError_t scratch_for_current_device(float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= MAX_DEVICES) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_router_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_scratch_ptr[dev];
  return cudaSuccess;
}

// The failure text goes where gm_last_error(NULL) reads it.
int fail(int code, const char* msg, cudaError_t e = cudaSuccess) {
  char buf[256];
  snprintf(buf, sizeof buf, "%s%s%s", msg, e != cudaSuccess ? ": " : "",
           e != cudaSuccess ? cudaGetErrorString(e) : "");
  set_thread_error(buf);
  return code;
}

}  // namespace
}  // namespace gm

extern "C" {

int gm_router_select_noalloc(const void* x, const void* router_w, const void* router_scale,
                             const void* per_expert_scale, int T, int32_t* route_idx,
                             float* route_w, void* stream) {
  using namespace gm;
  if (T < 0 || T > NOALLOC_MAX_TOKENS)
    return fail(GM_EINVAL, "gm_router_select_noalloc: T outside [0, 256], the fixed scratch limit");
  if (T == 0) return GM_OK;
  if (!x || !router_w || !router_scale || !per_expert_scale || !route_idx || !route_w)
    return fail(GM_EINVAL, "gm_router_select_noalloc: NULL pointer");
  float* scratch = nullptr;
  cudaError_t e = scratch_for_current_device(&scratch);
  if (e != cudaSuccess)
    return fail(GM_ECUDA, "gm_router_select_noalloc: cudaGetSymbolAddress of the scratch failed", e);
  // Every scratch element a later kernel reads is written earlier in the same
  // call (inv_rms, then all K-slice partials); the logit kernel's tile
  // counters (after inv_rms) are cleared here.
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const uint16_t* xb = static_cast<const uint16_t*>(x);
  float* inv = scratch + (size_t)ROUTER_SLICES * T * E;
  int* counters = reinterpret_cast<int*>(inv + T);
  e = cudaMemsetAsync(counters, 0, sizeof(int) * router_tile_counters(T), s);
  if (e == cudaSuccess) e = launch_rms_inv(xb, T, inv, s);
  if (e == cudaSuccess)
    e = launch_router_logits(xb, static_cast<const uint16_t*>(router_w),
                             static_cast<const uint16_t*>(router_scale), T, scratch, nullptr, counters, s);
  if (e == cudaSuccess)
    e = launch_topk(scratch, static_cast<const uint16_t*>(per_expert_scale), inv, T, route_idx, route_w, s);
  if (e != cudaSuccess) return fail(GM_ECUDA, "gm_router_select_noalloc: launch failed", e);
  return GM_OK;
}

}  // extern "C"
