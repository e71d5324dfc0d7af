// Shared helpers for the mHC sm_100a kernels: status codes, the per-thread
// error string behind mhc_get_last_error_string(), warp reductions and the
// small per-token math every kernel family uses.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <stdarg.h>

#include "../../include/mhc_b200.h"

namespace mhc {

// Per-thread error string (the C-ABI is reentrant: no shared mutable state
// besides this thread-local buffer).
void set_error(const char* fmt, ...);

inline int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  set_error("%s", buf);
  return code;
}

// Checks the launch that was just issued; converts a CUDA error into a status.
inline int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    return fail(MHC_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
  }
  return MHC_OK;
}

// Kernel timing: RAII bracket that records CUDA events around a launch when
// profiling is enabled (mhc_profile_enable); a no-op branch otherwise.
bool profiling_enabled();
void profile_record(const char* name, cudaEvent_t start, cudaEvent_t stop);
cudaEvent_t profile_event();

struct ProfScope {
  const char* name;
  cudaStream_t stream;
  cudaEvent_t start = nullptr;
  ProfScope(const char* n, cudaStream_t s) : name(n), stream(s) {
    if (profiling_enabled()) {
      start = profile_event();
      if (start) cudaEventRecord(start, stream);
    }
  }
  ~ProfScope() {
    if (start) {
      cudaEvent_t stop = profile_event();
      if (stop) {
        cudaEventRecord(stop, stream);
        profile_record(name, start, stop);
      }
    }
  }
};

// Dynamic-forward helpers defined in layer.cu, used by the allocation-free
// entry point in noalloc.cu.
int fwd_dynamic_check_args(const char* what, int64_t B, int n, int64_t C, int iters,
                           float s_eps, float r_eps);
size_t fwd_dynamic_scratch_bytes(int64_t B, int n, int64_t C, bool need_rec);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

#define MHC_REQUIRE(cond, code, ...)          \
  do {                                        \
    if (!(cond)) return ::mhc::fail((code), __VA_ARGS__); \
  } while (0)

#define MHC_REQUIRE_PTR(p) MHC_REQUIRE((p) != nullptr, MHC_ERR_INVALID_ARG, "%s must not be NULL", #p)

inline int num_sms() {
  static thread_local int cached_dev = -1;
  static thread_local int cached_sms = 148;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev != cached_dev) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && v > 0)
      cached_sms = v;
    cached_dev = dev;
  }
  return cached_sms;
}

// ---------------------------------------------------------------------------
// Device helpers
// ---------------------------------------------------------------------------

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float sigmoidf_(float t) { return 1.0f / (1.0f + expf(-t)); }

// Sum `V` per-lane values over the 32 lanes of a warp.  On return lane 0 holds
// all V totals in acc[] (other lanes hold partial garbage).  Used only at the
// end of long loops, so the simple butterfly is cheap relative to the loop.
template <int V>
__device__ __forceinline__ void warp_sum_array(float (&acc)[V]) {
#pragma unroll
  for (int v = 0; v < V; ++v) acc[v] = warp_sum(acc[v]);
}

// Block-wide sum of V values per thread; result written to out[0..V) by
// thread 0 (and returned in shared `red` for every thread after the final
// __syncthreads).  `red` must hold (blockDim/32) * V floats.
template <int V>
__device__ __forceinline__ void block_sum_array(float (&acc)[V], float* red, float* out_shared) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
#pragma unroll
  for (int v = 0; v < V; ++v) {
    float s = warp_sum(acc[v]);
    if (lane == 0) red[warp * V + v] = s;
  }
  __syncthreads();
  for (int v = threadIdx.x; v < V; v += blockDim.x) {
    float s = 0.f;
    for (int w = 0; w < nwarps; ++w) s += red[w * V + v];
    out_shared[v] = s;
  }
  __syncthreads();
}

}  // namespace mhc
