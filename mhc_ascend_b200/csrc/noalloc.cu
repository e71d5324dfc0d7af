// Allocation-free entry point for the dynamic-H layer forward.
//
// Some callers of this library cannot hand it a workspace: a C host with no
// device allocator of its own, a serving process that reserved all of its
// device memory at start-up and must not allocate afterwards, or a real-time
// path that cannot afford cudaMalloc / cudaFree (they can synchronise the
// whole device).  mhc_layer_fwd_dynamic_noalloc() serves them: it runs the
// same kernels as mhc_layer_fwd_dynamic() with its scratch taken from a
// fixed-size array that lives in this library's device image.
//
// The array below is a device variable.  In host code its name is only a
// host-side stand-in for it, not a device address; the device address is
// looked up with cudaGetSymbolAddress() once per device, on the first call
// made while that device is current, and cached.  That first call therefore
// does more than launch kernels (it may load the module on the device): make
// it before any stream capture.  Every later call on the device reuses the
// cached address and the same array, so calls whose kernels overlap on the
// GPU (different streams, or several host threads) race on the scratch and
// must be serialised by the caller.  The array keeps whatever the previous
// call left in it; this entry point needs no zeroed scratch, because every
// scratch word a call reads was written earlier in that same call.
#include "common.cuh"

#include <mutex>

namespace {

// Fixed scratch capacity: 16 MiB per device that loads the library, held
// until the process exits.  What fits depends on the shape and on the SM
// count (the projection's split plan follows it): on a 148-SM B200 at n = 4,
// C = 4096 about 20k tokens when the caller keeps token_state and about 16k
// when the record lives in the scratch too (C = 7168: ~10.7k / ~5.4k).
constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 128;
std::mutex g_noalloc_mu;
void* g_noalloc_addr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device (looked up once).
int noalloc_scratch(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess)
    return mhc::fail(MHC_ERR_CUDA, "mhc_layer_fwd_dynamic_noalloc: cudaGetDevice failed: %s",
                     cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices)
    return mhc::fail(MHC_ERR_UNSUPPORTED, "mhc_layer_fwd_dynamic_noalloc: device %d out of range",
                     dev);
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (g_noalloc_addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
      return mhc::fail(MHC_ERR_CUDA,
                       "mhc_layer_fwd_dynamic_noalloc: cudaGetSymbolAddress failed on device %d: %s",
                       dev, cudaGetErrorString(e));
    g_noalloc_addr[dev] = p;
  }
  *out = g_noalloc_addr[dev];
  return MHC_OK;
}

}  // namespace

extern "C" int mhc_layer_fwd_dynamic_noalloc(
    const float* x, const float* rmsnorm_weight, const float* phi_pre, const float* phi_post,
    const float* phi_res, const float* alpha_pre, const float* alpha_post, const float* alpha_res,
    const float* b_pre, const float* b_post, const float* b_res, float* out, float* token_state,
    int64_t batch, int32_t n, int64_t hidden, int32_t sinkhorn_iters, float sinkhorn_eps,
    float rmsnorm_eps, void* stream) {
  // Bad arguments are reported as such, before the size check or any device call.
  int rc = mhc::fwd_dynamic_check_args("mhc_layer_fwd_dynamic_noalloc", batch, n, hidden,
                                       sinkhorn_iters, sinkhorn_eps, rmsnorm_eps);
  if (rc) return rc;
  if (batch == 0)  // nothing to compute: pointer checks only, no device work
    return mhc_layer_fwd_dynamic(x, rmsnorm_weight, phi_pre, phi_post, phi_res, alpha_pre,
                                 alpha_post, alpha_res, b_pre, b_post, b_res, out, token_state,
                                 batch, n, hidden, sinkhorn_iters, sinkhorn_eps, rmsnorm_eps,
                                 nullptr, 0, stream);
  // Exact need of this call: the token record is scratch only without token_state.
  const size_t need =
      mhc::fwd_dynamic_scratch_bytes(batch, n, hidden, token_state == nullptr);
  if (need > kNoAllocScratchBytes)
    return mhc::fail(MHC_ERR_UNSUPPORTED,
                     "mhc_layer_fwd_dynamic_noalloc: batch=%lld n=%d hidden=%lld needs %zu bytes of "
                     "scratch, more than the fixed %zu; use mhc_layer_fwd_dynamic with a workspace "
                     "or split the batch",
                     (long long)batch, n, (long long)hidden, need, kNoAllocScratchBytes);
  void* scratch = nullptr;
  rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  return mhc_layer_fwd_dynamic(x, rmsnorm_weight, phi_pre, phi_post, phi_res, alpha_pre,
                               alpha_post, alpha_res, b_pre, b_post, b_res, out, token_state,
                               batch, n, hidden, sinkhorn_iters, sinkhorn_eps, rmsnorm_eps,
                               scratch, kNoAllocScratchBytes, stream);
}
