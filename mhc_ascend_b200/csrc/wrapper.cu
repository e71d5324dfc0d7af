// Stream packing and stream mean of MHCResidualWrapper (reference
// layer.py:287-316), each one HBM pass instead of a chain of framework ops.
//
//   pack : x[t, i, c] = i == 1 ? branch[t, c] : s_i * residual[t, c]
//          (s_0 = 1; s_i = 0.1^(i-1) in "decay" mode, 0 in "zero" mode; a
//          zero scale writes 0, like the reference's zeros_like)
//   pack reverse : g_res = sum_{i != 1, s_i != 0} s_i g[t, i, c], g_branch = g[t, 1, c]
//   mean : out[t, c] = (sum_i x[t, i, c]) / n        reverse: g_x[t, i, c] = g[t, c] / n
//          (true divisions, as the framework's mean and its gradient)
//
// The scales arrive from the host (n <= 64 values) and travel as a kernel
// argument.  All loops are grid-stride over (token, channel) with float4
// accesses when C % 4 == 0 and the pointers are 16-byte aligned.
#include "common.cuh"

#include <cuda_bf16.h>

namespace mhc {
namespace {

constexpr int kMaxStreams = 64;

// grid of a grid-stride loop over `work` items: 16 blocks of 256 per SM at most
inline unsigned grid_for(int64_t work) {
  int64_t g = (work + 255) / 256;
  if (g < 1) g = 1;
  if (g > 148 * 16) g = 148 * 16;
  return (unsigned)g;
}

struct Scales {
  float s[kMaxStreams];
};

__device__ __forceinline__ float bf16_round(float v) {
  return __bfloat162float(__float2bfloat16_rn(v));
}

__device__ __forceinline__ float4 scale4(float s, float4 v) {
  return make_float4(s * v.x, s * v.y, s * v.z, s * v.w);
}

template <bool VEC>
__global__ void __launch_bounds__(256)
    pack_fwd_kernel(const float* __restrict__ res, const float* __restrict__ br,
                    float* __restrict__ out, int64_t T, int n, int64_t C, Scales sc) {
  const int64_t Cq = VEC ? C / 4 : C;
  const int64_t total = T * Cq;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = e / Cq, q = e - t * Cq;
    if (VEC) {
      const float4 r = __ldg(reinterpret_cast<const float4*>(res) + e);
      float4* o = reinterpret_cast<float4*>(out) + t * n * Cq + q;
      for (int i = 0; i < n; ++i) {
        float4 v;
        if (i == 1) v = __ldg(reinterpret_cast<const float4*>(br) + e);
        else if (i == 0) v = r;
        else if (sc.s[i] == 0.f) v = make_float4(0.f, 0.f, 0.f, 0.f);
        else v = scale4(sc.s[i], r);
        o[i * Cq] = v;
      }
    } else {
      const float r = res[e];
      float* o = out + t * n * C + q;
      for (int i = 0; i < n; ++i)
        o[i * C] = i == 1 ? br[e] : (i == 0 ? r : (sc.s[i] == 0.f ? 0.f : sc.s[i] * r));
    }
  }
}

// bf16 residual / branch (the reference packs in residual.dtype, layer.py:299-308):
// streams i >= 2 are s_i * residual rounded to bf16 -- a bf16 tensor times a
// Python float is computed in fp32 and rounded to bf16 -- then widened to the
// fp32 layer input, as the reference's x.float() (layer.py:101) does.
template <bool VEC>
__global__ void __launch_bounds__(256)
    pack_fwd_bf16_kernel(const __nv_bfloat16* __restrict__ res,
                         const __nv_bfloat16* __restrict__ br, float* __restrict__ out,
                         int64_t T, int n, int64_t C, Scales sc) {
  const int64_t Cq = VEC ? C / 4 : C;
  const int64_t total = T * Cq;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = e / Cq, q = e - t * Cq;
    if (VEC) {
      const uint2 rr = __ldg(reinterpret_cast<const uint2*>(res) + e);
      const __nv_bfloat162* r2 = reinterpret_cast<const __nv_bfloat162*>(&rr);
      const float2 ra = __bfloat1622float2(r2[0]), rb = __bfloat1622float2(r2[1]);
      const float4 r = make_float4(ra.x, ra.y, rb.x, rb.y);
      float4* o = reinterpret_cast<float4*>(out) + t * n * Cq + q;
      for (int i = 0; i < n; ++i) {
        float4 v;
        if (i == 1) {
          const uint2 bb = __ldg(reinterpret_cast<const uint2*>(br) + e);
          const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&bb);
          const float2 ba = __bfloat1622float2(b2[0]), bc = __bfloat1622float2(b2[1]);
          v = make_float4(ba.x, ba.y, bc.x, bc.y);
        } else if (i == 0) {
          v = r;
        } else if (sc.s[i] == 0.f) {
          v = make_float4(0.f, 0.f, 0.f, 0.f);
        } else {
          const float s = sc.s[i];
          v = make_float4(bf16_round(s * r.x), bf16_round(s * r.y), bf16_round(s * r.z),
                          bf16_round(s * r.w));
        }
        o[i * Cq] = v;
      }
    } else {
      const float r = __bfloat162float(res[e]);
      float* o = out + t * n * C + q;
      for (int i = 0; i < n; ++i)
        o[i * C] = i == 1 ? __bfloat162float(br[e])
                          : (i == 0 ? r : (sc.s[i] == 0.f ? 0.f : bf16_round(sc.s[i] * r)));
    }
  }
}

template <bool VEC>
__global__ void __launch_bounds__(256)
    pack_bwd_kernel(const float* __restrict__ g, float* __restrict__ gres,
                    float* __restrict__ gbr, int64_t T, int n, int64_t C, Scales sc) {
  const int64_t Cq = VEC ? C / 4 : C;
  const int64_t total = T * Cq;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = e / Cq, q = e - t * Cq;
    if (VEC) {
      const float4* gi = reinterpret_cast<const float4*>(g) + t * n * Cq + q;
      float4 acc = __ldg(gi);
      for (int i = 2; i < n; ++i) {
        if (sc.s[i] == 0.f) continue;
        const float4 v = __ldg(gi + i * Cq);
        acc.x += sc.s[i] * v.x; acc.y += sc.s[i] * v.y;
        acc.z += sc.s[i] * v.z; acc.w += sc.s[i] * v.w;
      }
      reinterpret_cast<float4*>(gres)[e] = acc;
      if (n >= 2 && gbr) reinterpret_cast<float4*>(gbr)[e] = __ldg(gi + Cq);
    } else {
      const float* gi = g + t * n * C + q;
      float acc = gi[0];
      for (int i = 2; i < n; ++i)
        if (sc.s[i] != 0.f) acc += sc.s[i] * gi[i * C];
      gres[e] = acc;
      if (n >= 2 && gbr) gbr[e] = gi[C];
    }
  }
}

template <bool VEC>
__global__ void __launch_bounds__(256)
    mean_fwd_kernel(const float* __restrict__ x, float* __restrict__ out, int64_t T, int n,
                    int64_t C) {
  const int64_t Cq = VEC ? C / 4 : C;
  const int64_t total = T * Cq;
  const float nf = (float)n;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = e / Cq, q = e - t * Cq;
    if (VEC) {
      const float4* xi = reinterpret_cast<const float4*>(x) + t * n * Cq + q;
      float4 acc = __ldg(xi);
      for (int i = 1; i < n; ++i) {
        const float4 v = __ldg(xi + i * Cq);
        acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
      }
      reinterpret_cast<float4*>(out)[e] = make_float4(acc.x / nf, acc.y / nf, acc.z / nf, acc.w / nf);
    } else {
      const float* xi = x + t * n * C + q;
      float acc = xi[0];
      for (int i = 1; i < n; ++i) acc += xi[i * C];
      out[e] = acc / nf;
    }
  }
}

template <bool VEC>
__global__ void __launch_bounds__(256)
    mean_bwd_kernel(const float* __restrict__ g, float* __restrict__ gx, int64_t T, int n,
                    int64_t C) {
  const int64_t Cq = VEC ? C / 4 : C;
  const int64_t total = T * Cq;
  const float nf = (float)n;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = e / Cq, q = e - t * Cq;
    if (VEC) {
      const float4 gv = __ldg(reinterpret_cast<const float4*>(g) + e);
      const float4 v = make_float4(gv.x / nf, gv.y / nf, gv.z / nf, gv.w / nf);
      float4* o = reinterpret_cast<float4*>(gx) + t * n * Cq + q;
      for (int i = 0; i < n; ++i) o[i * Cq] = v;
    } else {
      const float v = g[e] / nf;
      float* o = gx + t * n * C + q;
      for (int i = 0; i < n; ++i) o[i * C] = v;
    }
  }
}

int check_shape(const char* what, int64_t T, int n, int64_t C) {
  MHC_REQUIRE(T >= 0 && C >= 0, MHC_ERR_INVALID_ARG, "%s: negative shape", what);
  MHC_REQUIRE(n >= 1 && n <= kMaxStreams, MHC_ERR_UNSUPPORTED, "%s: n must be in [1, %d], got %d",
              what, kMaxStreams, n);
  return MHC_OK;
}

bool vec_ok(int64_t C, std::initializer_list<const void*> ptrs) {
  if (C % 4) return false;
  for (const void* p : ptrs)
    if (p && !aligned16(p)) return false;
  return true;
}

Scales host_scales(const float* scales, int n) {
  Scales sc{};
  for (int i = 0; i < n; ++i) sc.s[i] = scales[i];
  sc.s[0] = 1.0f;
  return sc;
}

}  // namespace
}  // namespace mhc

using namespace mhc;

extern "C" int mhc_wrapper_pack_fwd(const float* residual, const float* branch, float* out,
                                    const float* scales, int64_t tokens, int32_t n,
                                    int64_t hidden, void* stream) {
  int rc = check_shape("mhc_wrapper_pack_fwd", tokens, n, hidden);
  if (rc) return rc;
  MHC_REQUIRE_PTR(residual); MHC_REQUIRE_PTR(out); MHC_REQUIRE_PTR(scales);
  MHC_REQUIRE(n < 2 || branch != nullptr, MHC_ERR_INVALID_ARG,
              "mhc_wrapper_pack_fwd: branch must not be NULL for n >= 2");
  if (tokens == 0 || hidden == 0) return MHC_OK;
  const Scales sc = host_scales(scales, n);
  cudaStream_t s = (cudaStream_t)stream;
  ProfScope _ps("wrapper_pack", s);
  if (vec_ok(hidden, {residual, branch, out}))
    pack_fwd_kernel<true><<<grid_for(tokens * hidden / 4), 256, 0, s>>>(
        residual, branch, out, tokens, n, hidden, sc);
  else
    pack_fwd_kernel<false><<<grid_for(tokens * hidden), 256, 0, s>>>(
        residual, branch, out, tokens, n, hidden, sc);
  return check_launch("mhc_wrapper_pack_fwd");
}

extern "C" int mhc_wrapper_pack_fwd_bf16(const void* residual, const void* branch, float* out,
                                         const float* scales, int64_t tokens, int32_t n,
                                         int64_t hidden, void* stream) {
  int rc = check_shape("mhc_wrapper_pack_fwd_bf16", tokens, n, hidden);
  if (rc) return rc;
  MHC_REQUIRE_PTR(residual); MHC_REQUIRE_PTR(out); MHC_REQUIRE_PTR(scales);
  MHC_REQUIRE(n < 2 || branch != nullptr, MHC_ERR_INVALID_ARG,
              "mhc_wrapper_pack_fwd_bf16: branch must not be NULL for n >= 2");
  if (tokens == 0 || hidden == 0) return MHC_OK;
  const Scales sc = host_scales(scales, n);
  cudaStream_t s = (cudaStream_t)stream;
  const __nv_bfloat16* r = (const __nv_bfloat16*)residual;
  const __nv_bfloat16* b = (const __nv_bfloat16*)branch;
  const bool vec = hidden % 4 == 0 && ((uintptr_t)residual & 7) == 0 &&
                   (branch == nullptr || ((uintptr_t)branch & 7) == 0) && aligned16(out);
  ProfScope _ps("wrapper_pack_bf16", s);
  if (vec)
    pack_fwd_bf16_kernel<true><<<grid_for(tokens * hidden / 4), 256, 0, s>>>(r, b, out, tokens, n,
                                                                           hidden, sc);
  else
    pack_fwd_bf16_kernel<false><<<grid_for(tokens * hidden), 256, 0, s>>>(r, b, out, tokens, n,
                                                                        hidden, sc);
  return check_launch("mhc_wrapper_pack_fwd_bf16");
}

extern "C" int mhc_wrapper_pack_bwd(const float* grad_out, float* grad_residual,
                                    float* grad_branch, const float* scales, int64_t tokens,
                                    int32_t n, int64_t hidden, void* stream) {
  int rc = check_shape("mhc_wrapper_pack_bwd", tokens, n, hidden);
  if (rc) return rc;
  MHC_REQUIRE_PTR(grad_out); MHC_REQUIRE_PTR(grad_residual); MHC_REQUIRE_PTR(scales);
  if (tokens == 0 || hidden == 0) return MHC_OK;
  const Scales sc = host_scales(scales, n);
  cudaStream_t s = (cudaStream_t)stream;
  ProfScope _ps("wrapper_pack_bwd", s);
  if (vec_ok(hidden, {grad_out, grad_residual, grad_branch}))
    pack_bwd_kernel<true><<<grid_for(tokens * hidden / 4), 256, 0, s>>>(
        grad_out, grad_residual, grad_branch, tokens, n, hidden, sc);
  else
    pack_bwd_kernel<false><<<grid_for(tokens * hidden), 256, 0, s>>>(
        grad_out, grad_residual, grad_branch, tokens, n, hidden, sc);
  return check_launch("mhc_wrapper_pack_bwd");
}

extern "C" int mhc_stream_mean_fwd(const float* inp, float* out, int64_t tokens, int32_t n,
                                   int64_t hidden, void* stream) {
  int rc = check_shape("mhc_stream_mean_fwd", tokens, n, hidden);
  if (rc) return rc;
  MHC_REQUIRE_PTR(inp); MHC_REQUIRE_PTR(out);
  if (tokens == 0 || hidden == 0) return MHC_OK;
  cudaStream_t s = (cudaStream_t)stream;
  ProfScope _ps("stream_mean", s);
  if (vec_ok(hidden, {inp, out}))
    mean_fwd_kernel<true><<<grid_for(tokens * hidden / 4), 256, 0, s>>>(
        inp, out, tokens, n, hidden);
  else
    mean_fwd_kernel<false><<<grid_for(tokens * hidden), 256, 0, s>>>(
        inp, out, tokens, n, hidden);
  return check_launch("mhc_stream_mean_fwd");
}

extern "C" int mhc_stream_mean_bwd(const float* grad_out, float* grad_inp, int64_t tokens,
                                   int32_t n, int64_t hidden, void* stream) {
  int rc = check_shape("mhc_stream_mean_bwd", tokens, n, hidden);
  if (rc) return rc;
  MHC_REQUIRE_PTR(grad_out); MHC_REQUIRE_PTR(grad_inp);
  if (tokens == 0 || hidden == 0) return MHC_OK;
  cudaStream_t s = (cudaStream_t)stream;
  ProfScope _ps("stream_mean_bwd", s);
  if (vec_ok(hidden, {grad_out, grad_inp}))
    mean_bwd_kernel<true><<<grid_for(tokens * hidden / 4), 256, 0, s>>>(
        grad_out, grad_inp, tokens, n, hidden);
  else
    mean_bwd_kernel<false><<<grid_for(tokens * hidden), 256, 0, s>>>(
        grad_out, grad_inp, tokens, n, hidden);
  return check_launch("mhc_stream_mean_bwd");
}
