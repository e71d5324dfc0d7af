// Standalone mHC operators: stream aggregate, stream distribute-mix-add,
// RMSNorm, row RMS and the dynamic-H projection (forward and backward).
//
// These back the per-operator Python API (ops.py: StreamAggregateFunction,
// StreamDistributeMixAddFunction, RMSNormFunction, FusedProjectionFunction,
// compute_rms) and replace the Ascend kernels of stream_ops.cpp,
// rmsnorm.cpp, compute_rms.cpp and fused_ops.cpp.  The fused layer path does
// not use them (layer_dynamic.cu / layer_static.cu fuse the whole layer).
//
// All reductions over the batch (grad_weight of RMSNorm, grad_weight of the
// projection) are two-level fixed-order reductions through a workspace:
// deterministic, no atomics (the reference uses AtomicAdd, rmsnorm.cpp:337).
#include "common.cuh"

namespace mhc {
namespace {

constexpr int kThreads = 256;

// ---------------------------------------------------------------------------
// stream_aggregate (stream_ops.cpp:26-269 fwd, :574-830 bwd)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads)
    aggregate_fwd_kernel(const float* __restrict__ x, const float* __restrict__ h_raw,
                         float* __restrict__ out, float* __restrict__ h_act, int n, int64_t C,
                         int64_t B) {
  extern __shared__ float sh[];  // n activations
  for (int64_t b = blockIdx.y; b < B; b += gridDim.y) {
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float a = sigmoidf_(h_raw[b * n + i]);
    sh[i] = a;
    if (blockIdx.x == 0) h_act[b * n + i] = a;
  }
  __syncthreads();
  for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < C;
       c += (int64_t)gridDim.x * blockDim.x) {
    float s = 0.f;
    for (int i = 0; i < n; ++i) s += sh[i] * x[(b * n + i) * C + c];
    out[b * C + c] = s;
  }
  }
}

__global__ void __launch_bounds__(kThreads)
    aggregate_bwd_kernel(const float* __restrict__ g, const float* __restrict__ x,
                         const float* __restrict__ h_act, float* __restrict__ gx,
                         float* __restrict__ gh, int n, int64_t C) {
  const int64_t b = blockIdx.x;
  __shared__ float red[32];
  for (int i = 0; i < n; ++i) {
    const float hi = h_act[b * n + i];
    float acc = 0.f;
    for (int64_t c = threadIdx.x; c < C; c += blockDim.x) {
      const float gv = g[b * C + c];
      gx[(b * n + i) * C + c] = hi * gv;
      acc += gv * x[(b * n + i) * C + c];
    }
    acc = warp_sum(acc);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
      float s = 0.f;
      for (int w = 0; w < (int)(blockDim.x >> 5); ++w) s += red[w];
      gh[b * n + i] = s;
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// stream_distribute_mix_add (stream_ops.cpp:275-568 fwd, :836-1127 bwd)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads)
    distribute_fwd_kernel(const float* __restrict__ y, const float* __restrict__ hp_raw,
                          const float* __restrict__ M, const float* __restrict__ x,
                          float* __restrict__ out, float* __restrict__ hp_act, int n,
                          int64_t C, int64_t B) {
  extern __shared__ float sh[];  // n post activations, then n*n M
  float* s_hp = sh;
  float* s_M = sh + n;
  for (int64_t b = blockIdx.y; b < B; b += gridDim.y) {
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float a = 2.f * sigmoidf_(hp_raw[b * n + i]);
    s_hp[i] = a;
    if (blockIdx.x == 0) hp_act[b * n + i] = a;
  }
  for (int e = threadIdx.x; e < n * n; e += blockDim.x) s_M[e] = M[b * n * n + e];
  __syncthreads();
  for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < C;
       c += (int64_t)gridDim.x * blockDim.x) {
    const float yv = y[b * C + c];
    for (int i = 0; i < n; ++i) {
      float s = s_hp[i] * yv;
      for (int j = 0; j < n; ++j) s += s_M[i * n + j] * x[(b * n + j) * C + c];
      out[(b * n + i) * C + c] = s;
    }
  }
  }
}

// Per token: grad_x[j,c] = sum_i M[i,j] g[i,c]; grad_y[c] = sum_i hp_i g[i,c];
// grad_M[i,j] = sum_c g[i,c] x[j,c]; grad_hp[i] = sum_c g[i,c] y[c].
__global__ void __launch_bounds__(kThreads)
    distribute_bwd_kernel(const float* __restrict__ g, const float* __restrict__ x,
                          const float* __restrict__ y, const float* __restrict__ M,
                          const float* __restrict__ hp_act, float* __restrict__ gx,
                          float* __restrict__ gy, float* __restrict__ gM,
                          float* __restrict__ ghp, int n, int64_t C) {
  const int64_t b = blockIdx.x;
  extern __shared__ float sh[];  // n*n M, n hp, (n*n + n) * nwarps partials
  float* s_M = sh;
  float* s_hp = sh + n * n;
  float* s_red = s_hp + n;
  const int nwarps = blockDim.x >> 5, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int e = threadIdx.x; e < n * n; e += blockDim.x) s_M[e] = M[b * n * n + e];
  for (int i = threadIdx.x; i < n; i += blockDim.x) s_hp[i] = hp_act[b * n + i];
  __syncthreads();
  // elementwise part
  for (int64_t c = threadIdx.x; c < C; c += blockDim.x) {
    float gys = 0.f;
    for (int i = 0; i < n; ++i) gys += s_hp[i] * g[(b * n + i) * C + c];
    gy[b * C + c] = gys;
    for (int j = 0; j < n; ++j) {
      float s = 0.f;
      for (int i = 0; i < n; ++i) s += s_M[i * n + j] * g[(b * n + i) * C + c];
      gx[(b * n + j) * C + c] = s;
    }
  }
  // reductions: pair p < n*n -> grad_M, p in [n*n, n*n+n) -> grad_hp
  const int npairs = n * n + n;
  for (int p = 0; p < npairs; ++p) {
    const int i = p < n * n ? p / n : p - n * n;
    const float* rhs = p < n * n ? x + (b * n + (p % n)) * C : y + b * C;
    const float* lhs = g + (b * n + i) * C;
    float acc = 0.f;
    for (int64_t c = threadIdx.x; c < C; c += blockDim.x) acc += lhs[c] * rhs[c];
    acc = warp_sum(acc);
    if (lane == 0) s_red[p * nwarps + warp] = acc;
  }
  __syncthreads();
  for (int p = threadIdx.x; p < npairs; p += blockDim.x) {
    float s = 0.f;
    for (int w = 0; w < nwarps; ++w) s += s_red[p * nwarps + w];
    if (p < n * n) gM[b * n * n + p] = s;
    else ghp[b * n + (p - n * n)] = s;
  }
}

// ---------------------------------------------------------------------------
// RMSNorm (rmsnorm.cpp:135-189 fwd, :352-425 bwd) and row RMS
// (compute_rms.cpp:69-118)
// ---------------------------------------------------------------------------
__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float s = 0.f;
  for (int w = 0; w < nw; ++w) s += red[w];
  return s;
}

__global__ void __launch_bounds__(kThreads)
    rms_kernel(const float* __restrict__ x, float* __restrict__ rms, int64_t K, float eps) {
  __shared__ float red[32];
  const int64_t b = blockIdx.x;
  float acc = 0.f;
  for (int64_t k = threadIdx.x; k < K; k += blockDim.x) {
    const float v = x[b * K + k];
    acc += v * v;
  }
  const float s = block_sum(acc, red);
  if (threadIdx.x == 0) rms[b] = sqrtf(s / (float)K + eps);
}

__global__ void __launch_bounds__(kThreads)
    rmsnorm_fwd_kernel(const float* __restrict__ x, const float* __restrict__ w,
                       float* __restrict__ out, float* __restrict__ rms, int64_t C, float eps) {
  __shared__ float red[32];
  const int64_t b = blockIdx.x;
  float acc = 0.f;
  for (int64_t c = threadIdx.x; c < C; c += blockDim.x) {
    const float v = x[b * C + c];
    acc += v * v;
  }
  const float s = block_sum(acc, red);
  const float r = sqrtf(s / (float)C + eps);
  if (threadIdx.x == 0) rms[b] = r;
  for (int64_t c = threadIdx.x; c < C; c += blockDim.x) out[b * C + c] = (x[b * C + c] / r) * w[c];
}

// grad_x = g*w/r - x * sum(g*w*x) / (C r^3)
__global__ void __launch_bounds__(kThreads)
    rmsnorm_bwd_x_kernel(const float* __restrict__ g, const float* __restrict__ x,
                         const float* __restrict__ w, const float* __restrict__ rms,
                         float* __restrict__ gx, int64_t C) {
  __shared__ float red[32];
  const int64_t b = blockIdx.x;
  const float r = rms[b];
  float acc = 0.f;
  for (int64_t c = threadIdx.x; c < C; c += blockDim.x) acc += g[b * C + c] * w[c] * x[b * C + c];
  const float dot = block_sum(acc, red);
  const float inv_r = 1.f / r;
  const float beta = dot / ((float)C * r * r * r);
  for (int64_t c = threadIdx.x; c < C; c += blockDim.x)
    gx[b * C + c] = g[b * C + c] * w[c] * inv_r - x[b * C + c] * beta;
}

// partial[chunk, c] = sum over rows of the chunk of g*x/r
__global__ void __launch_bounds__(kThreads)
    rmsnorm_bwd_w_partial_kernel(const float* __restrict__ g, const float* __restrict__ x,
                                 const float* __restrict__ rms, float* __restrict__ part,
                                 int64_t B, int64_t C, int64_t rows_per_chunk) {
  const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t chunk = blockIdx.y;
  if (c >= C) return;
  const int64_t b0 = chunk * rows_per_chunk;
  const int64_t b1 = b0 + rows_per_chunk < B ? b0 + rows_per_chunk : B;
  float acc = 0.f;
  for (int64_t b = b0; b < b1; ++b) acc += g[b * C + c] * x[b * C + c] / rms[b];
  part[chunk * C + c] = acc;
}

// out[c] = sum_chunk part[chunk, c]   (fixed order)
__global__ void __launch_bounds__(kThreads)
    sum_chunks_kernel(const float* __restrict__ part, float* __restrict__ out, int64_t nchunks,
                      int64_t L) {
  const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= L) return;
  float s = 0.f;
  for (int64_t k = 0; k < nchunks; ++k) s += part[k * L + c];
  out[c] = s;
}

// ---------------------------------------------------------------------------
// Projection out[b,o] = sum_k x[b,k] w[o,k]   (fused_ops.cpp:136-202 role)
// Tile: 16 rows x out_dim, K staged through shared memory.
// ---------------------------------------------------------------------------
constexpr int PJ_ROWS = 16;
constexpr int PJ_KT = 64;

__global__ void __launch_bounds__(512)
    proj_fwd_kernel(const float* __restrict__ x, const float* __restrict__ w,
                    float* __restrict__ out, int64_t B, int64_t K, int O) {
  extern __shared__ float sh[];
  float* sx = sh;                         // [PJ_ROWS][PJ_KT]
  float* sw = sh + PJ_ROWS * PJ_KT;       // [O][PJ_KT + 1]
  const int64_t b0 = (int64_t)blockIdx.x * PJ_ROWS;
  const int tid = threadIdx.x;
  const int r = tid / O, o = tid % O;
  const bool active = r < PJ_ROWS;
  float acc = 0.f;
  for (int64_t k0 = 0; k0 < K; k0 += PJ_KT) {
    for (int e = tid; e < PJ_ROWS * PJ_KT; e += blockDim.x) {
      const int rr = e / PJ_KT, kk = e % PJ_KT;
      const int64_t b = b0 + rr, k = k0 + kk;
      sx[e] = (b < B && k < K) ? x[b * K + k] : 0.f;
    }
    for (int e = tid; e < O * PJ_KT; e += blockDim.x) {
      const int oo = e / PJ_KT, kk = e % PJ_KT;
      const int64_t k = k0 + kk;
      sw[oo * (PJ_KT + 1) + kk] = k < K ? w[(int64_t)oo * K + k] : 0.f;
    }
    __syncthreads();
    if (active) {
#pragma unroll 8
      for (int kk = 0; kk < PJ_KT; ++kk) acc += sx[r * PJ_KT + kk] * sw[o * (PJ_KT + 1) + kk];
    }
    __syncthreads();
  }
  if (active && b0 + r < B) out[(b0 + r) * O + o] = acc;
}

// grad_x[b,k] = sum_o g[b,o] w[o,k]
__global__ void __launch_bounds__(kThreads)
    proj_bwd_x_kernel(const float* __restrict__ g, const float* __restrict__ w,
                      float* __restrict__ gx, int64_t K, int O, int64_t B) {
  extern __shared__ float sg[];
  for (int64_t b = blockIdx.y; b < B; b += gridDim.y) {
  __syncthreads();
  for (int o = threadIdx.x; o < O; o += blockDim.x) sg[o] = g[b * O + o];
  __syncthreads();
  for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < K;
       k += (int64_t)gridDim.x * blockDim.x) {
    float s = 0.f;
    for (int o = 0; o < O; ++o) s += sg[o] * w[(int64_t)o * K + k];
    gx[b * K + k] = s;
  }
  }
}

// partial[chunk, o, k] = sum_{b in chunk} g[b,o] x[b,k]
__global__ void __launch_bounds__(kThreads)
    proj_bwd_w_partial_kernel(const float* __restrict__ g, const float* __restrict__ x,
                              float* __restrict__ part, int64_t B, int64_t K, int O,
                              int64_t rows_per_chunk) {
  const int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t chunk = blockIdx.y;
  const int o = blockIdx.z;
  if (k >= K) return;
  const int64_t b0 = chunk * rows_per_chunk;
  const int64_t b1 = b0 + rows_per_chunk < B ? b0 + rows_per_chunk : B;
  float acc = 0.f;
  for (int64_t b = b0; b < b1; ++b) acc += g[b * O + o] * x[b * K + k];
  part[(chunk * O + o) * K + k] = acc;
}

int64_t chunks_for(int64_t B) { return B < 64 ? 1 : (B + 63) / 64 < 64 ? (B + 63) / 64 : 64; }

unsigned grid_x(int64_t C) {
  int64_t g = (C + kThreads - 1) / kThreads;
  return (unsigned)(g < 1 ? 1 : g);
}

int check_common(const char* what, int64_t B, int n, int64_t C) {
  MHC_REQUIRE(B >= 0 && C >= 0, MHC_ERR_INVALID_ARG, "%s: negative shape", what);
  MHC_REQUIRE(n >= 1, MHC_ERR_INVALID_ARG, "%s: n must be >= 1, got %d", what, n);
  MHC_REQUIRE(B < 65536LL * 32768LL, MHC_ERR_UNSUPPORTED, "%s: batch too large", what);
  return MHC_OK;
}

}  // namespace
}  // namespace mhc

using namespace mhc;

extern "C" int mhc_stream_aggregate_fwd(const float* inp, const float* H_pre_raw, float* out,
                                        float* H_pre_act, int64_t batch, int32_t n,
                                        int64_t hidden, void* stream) {
  int rc = check_common("stream_aggregate_fwd", batch, n, hidden);
  if (rc) return rc;
  MHC_REQUIRE_PTR(inp); MHC_REQUIRE_PTR(H_pre_raw); MHC_REQUIRE_PTR(out); MHC_REQUIRE_PTR(H_pre_act);
  if (batch == 0) return MHC_OK;
  dim3 grid(grid_x(hidden) < 8 ? grid_x(hidden) : 8, (unsigned)(batch < 65535 ? batch : 65535));
  aggregate_fwd_kernel<<<grid, kThreads, n * sizeof(float), (cudaStream_t)stream>>>(
      inp, H_pre_raw, out, H_pre_act, n, hidden, batch);
  return check_launch("stream_aggregate_fwd");
}

extern "C" int mhc_stream_aggregate_bwd(const float* grad_out, const float* inp,
                                        const float* H_pre_act, float* grad_inp,
                                        float* grad_H_pre_act, int64_t batch, int32_t n,
                                        int64_t hidden, void* stream) {
  int rc = check_common("stream_aggregate_bwd", batch, n, hidden);
  if (rc) return rc;
  MHC_REQUIRE_PTR(grad_out); MHC_REQUIRE_PTR(inp); MHC_REQUIRE_PTR(H_pre_act);
  MHC_REQUIRE_PTR(grad_inp); MHC_REQUIRE_PTR(grad_H_pre_act);
  if (batch == 0) return MHC_OK;
  aggregate_bwd_kernel<<<(unsigned)batch, kThreads, 0, (cudaStream_t)stream>>>(
      grad_out, inp, H_pre_act, grad_inp, grad_H_pre_act, n, hidden);
  return check_launch("stream_aggregate_bwd");
}

extern "C" int mhc_stream_distribute_mix_add_fwd(const float* y_norm, const float* H_post_raw,
                                                 const float* M, const float* x_inp, float* out,
                                                 float* H_post_act, int64_t batch, int32_t n,
                                                 int64_t hidden, void* stream) {
  int rc = check_common("stream_distribute_mix_add_fwd", batch, n, hidden);
  if (rc) return rc;
  MHC_REQUIRE_PTR(y_norm); MHC_REQUIRE_PTR(H_post_raw); MHC_REQUIRE_PTR(M);
  MHC_REQUIRE_PTR(x_inp); MHC_REQUIRE_PTR(out); MHC_REQUIRE_PTR(H_post_act);
  MHC_REQUIRE(n <= 64, MHC_ERR_UNSUPPORTED, "stream_distribute_mix_add_fwd: n > 64");
  if (batch == 0) return MHC_OK;
  dim3 grid(grid_x(hidden) < 8 ? grid_x(hidden) : 8, (unsigned)(batch < 65535 ? batch : 65535));
  distribute_fwd_kernel<<<grid, kThreads, (n + n * n) * sizeof(float), (cudaStream_t)stream>>>(
      y_norm, H_post_raw, M, x_inp, out, H_post_act, n, hidden, batch);
  return check_launch("stream_distribute_mix_add_fwd");
}

extern "C" int mhc_stream_distribute_mix_add_bwd(const float* grad_out, const float* x_inp,
                                                 const float* y_norm, const float* M,
                                                 const float* H_post_act, float* grad_x,
                                                 float* grad_y_norm, float* grad_M,
                                                 float* grad_H_post_act, int64_t batch,
                                                 int32_t n, int64_t hidden, void* stream) {
  int rc = check_common("stream_distribute_mix_add_bwd", batch, n, hidden);
  if (rc) return rc;
  MHC_REQUIRE_PTR(grad_out); MHC_REQUIRE_PTR(x_inp); MHC_REQUIRE_PTR(y_norm);
  MHC_REQUIRE_PTR(M); MHC_REQUIRE_PTR(H_post_act); MHC_REQUIRE_PTR(grad_x);
  MHC_REQUIRE_PTR(grad_y_norm); MHC_REQUIRE_PTR(grad_M); MHC_REQUIRE_PTR(grad_H_post_act);
  MHC_REQUIRE(n <= 32, MHC_ERR_UNSUPPORTED, "stream_distribute_mix_add_bwd: n > 32");
  if (batch == 0) return MHC_OK;
  const int nwarps = kThreads / 32;
  const size_t smem = (size_t)(n * n + n + (n * n + n) * nwarps) * sizeof(float);
  distribute_bwd_kernel<<<(unsigned)batch, kThreads, smem, (cudaStream_t)stream>>>(
      grad_out, x_inp, y_norm, M, H_post_act, grad_x, grad_y_norm, grad_M, grad_H_post_act, n,
      hidden);
  return check_launch("stream_distribute_mix_add_bwd");
}

extern "C" int mhc_compute_rms_fwd(const float* inp, float* rms, int64_t batch, int64_t k,
                                   float eps, void* stream) {
  int rc = check_common("compute_rms_fwd", batch, 1, k);
  if (rc) return rc;
  MHC_REQUIRE_PTR(inp); MHC_REQUIRE_PTR(rms);
  MHC_REQUIRE(k >= 1, MHC_ERR_INVALID_ARG, "compute_rms_fwd: row length must be >= 1");
  if (batch == 0) return MHC_OK;
  rms_kernel<<<(unsigned)batch, kThreads, 0, (cudaStream_t)stream>>>(inp, rms, k, eps);
  return check_launch("compute_rms_fwd");
}

extern "C" int mhc_rmsnorm_fwd(const float* inp, const float* weight, float* out, float* rms,
                               int64_t batch, int64_t hidden, float eps, void* stream) {
  int rc = check_common("rmsnorm_fwd", batch, 1, hidden);
  if (rc) return rc;
  MHC_REQUIRE_PTR(inp); MHC_REQUIRE_PTR(weight); MHC_REQUIRE_PTR(out); MHC_REQUIRE_PTR(rms);
  MHC_REQUIRE(hidden >= 1, MHC_ERR_INVALID_ARG, "rmsnorm_fwd: hidden must be >= 1");
  if (batch == 0) return MHC_OK;
  rmsnorm_fwd_kernel<<<(unsigned)batch, kThreads, 0, (cudaStream_t)stream>>>(inp, weight, out, rms,
                                                                             hidden, eps);
  return check_launch("rmsnorm_fwd");
}

extern "C" size_t mhc_rmsnorm_bwd_workspace_bytes(int64_t batch, int64_t hidden) {
  if (batch <= 0 || hidden <= 0) return 0;
  return (size_t)chunks_for(batch) * (size_t)hidden * sizeof(float);
}

extern "C" int mhc_rmsnorm_bwd(const float* grad_out, const float* inp, const float* weight,
                               const float* rms, float* grad_inp, float* grad_weight,
                               int64_t batch, int64_t hidden, void* workspace,
                               size_t workspace_bytes, void* stream) {
  int rc = check_common("rmsnorm_bwd", batch, 1, hidden);
  if (rc) return rc;
  MHC_REQUIRE_PTR(grad_out); MHC_REQUIRE_PTR(inp); MHC_REQUIRE_PTR(weight);
  MHC_REQUIRE_PTR(rms); MHC_REQUIRE_PTR(grad_inp); MHC_REQUIRE_PTR(grad_weight);
  cudaStream_t s = (cudaStream_t)stream;
  if (batch == 0) {
    if (hidden > 0) cudaMemsetAsync(grad_weight, 0, hidden * sizeof(float), s);
    return check_launch("rmsnorm_bwd");
  }
  const size_t need = mhc_rmsnorm_bwd_workspace_bytes(batch, hidden);
  MHC_REQUIRE(workspace != nullptr && workspace_bytes >= need, MHC_ERR_WORKSPACE,
              "rmsnorm_bwd: workspace of %zu bytes required, got %zu", need, workspace_bytes);
  rmsnorm_bwd_x_kernel<<<(unsigned)batch, kThreads, 0, s>>>(grad_out, inp, weight, rms, grad_inp,
                                                           hidden);
  rc = check_launch("rmsnorm_bwd");
  if (rc) return rc;
  const int64_t nch = chunks_for(batch);
  const int64_t rows = (batch + nch - 1) / nch;
  float* part = (float*)workspace;
  rmsnorm_bwd_w_partial_kernel<<<dim3(grid_x(hidden), (unsigned)nch), kThreads, 0, s>>>(
      grad_out, inp, rms, part, batch, hidden, rows);
  sum_chunks_kernel<<<grid_x(hidden), kThreads, 0, s>>>(part, grad_weight, nch, hidden);
  return check_launch("rmsnorm_bwd");
}

extern "C" int mhc_fused_rmsnorm_matmul_fwd(const float* inp, const float* weight, float* out,
                                            int64_t batch, int64_t k, int32_t out_dim,
                                            void* stream) {
  int rc = check_common("fused_rmsnorm_matmul_fwd", batch, 1, k);
  if (rc) return rc;
  MHC_REQUIRE_PTR(inp); MHC_REQUIRE_PTR(weight); MHC_REQUIRE_PTR(out);
  MHC_REQUIRE(out_dim >= 1 && out_dim <= 32, MHC_ERR_UNSUPPORTED,
              "fused_rmsnorm_matmul_fwd: out_dim must be in [1, 32], got %d", out_dim);
  if (batch == 0) return MHC_OK;
  const int threads = ((PJ_ROWS * out_dim + 31) / 32) * 32;
  const size_t smem = (PJ_ROWS * PJ_KT + out_dim * (PJ_KT + 1)) * sizeof(float);
  proj_fwd_kernel<<<(unsigned)((batch + PJ_ROWS - 1) / PJ_ROWS), threads, smem,
                    (cudaStream_t)stream>>>(inp, weight, out, batch, k, out_dim);
  return check_launch("fused_rmsnorm_matmul_fwd");
}

extern "C" size_t mhc_fused_rmsnorm_matmul_bwd_workspace_bytes(int64_t batch, int64_t k,
                                                               int32_t out_dim) {
  if (batch <= 0 || k <= 0 || out_dim <= 0) return 0;
  return (size_t)chunks_for(batch) * (size_t)out_dim * (size_t)k * sizeof(float);
}

extern "C" int mhc_fused_rmsnorm_matmul_bwd(const float* grad_out, const float* inp,
                                            const float* weight, float* grad_inp,
                                            float* grad_weight, int64_t batch, int64_t k,
                                            int32_t out_dim, void* workspace,
                                            size_t workspace_bytes, void* stream) {
  int rc = check_common("fused_rmsnorm_matmul_bwd", batch, 1, k);
  if (rc) return rc;
  MHC_REQUIRE_PTR(grad_out); MHC_REQUIRE_PTR(inp); MHC_REQUIRE_PTR(weight);
  MHC_REQUIRE_PTR(grad_inp); MHC_REQUIRE_PTR(grad_weight);
  MHC_REQUIRE(out_dim >= 1 && out_dim <= 4096, MHC_ERR_UNSUPPORTED,
              "fused_rmsnorm_matmul_bwd: out_dim out of range");
  cudaStream_t s = (cudaStream_t)stream;
  if (batch == 0) {
    cudaMemsetAsync(grad_weight, 0, (size_t)out_dim * k * sizeof(float), s);
    return check_launch("fused_rmsnorm_matmul_bwd");
  }
  const size_t need = mhc_fused_rmsnorm_matmul_bwd_workspace_bytes(batch, k, out_dim);
  MHC_REQUIRE(workspace != nullptr && workspace_bytes >= need, MHC_ERR_WORKSPACE,
              "fused_rmsnorm_matmul_bwd: workspace of %zu bytes required, got %zu", need,
              workspace_bytes);
  dim3 gx_grid(grid_x(k) < 64 ? grid_x(k) : 64, (unsigned)(batch < 65535 ? batch : 65535));
  proj_bwd_x_kernel<<<gx_grid, kThreads, out_dim * sizeof(float), s>>>(grad_out, weight, grad_inp,
                                                                      k, out_dim, batch);
  rc = check_launch("fused_rmsnorm_matmul_bwd");
  if (rc) return rc;
  const int64_t nch = chunks_for(batch);
  const int64_t rows = (batch + nch - 1) / nch;
  float* part = (float*)workspace;
  proj_bwd_w_partial_kernel<<<dim3(grid_x(k), (unsigned)nch, (unsigned)out_dim), kThreads, 0, s>>>(
      grad_out, inp, part, batch, k, out_dim, rows);
  const int64_t L = (int64_t)out_dim * k;
  sum_chunks_kernel<<<(unsigned)((L + kThreads - 1) / kThreads), kThreads, 0, s>>>(part, grad_weight,
                                                                                 nch, L);
  return check_launch("fused_rmsnorm_matmul_bwd");
}
