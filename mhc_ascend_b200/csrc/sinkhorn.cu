// Standalone batched Sinkhorn-Knopp (forward and reverse mode).
//
// Replaces the Ascend kernels of sinkhorn_knopp.cpp (fwd :118-665, bwd
// :856-1814) behind sinkhorn_knopp_fwd / sinkhorn_knopp_bwd
// (bindings.cpp:155-231).  Layout: [batch, n, n] fp32 row-major.
//   n <= 8 : one matrix per thread, all n*n entries in registers.
//   n <= 32: one matrix per warp, lane j owns column j; row sums are warp
//            reductions; the per-iteration denominators for the reverse pass
//            live in shared memory.
#include "common.cuh"
#include "sinkhorn.cuh"

namespace mhc {
namespace {

template <int N>
__global__ void __launch_bounds__(128) sk_fwd_thread_kernel(const float* __restrict__ inp,
                                                            float* __restrict__ out,
                                                            int64_t batch, int iters, float eps) {
  const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= batch) return;
  float a[N * N];
  const float* src = inp + b * (N * N);
#pragma unroll
  for (int e = 0; e < N * N; ++e) a[e] = src[e];
  sk_forward<N, float>(a, iters, eps);
  float* dst = out + b * (N * N);
#pragma unroll
  for (int e = 0; e < N * N; ++e) dst[e] = a[e];
}

template <int N>
__global__ void __launch_bounds__(128) sk_bwd_thread_kernel(const float* __restrict__ grad_out,
                                                            const float* __restrict__ inp,
                                                            float* __restrict__ grad_inp,
                                                            int64_t batch, int iters, float eps) {
  const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= batch) return;
  float x0[N * N], g[N * N];
  const float* src = inp + b * (N * N);
  const float* gsrc = grad_out + b * (N * N);
#pragma unroll
  for (int e = 0; e < N * N; ++e) {
    x0[e] = src[e];
    g[e] = gsrc[e];
  }
  double xd[N * N], gd[N * N];
#pragma unroll
  for (int e = 0; e < N * N; ++e) { xd[e] = x0[e]; gd[e] = g[e]; }
  sk_backward<N, double>(xd, gd, iters, (double)eps);
#pragma unroll
  for (int e = 0; e < N * N; ++e) g[e] = (float)gd[e];
  float* dst = grad_inp + b * (N * N);
#pragma unroll
  for (int e = 0; e < N * N; ++e) dst[e] = g[e];
}

constexpr int WARPS_PER_BLOCK = 4;

// One matrix per warp, lane j holds column j (rows 0..n-1), n <= NM <= 32.
// Loops run over the compile-time NM with `i < n` guards, so the rows stay
// in registers.
//
// Row sums use a transpose-reduce: recursive halving over the lane bits
// (16 + 8 + 4 + 2 + 1 = 31 shuffles for 32 rows) leaves lane l holding the
// sum of row l over all lanes; that lane forms the row's denominator and
// reciprocal once and the warp reads them back with one shuffle per row.
// (A butterfly per row costs 5 shuffles per row and a division per element.)
// Rows beyond NM are zero-padded to 32.
template <int NM, typename T>
__device__ __forceinline__ T warp_row_sums_to_lanes(const T (&v)[NM], int lane) {
  T w[32];
#pragma unroll
  for (int k = 0; k < 32; ++k) w[k] = k < NM ? v[k] : T(0);
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    const bool up = (lane & o) != 0;
#pragma unroll
    for (int k = 0; k < o; ++k) {
      const T send = up ? w[k] : w[k + o];
      const T keep = up ? w[k + o] : w[k];
      w[k] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
  }
  return w[0];  // sum of row `lane`
}

template <int NM, typename T>
__device__ __forceinline__ void warp_sk_step(T (&a)[NM], int n, int lane, T eps, T* dr, T* dc) {
  const bool active = lane < n;
  {
    T v[NM];
#pragma unroll
    for (int i = 0; i < NM; ++i) v[i] = (i < n && active) ? a[i] : T(0);
    const T d_mine = warp_row_sums_to_lanes<NM, T>(v, lane) + eps;
    const T inv_mine = T(1) / d_mine;
    if (dr && lane < n) dr[lane] = d_mine;
#pragma unroll
    for (int i = 0; i < NM; ++i)
      if (i < n) {
        const T inv_i = __shfl_sync(0xffffffffu, inv_mine, i);  // every lane takes part
        a[i] = active ? a[i] * inv_i : T(0);
      }
  }
  T s = 0;
#pragma unroll
  for (int i = 0; i < NM; ++i)
    if (i < n) s += a[i];
  const T d = s + eps;
  if (dc && active) dc[lane] = d;
  if (active) {
    const T inv = T(1) / d;
#pragma unroll
    for (int i = 0; i < NM; ++i)
      if (i < n) a[i] = a[i] * inv;
  }
}

template <int NM>
__global__ void __launch_bounds__(WARPS_PER_BLOCK * 32)
    sk_fwd_warp_kernel(const float* __restrict__ inp, float* __restrict__ out, int64_t batch,
                       int n, int iters, float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t b = (int64_t)blockIdx.x * WARPS_PER_BLOCK + (threadIdx.x >> 5);
  if (b >= batch) return;
  float a[NM];
  const float* src = inp + b * n * n;
#pragma unroll
  for (int i = 0; i < NM; ++i) a[i] = (i < n && lane < n) ? src[i * n + lane] : 0.f;
  for (int t = 0; t < iters; ++t) warp_sk_step<NM, float>(a, n, lane, eps, nullptr, nullptr);
  float* dst = out + b * n * n;
  if (lane < n) {
#pragma unroll
    for (int i = 0; i < NM; ++i)
      if (i < n) dst[i * n + lane] = a[i];
  }
}

// Reverse mode runs in fp64 (the doubly-stochastic projection cancels the
// row/column-constant part of the incoming gradient).
constexpr int BWD_WARPS = 2;

template <int NM>
__global__ void __launch_bounds__(BWD_WARPS * 32)
    sk_bwd_warp_kernel(const float* __restrict__ grad_out, const float* __restrict__ inp,
                       float* __restrict__ grad_inp, int64_t batch, int n, int iters,
                       float eps_f) {
  __shared__ double s_dr[BWD_WARPS][SK_SEG][32];
  __shared__ double s_dc[BWD_WARPS][SK_SEG][32];
  const double eps = eps_f;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int64_t b = (int64_t)blockIdx.x * BWD_WARPS + w;
  if (b >= batch) return;
  const bool active = lane < n;
  double g[NM], z[NM];
  const float* src = inp + b * n * n;
  const float* gsrc = grad_out + b * n * n;
#pragma unroll
  for (int i = 0; i < NM; ++i) g[i] = (i < n && active) ? gsrc[i * n + lane] : 0.0;
  int seg_end = iters;
  while (seg_end > 0) {
    const int seg_start = seg_end > SK_SEG ? seg_end - SK_SEG : 0;
#pragma unroll
    for (int i = 0; i < NM; ++i) z[i] = (i < n && active) ? src[i * n + lane] : 0.0;
    for (int t = 0; t < seg_start; ++t) warp_sk_step<NM, double>(z, n, lane, eps, nullptr, nullptr);
    for (int t = seg_start; t < seg_end; ++t)
      warp_sk_step<NM, double>(z, n, lane, eps, s_dr[w][t - seg_start], s_dc[w][t - seg_start]);
    __syncwarp();
    for (int t = seg_end - 1; t >= seg_start; --t) {
      // column step
      const double dcj = active ? s_dc[w][t - seg_start][lane] : 1.0;
      double s = 0.0;
#pragma unroll
      for (int i = 0; i < NM; ++i)
        if (i < n) s += g[i] * z[i];
      const double inv = 1.0 / dcj;
#pragma unroll
      for (int i = 0; i < NM; ++i) {
        if (i < n) {
          g[i] = active ? (g[i] - s) * inv : 0.0;
          z[i] = z[i] * dcj;
        }
      }
      // row step: lane l reduces row l, then broadcasts its sum and 1/d
      {
        double v[NM];
#pragma unroll
        for (int i = 0; i < NM; ++i) v[i] = (i < n && active) ? g[i] * z[i] : 0.0;
        const double si_mine = warp_row_sums_to_lanes<NM, double>(v, lane);
        const double d_mine = lane < n ? s_dr[w][t - seg_start][lane] : 1.0;
        const double inv_mine = 1.0 / d_mine;
#pragma unroll
        for (int i = 0; i < NM; ++i) {
          if (i < n) {
            const double si = __shfl_sync(0xffffffffu, si_mine, i);
            const double d = __shfl_sync(0xffffffffu, d_mine, i);
            const double inv = __shfl_sync(0xffffffffu, inv_mine, i);
            g[i] = active ? (g[i] - si) * inv : 0.0;
            z[i] = z[i] * d;
          }
        }
      }
    }
    __syncwarp();
    seg_end = seg_start;
  }
  float* dst = grad_inp + b * n * n;
  if (active) {
#pragma unroll
    for (int i = 0; i < NM; ++i)
      if (i < n) dst[i * n + lane] = (float)g[i];
  }
}

template <int N>
int launch_thread_fwd(const float* inp, float* out, int64_t batch, int iters, float eps,
                      cudaStream_t s) {
  const int threads = 128;
  const int64_t blocks = (batch + threads - 1) / threads;
  sk_fwd_thread_kernel<N><<<(unsigned)blocks, threads, 0, s>>>(inp, out, batch, iters, eps);
  return check_launch("sinkhorn_knopp_fwd");
}

template <int N>
int launch_thread_bwd(const float* go, const float* inp, float* gi, int64_t batch, int iters,
                      float eps, cudaStream_t s) {
  const int threads = 128;
  const int64_t blocks = (batch + threads - 1) / threads;
  sk_bwd_thread_kernel<N><<<(unsigned)blocks, threads, 0, s>>>(go, inp, gi, batch, iters, eps);
  return check_launch("sinkhorn_knopp_bwd");
}

int validate(const void* a, const void* b, int64_t batch, int n, int iters, float eps) {
  MHC_REQUIRE(a != nullptr && b != nullptr, MHC_ERR_INVALID_ARG, "sinkhorn_knopp: NULL pointer");
  MHC_REQUIRE(batch >= 0, MHC_ERR_INVALID_ARG, "sinkhorn_knopp: batch must be >= 0, got %lld",
              (long long)batch);
  MHC_REQUIRE(n >= 1 && n <= 32, MHC_ERR_UNSUPPORTED,
              "sinkhorn_knopp: matrix size n must be in [1, 32], got %d", n);
  MHC_REQUIRE(iters >= 0, MHC_ERR_INVALID_ARG, "sinkhorn_knopp: num_iters must be >= 0, got %d",
              iters);
  MHC_REQUIRE(eps >= 0.f, MHC_ERR_INVALID_ARG, "sinkhorn_knopp: eps must be >= 0");
  MHC_REQUIRE(batch <= (int64_t)INT32_MAX * 32, MHC_ERR_UNSUPPORTED, "sinkhorn_knopp: batch too large");
  return MHC_OK;
}

}  // namespace
}  // namespace mhc

using namespace mhc;

extern "C" int mhc_sinkhorn_knopp_fwd(const float* inp, float* out, int64_t batch, int32_t n,
                                      int32_t num_iters, float eps, void* stream) {
  int rc = validate(inp, out, batch, n, num_iters, eps);
  if (rc) return rc;
  if (batch == 0) return MHC_OK;
  cudaStream_t s = (cudaStream_t)stream;
  switch (n) {
    case 1: return launch_thread_fwd<1>(inp, out, batch, num_iters, eps, s);
    case 2: return launch_thread_fwd<2>(inp, out, batch, num_iters, eps, s);
    case 3: return launch_thread_fwd<3>(inp, out, batch, num_iters, eps, s);
    case 4: return launch_thread_fwd<4>(inp, out, batch, num_iters, eps, s);
    case 5: return launch_thread_fwd<5>(inp, out, batch, num_iters, eps, s);
    case 6: return launch_thread_fwd<6>(inp, out, batch, num_iters, eps, s);
    case 7: return launch_thread_fwd<7>(inp, out, batch, num_iters, eps, s);
    case 8: return launch_thread_fwd<8>(inp, out, batch, num_iters, eps, s);
    default: {
      const int64_t blocks = (batch + WARPS_PER_BLOCK - 1) / WARPS_PER_BLOCK;
      ProfScope _ps("sinkhorn_fwd", s);
      if (n <= 16)
        sk_fwd_warp_kernel<16><<<(unsigned)blocks, WARPS_PER_BLOCK * 32, 0, s>>>(inp, out, batch, n, num_iters, eps);
      else
        sk_fwd_warp_kernel<32><<<(unsigned)blocks, WARPS_PER_BLOCK * 32, 0, s>>>(inp, out, batch, n, num_iters, eps);
      return check_launch("sinkhorn_knopp_fwd");
    }
  }
}

extern "C" int mhc_sinkhorn_knopp_bwd(const float* grad_out, const float* inp, const float* out,
                                      float* grad_inp, int64_t batch, int32_t n,
                                      int32_t num_iters, float eps, void* stream) {
  (void)out;
  int rc = validate(grad_out, grad_inp, batch, n, num_iters, eps);
  if (rc) return rc;
  MHC_REQUIRE_PTR(inp);
  if (batch == 0) return MHC_OK;
  cudaStream_t s = (cudaStream_t)stream;
  switch (n) {
    case 1: return launch_thread_bwd<1>(grad_out, inp, grad_inp, batch, num_iters, eps, s);
    case 2: return launch_thread_bwd<2>(grad_out, inp, grad_inp, batch, num_iters, eps, s);
    case 3: return launch_thread_bwd<3>(grad_out, inp, grad_inp, batch, num_iters, eps, s);
    case 4: return launch_thread_bwd<4>(grad_out, inp, grad_inp, batch, num_iters, eps, s);
    case 5: return launch_thread_bwd<5>(grad_out, inp, grad_inp, batch, num_iters, eps, s);
    case 6: return launch_thread_bwd<6>(grad_out, inp, grad_inp, batch, num_iters, eps, s);
    case 7: return launch_thread_bwd<7>(grad_out, inp, grad_inp, batch, num_iters, eps, s);
    case 8: return launch_thread_bwd<8>(grad_out, inp, grad_inp, batch, num_iters, eps, s);
    default: {
      const int64_t blocks = (batch + BWD_WARPS - 1) / BWD_WARPS;
      ProfScope _ps("sinkhorn_bwd", s);
      if (n <= 16)
        sk_bwd_warp_kernel<16><<<(unsigned)blocks, BWD_WARPS * 32, 0, s>>>(grad_out, inp, grad_inp, batch, n, num_iters, eps);
      else
        sk_bwd_warp_kernel<32><<<(unsigned)blocks, BWD_WARPS * 32, 0, s>>>(grad_out, inp, grad_inp, batch, n, num_iters, eps);
      return check_launch("sinkhorn_knopp_bwd");
    }
  }
}
