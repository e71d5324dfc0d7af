// Register-resident Sinkhorn-Knopp for one N x N matrix per thread (N <= 8),
// forward and exact reverse mode.  Used by the standalone operator and by the
// fused layer kernels (per-token H_res normalisation).
//
// Forward (reference formulation ops_pytorch_backward.py:24-31): per
// iteration, A[i,:] /= (sum_j A[i,j] + eps), then A[:,j] /= (sum_i A[i,j] + eps).
//
// Reverse mode.  For a row step Y = diag(1/d) X with d_i = sum_j X_ij + eps:
//     dX_ij = (dY_ij - sum_k dY_ik Y_ik) / d_i
// and symmetrically for a column step.  This is the exact derivative of the
// formulation above (what autograd produces), not the Ascend kernel's variant
// (sinkhorn_knopp.cpp:1016-1264 multiplies the row correction by the inverse
// once more).  The intermediate matrices are recovered backwards from the
// stored denominators (Y_t = Z_t * dc_t, Z_{t-1} = Y_t * dr_t), so only 2N
// floats per iteration are kept; iterations are processed in segments of
// SK_SEG so any iteration count works with bounded local memory (the
// reference's history buffer silently caps at 32, sinkhorn_knopp.cpp:821).
#pragma once

#include <cuda_runtime.h>

namespace mhc {

constexpr int SK_SEG = 32;

// One iteration (row step, then column step).  T = float divides like the
// reference formulation (A / (sum + eps)); T = double (backward replays)
// multiplies by the reciprocal.  dr/dc (optional) receive the denominators.
template <int N, typename T>
__device__ __forceinline__ void sk_step(T (&a)[N * N], T eps, T* dr, T* dc) {
#pragma unroll
  for (int i = 0; i < N; ++i) {
    T s = 0;
#pragma unroll
    for (int j = 0; j < N; ++j) s += a[i * N + j];
    const T d = s + eps;
    if (dr) dr[i] = d;
    if (sizeof(T) == 8) {
      const T inv = T(1) / d;
#pragma unroll
      for (int j = 0; j < N; ++j) a[i * N + j] *= inv;
    } else {
#pragma unroll
      for (int j = 0; j < N; ++j) a[i * N + j] = a[i * N + j] / d;
    }
  }
#pragma unroll
  for (int j = 0; j < N; ++j) {
    T s = 0;
#pragma unroll
    for (int i = 0; i < N; ++i) s += a[i * N + j];
    const T d = s + eps;
    if (dc) dc[j] = d;
    if (sizeof(T) == 8) {
      const T inv = T(1) / d;
#pragma unroll
      for (int i = 0; i < N; ++i) a[i * N + j] *= inv;
    } else {
#pragma unroll
      for (int i = 0; i < N; ++i) a[i * N + j] = a[i * N + j] / d;
    }
  }
}

template <int N, typename T>
__device__ __forceinline__ void sk_forward(T (&a)[N * N], int iters, T eps) {
  for (int t = 0; t < iters; ++t) sk_step<N, T>(a, eps, nullptr, nullptr);
}

// g: on entry dL/d(output), on exit dL/d(input).  x0 is the forward input.
template <int N, typename T>
__device__ __forceinline__ void sk_backward(const T (&x0)[N * N], T (&g)[N * N], int iters,
                                            T eps) {
  T dr[SK_SEG * N], dc[SK_SEG * N];
  int seg_end = iters;
  while (seg_end > 0) {
    const int seg_start = seg_end > SK_SEG ? seg_end - SK_SEG : 0;
    T z[N * N];
#pragma unroll
    for (int e = 0; e < N * N; ++e) z[e] = x0[e];
    for (int t = 0; t < seg_start; ++t) sk_step<N, T>(z, eps, nullptr, nullptr);
    for (int t = seg_start; t < seg_end; ++t)
      sk_step<N, T>(z, eps, dr + (t - seg_start) * N, dc + (t - seg_start) * N);
    for (int t = seg_end - 1; t >= seg_start; --t) {
      const T* drt = dr + (t - seg_start) * N;
      const T* dct = dc + (t - seg_start) * N;
      // column step: Z = Y / dc
#pragma unroll
      for (int j = 0; j < N; ++j) {
        const T d = dct[j];
        const T inv = T(1) / d;
        T s = 0;
#pragma unroll
        for (int i = 0; i < N; ++i) s += g[i * N + j] * z[i * N + j];
#pragma unroll
        for (int i = 0; i < N; ++i) {
          g[i * N + j] = (g[i * N + j] - s) * inv;
          z[i * N + j] = z[i * N + j] * d;  // now Y_t
        }
      }
      // row step: Y = X / dr
#pragma unroll
      for (int i = 0; i < N; ++i) {
        const T d = drt[i];
        const T inv = T(1) / d;
        T s = 0;
#pragma unroll
        for (int j = 0; j < N; ++j) s += g[i * N + j] * z[i * N + j];
#pragma unroll
        for (int j = 0; j < N; ++j) {
          g[i * N + j] = (g[i * N + j] - s) * inv;
          z[i * N + j] = z[i * N + j] * d;  // now Z_{t-1}
        }
      }
    }
    seg_end = seg_start;
  }
}

}  // namespace mhc
