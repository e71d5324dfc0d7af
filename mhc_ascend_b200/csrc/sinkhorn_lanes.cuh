// Sinkhorn-Knopp with one matrix spread over a group of G lanes of a warp
// (G = power of two >= N, lane r of the group holds row r; lanes r >= N hold
// a zero row).  Row sums are lane-local, column sums are butterfly shuffles
// over the group, so one iteration is one row and one column normalisation
// deep instead of N of each.  Same formulation and reverse mode as
// sinkhorn.cuh (row step then column step, A / (sum + eps); exact derivative).
#pragma once

#include <cuda_runtime.h>

namespace mhc {

template <int G, typename T>
__device__ __forceinline__ T group_sum(T v) {
#pragma unroll
  for (int o = 1; o < G; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// One iteration on this lane's row; dr / dc_own (optional) receive this
// row's denominator and the denominator of column r (the column the lane owns).
template <int N, int G, typename T>
__device__ __forceinline__ void skl_step(T (&a)[N], T eps, int r, T* dr, T* dc_own) {
  T s = 0;
#pragma unroll
  for (int j = 0; j < N; ++j) s += a[j];
  const T d = s + eps;
  if (dr) *dr = d;
  if (sizeof(T) == 8) {
    const T inv = T(1) / d;
#pragma unroll
    for (int j = 0; j < N; ++j) a[j] *= inv;
  } else {
#pragma unroll
    for (int j = 0; j < N; ++j) a[j] = a[j] / d;
  }
  T cs[N];
#pragma unroll
  for (int j = 0; j < N; ++j) cs[j] = group_sum<G>(a[j]) + eps;
  T mine = 0;
#pragma unroll
  for (int j = 0; j < N; ++j)
    if (j == r) mine = cs[j];
  if (sizeof(T) == 8) {
    // one reciprocal per lane (its own column), shared over the group
    const T inv_mine = T(1) / mine;
    const int base = (int)(threadIdx.x & 31) & ~(G - 1);
#pragma unroll
    for (int j = 0; j < N; ++j) a[j] *= __shfl_sync(0xffffffffu, inv_mine, base + j);
  } else {
#pragma unroll
    for (int j = 0; j < N; ++j) a[j] = a[j] / cs[j];
  }
  if (dc_own) *dc_own = mine;
}

template <int N, int G, typename T>
__device__ __forceinline__ void skl_forward(T (&a)[N], int iters, T eps, int r) {
  for (int t = 0; t < iters; ++t) skl_step<N, G, T>(a, eps, r, nullptr, nullptr);
}

// g: this lane's row of dL/d(output) on entry, of dL/d(input) on exit; x0:
// this lane's row of the forward input.  All lanes of the warp must call it
// with the same iters (the shuffles span the whole warp).
template <int N, int G, typename T>
__device__ __forceinline__ void skl_backward(const T (&x0)[N], T (&g)[N], int iters, T eps, int r) {
  constexpr int SEG = 32;
  T dr[SEG], dco[SEG];
  const int lane = threadIdx.x & 31, base = lane & ~(G - 1);
  int seg_end = iters;
  while (seg_end > 0) {
    const int seg_start = seg_end > SEG ? seg_end - SEG : 0;
    T z[N];
#pragma unroll
    for (int j = 0; j < N; ++j) z[j] = x0[j];
    for (int t = 0; t < seg_start; ++t) skl_step<N, G, T>(z, eps, r, nullptr, nullptr);
    for (int t = seg_start; t < seg_end; ++t)
      skl_step<N, G, T>(z, eps, r, dr + (t - seg_start), dco + (t - seg_start));
    for (int t = seg_end - 1; t >= seg_start; --t) {
      const T dmine = dco[t - seg_start];
      const T imine = T(1) / dmine;   // this lane's column; shared over the group
      // column step: Z = Y / dc
#pragma unroll
      for (int j = 0; j < N; ++j) {
        const T d = __shfl_sync(0xffffffffu, dmine, base + j);
        const T inv = __shfl_sync(0xffffffffu, imine, base + j);
        const T s = group_sum<G>(g[j] * z[j]);
        g[j] = (g[j] - s) * inv;
        z[j] = z[j] * d;  // now Y_t
      }
      // row step: Y = X / dr
      const T d = dr[t - seg_start];
      T s = 0;
#pragma unroll
      for (int j = 0; j < N; ++j) s += g[j] * z[j];
      const T inv = T(1) / d;
#pragma unroll
      for (int j = 0; j < N; ++j) {
        g[j] = (g[j] - s) * inv;
        z[j] = z[j] * d;  // now Z_{t-1}
      }
    }
    seg_end = seg_start;
  }
}

}  // namespace mhc
